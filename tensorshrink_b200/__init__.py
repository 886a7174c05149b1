"""tensorshrink_b200: the tensorshrink QuantLinear hot path on B200 (sm_100a).

Public names follow the reference package (tensorshrink __init__.py:43-66)
for the parts this library implements: the GOAP codec, QuantLinear /
quantize_module, the GPU quantizer and the fused-kernel entry points.
"""

from .codec import (
    QuantizedTensor,
    DeviceQuant,
    quantize_tensor,
    dequantize_tensor,
    quantize_tensor_adaptive,
    quantize_device,
    quantize_device_adaptive,
    dequantize_device,
    relative_error,
)
from .modules import (
    QuantLinear,
    quantize_module,
    DEFAULT_SKIP_PATTERNS,
    T5_EXTRA_SKIP_PATTERNS,
    suggest_max_dequant_rows,
)
from .gpu_quantize import (
    quantize_tensor_gpu,
    quantize_tensor_gpu_adaptive,
    quantize_module_gpu,
)
from .kernels import (
    ChainStep,
    qlinear_chain,
    fused_quantized_linear,
    apply_outlier_correction,
    dequantize_weight,
)

__version__ = "0.1.0"

__all__ = [
    "QuantizedTensor", "DeviceQuant", "quantize_tensor", "dequantize_tensor", "quantize_tensor_adaptive",
    "quantize_device", "quantize_device_adaptive", "dequantize_device", "relative_error", "QuantLinear", "quantize_module", "DEFAULT_SKIP_PATTERNS",
    "T5_EXTRA_SKIP_PATTERNS", "suggest_max_dequant_rows", "quantize_tensor_gpu",
    "quantize_tensor_gpu_adaptive", "quantize_module_gpu", "fused_quantized_linear",
    "apply_outlier_correction", "dequantize_weight", "ChainStep", "qlinear_chain",
]
