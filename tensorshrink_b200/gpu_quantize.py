"""GPU quantization entry points (tensorshrink gpu_quantize.py:52-386),
backed by the hand-written quantize/pack kernel instead of torch ops.

Same signatures and the same codec variant as the reference module: a plain
uniform grid with no double quantization or codebook (the reference's GPU
path supports neither). The full codec, including those, is
`codec.quantize_device` / `codec.quantize_tensor`.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from .codec import (
    DEFAULT_ERROR_THRESHOLD,
    DEFAULT_GROUP_SIZE,
    DEFAULT_OUTLIER_FRAC,
    QuantizedTensor,
    quantize_device,
    quantize_device_adaptive,
)


def quantize_tensor_gpu(w: torch.Tensor, bits: int = 4, group_size: int = DEFAULT_GROUP_SIZE,
                        outlier_frac: float = DEFAULT_OUTLIER_FRAC) -> QuantizedTensor:
    """gpu_quantize.py:52-166: uniform-grid GOAP quantize on the GPU,
    returning a host QuantizedTensor."""
    if bits not in (2, 4, 8):
        raise ValueError("bits must be 2, 4, or 8")
    return quantize_device(w, bits=bits, group_size=group_size,
                           outlier_frac=outlier_frac).to_quantized_tensor()


def quantize_tensor_gpu_adaptive(w: torch.Tensor, group_size: int = DEFAULT_GROUP_SIZE,
                                 outlier_frac: float = DEFAULT_OUTLIER_FRAC,
                                 error_threshold: float = DEFAULT_ERROR_THRESHOLD,
                                 force_bits: Optional[int] = None) -> Tuple[QuantizedTensor, float, bool]:
    """gpu_quantize.py:169-209: 2 -> 4 -> 8 escalation."""
    dq, err, esc = quantize_device_adaptive(w, group_size=group_size, outlier_frac=outlier_frac,
                                            error_threshold=error_threshold, force_bits=force_bits,
                                            allowed_bits=(2, 4, 8))
    return dq.to_quantized_tensor(), err, esc


def quantize_module_gpu(model: torch.nn.Module, device: str = "cuda", bits: int = 4, group_size: int = 128,
                        outlier_frac: float = 0.001, adaptive: bool = False, error_threshold: float = 0.10,
                        min_numel: int = 16384,
                        skip_name_patterns=("norm", "ln_", "embed", "lm_head", "shared", "position"),
                        max_dequant_rows=4096, force_fp32_patterns=(), cache_budget_mb: float = 0.0,
                        host_cache_budget_mb: float = 0.0, fast_dequant: bool = True,
                        use_triton: bool = True, vram_budget_mb: Optional[float] = None,
                        quantize_workers: Optional[int] = None, verbose: bool = True) -> dict:
    """gpu_quantize.py:212-386: quantize every eligible Linear on `device`
    with the uniform grid (no double quantization, no codebook)."""
    from .modules import quantize_module
    with torch.cuda.device(torch.device(device)):
        return quantize_module(model, bits=bits, group_size=group_size, outlier_frac=outlier_frac,
                               adaptive=adaptive, error_threshold=error_threshold, min_numel=min_numel,
                               skip_name_patterns=skip_name_patterns, force_fp32_patterns=force_fp32_patterns,
                               vram_budget_mb=vram_budget_mb, verbose=verbose, companded=False,
                               double_quant=False, nf_quant=False)
