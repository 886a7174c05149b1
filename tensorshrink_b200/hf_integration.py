"""Hugging Face `transformers` quantizer plugin: select tensorshrink with
`from_pretrained(..., quantization_config=TensorShrinkConfig(...))`.

The reference plugin (hf_integration.py:77-465) hooks the transformers 4.x
loader (`create_quantized_param`), which 5.x no longer calls. This one uses
the 5.x contract: `param_needs_quantization` marks the weights of the
eligible nn.Linear layers (the `quantize_module` rule: `min_numel`, skip
patterns, `modules_to_not_convert`), and `get_quantize_ops` returns an op
that the checkpoint loader calls with each such weight as it streams off
disk. The op quantizes it on the GPU (`quantize_device`, or the adaptive
2/4/8 escalation) into a QuantLinear on the target device right away, so no
dense model is ever built on the device. The swap of nn.Linear for
QuantLinear (with the Linear's bias, which loads normally) happens after
loading. Persistence goes through the `.tsk` container
(`save_quant_module` / `load_quantized_module`); `is_serializable` is False,
as in the reference.
"""

from __future__ import annotations

from typing import Any, Dict, Optional, Tuple

import torch
import torch.nn as nn

_INSTALLED = False
METHOD = "tensorshrink"


def _base_classes():
    from transformers.core_model_loading import ConversionOps
    from transformers.quantizers.base import HfQuantizer
    from transformers.utils.quantization_config import QuantizationConfigMixin
    return ConversionOps, HfQuantizer, QuantizationConfigMixin


class TensorShrinkConfig:
    """`quantization_config=` value (reference hf_integration.py:77-196): the
    arguments of `quantize_module`, applied per tensor while loading."""

    def __init__(self, bits: int = 4, group_size: int = 128, outlier_frac: float = 0.001, adaptive: bool = False,
                 error_threshold: float = 0.10, min_numel: Optional[int] = None,
                 skip_name_patterns: Optional[Tuple[str, ...]] = None, force_fp32_patterns: Tuple[str, ...] = (),
                 max_dequant_rows=None, cache_budget_mb: float = 0.0, host_cache_budget_mb: float = 0.0,
                 fast_dequant: bool = True, use_triton: bool = True, vram_budget_mb: Optional[float] = None,
                 quantize_workers: Optional[int] = 4, verbose: bool = True, companded: bool = False,
                 double_quant: bool = True, dq_group_size: Optional[int] = None, nf_quant: bool = True,
                 modules_to_not_convert=None, **kwargs):
        from .codec import DEFAULT_DQ_GROUP_SIZE
        from .modules import DEFAULT_MIN_NUMEL, DEFAULT_SKIP_PATTERNS
        install()
        self.quant_method = METHOD
        self.bits, self.group_size, self.outlier_frac = bits, group_size, outlier_frac
        self.adaptive, self.error_threshold = adaptive, error_threshold
        self.min_numel = DEFAULT_MIN_NUMEL if min_numel is None else min_numel
        self.skip_name_patterns = tuple(DEFAULT_SKIP_PATTERNS if skip_name_patterns is None else skip_name_patterns)
        self.force_fp32_patterns = tuple(force_fp32_patterns)
        self.max_dequant_rows = max_dequant_rows
        self.cache_budget_mb, self.host_cache_budget_mb = cache_budget_mb, host_cache_budget_mb
        self.fast_dequant, self.use_triton = fast_dequant, use_triton
        self.vram_budget_mb = vram_budget_mb
        self.quantize_workers, self.verbose = quantize_workers, verbose
        self.companded, self.double_quant, self.nf_quant = companded, double_quant, nf_quant
        self.dq_group_size = DEFAULT_DQ_GROUP_SIZE if dq_group_size is None else dq_group_size
        self.modules_to_not_convert = list(modules_to_not_convert or [])
        self.post_init()

    def post_init(self):
        if self.bits not in (2, 4, 8):
            raise ValueError(f"TensorShrinkConfig.bits must be 2, 4 or 8, got {self.bits}")
        if self.group_size <= 0:
            raise ValueError(f"TensorShrinkConfig.group_size must be positive, got {self.group_size}")
        if self.vram_budget_mb is not None:
            raise NotImplementedError(
                "TensorShrinkConfig.vram_budget_mb needs every layer's cost before choosing any bit width; "
                "use quantize_module(model, vram_budget_mb=...) on a loaded model instead")

    # -- the QuantizationConfigMixin surface transformers uses --------------------------
    def to_dict(self) -> Dict[str, Any]:
        d = dict(self.__dict__)
        d["skip_name_patterns"] = list(self.skip_name_patterns)
        d["force_fp32_patterns"] = list(self.force_fp32_patterns)
        return d

    def to_diff_dict(self) -> Dict[str, Any]:
        return self.to_dict()

    def to_json_string(self, use_diff: bool = True) -> str:
        import json
        return json.dumps(self.to_dict(), indent=2, sort_keys=True) + "\n"

    def __iter__(self):
        yield from self.to_dict().items()

    def __repr__(self) -> str:
        return f"TensorShrinkConfig {self.to_json_string()}"

    def update(self, **kwargs) -> Dict[str, Any]:
        unused = {}
        for k, v in kwargs.items():
            if hasattr(self, k):
                setattr(self, k, v)
            else:
                unused[k] = v
        return unused

    @classmethod
    def from_dict(cls, config_dict: Dict[str, Any], return_unused_kwargs: bool = False, **kwargs):
        d = dict(config_dict)
        d.pop("quant_method", None)
        cfg = cls(**d)
        unused = cfg.update(**kwargs)
        return (cfg, unused) if return_unused_kwargs else cfg


def _quantize_weight(cfg: TensorShrinkConfig, w: torch.Tensor, device: torch.device):
    """DeviceQuant of one weight, as `quantize_module` would make it."""
    from .codec import quantize_device, quantize_device_adaptive, relative_error
    w = w.to(device)
    kw = dict(group_size=cfg.group_size, outlier_frac=cfg.outlier_frac, double_quant=cfg.double_quant,
              dq_group_size=cfg.dq_group_size, companded=cfg.companded, nf_quant=cfg.nf_quant and not cfg.companded)
    if cfg.adaptive:
        return quantize_device_adaptive(w, error_threshold=cfg.error_threshold, allowed_bits=(2, 4, 8), **kw)
    dq = quantize_device(w, bits=cfg.bits, **kw)
    return dq, relative_error(w, dq), False


def install() -> None:
    """Register the config and quantizer with transformers (once)."""
    global _INSTALLED
    if _INSTALLED:
        return
    ConversionOps, HfQuantizer, QuantizationConfigMixin = _base_classes()
    from transformers.quantizers import auto as auto_mod
    from transformers.quantizers.quantizers_utils import get_module_from_name

    class TensorShrinkQuantize(ConversionOps):
        """Called by the loader with one eligible Linear weight: quantize it
        on the device now, keep the QuantLinear for the swap after loading,
        and return nothing to assign (the dense weight is never stored)."""

        def __init__(self, quantizer):
            self.quantizer = quantizer

        def convert(self, input_dict, model=None, full_layer_name=None, missing_keys=None, **kwargs):
            from .modules import QuantLinear
            value = list(input_dict.values())[0]
            value = value[0] if isinstance(value, list) else value
            q = self.quantizer
            module_name = full_layer_name.rsplit(".", 1)[0]
            dev = q.target_device(module_name, value)
            dq, err, esc = _quantize_weight(q.quantization_config, value, dev)
            force32 = any(p in module_name.lower() for p in q.quantization_config.force_fp32_patterns)
            q.pending[module_name] = (QuantLinear.from_device_quant(dq, force_fp32_compute=force32), err, esc,
                                      value.numel() * value.element_size())
            if missing_keys is not None:
                missing_keys.discard(full_layer_name)
            return {}

    class TensorShrinkHfQuantizer(HfQuantizer):
        requires_calibration = False
        required_packages = None

        def __init__(self, quantization_config, **kwargs):
            super().__init__(quantization_config, **kwargs)
            self.pending: Dict[str, tuple] = {}
            self.targets = set()
            self.device_map = None
            self.stats = {"n_replaced": 0, "orig_bytes": 0, "packed_bytes": 0, "layers": []}

        def validate_environment(self, *args, **kwargs):
            if not torch.cuda.is_available():
                raise RuntimeError("tensorshrink quantizes on a CUDA device; none is available")
            self.device_map = kwargs.get("device_map")

        def target_device(self, module_name: str, value: torch.Tensor) -> torch.device:
            dm = self.device_map
            if isinstance(dm, dict):
                best = None
                for k, v in dm.items():
                    if k == "" or module_name == k or module_name.startswith(k + "."):
                        if best is None or len(k) > len(best[0]):
                            best = (k, v)
                if best is not None and best[1] not in ("cpu", "disk"):
                    v = best[1]
                    return torch.device("cuda", v) if isinstance(v, int) else torch.device(v)
            elif isinstance(dm, (str, torch.device)) and str(dm) not in ("cpu", "auto"):
                d = torch.device(dm)
                return d if d.type == "cuda" else torch.device("cuda", torch.cuda.current_device())
            if value.is_cuda:
                return value.device
            return torch.device("cuda", torch.cuda.current_device())

        def param_needs_quantization(self, model, param_name: str, **kwargs) -> bool:
            return param_name in self.targets

        def get_quantize_ops(self):
            return TensorShrinkQuantize(self)

        def _process_model_before_weight_loading(self, model, **kwargs):
            from .modules import _iter_target_linears
            cfg = self.quantization_config
            skip = tuple(cfg.skip_name_patterns) + tuple(cfg.modules_to_not_convert)
            self.targets = {f"{n}.weight" for n, _ in _iter_target_linears(model, cfg.min_numel, skip)}
            model.config.quantization_config = cfg
            return model

        def _process_model_after_weight_loading(self, model, **kwargs):
            from .modules import _set_module_by_name
            for name, (ql, err, esc, nbytes) in self.pending.items():
                lin = model.get_submodule(name)
                if getattr(lin, "bias", None) is not None:
                    if "bias" in ql.__dict__:
                        del ql.__dict__["bias"]          # the plain `None` attribute of a bias-less layer
                    ql.register_buffer("bias", lin.bias.detach().to(ql.packed.device))
                _set_module_by_name(model, name, ql)
                self.stats["n_replaced"] += 1
                self.stats["orig_bytes"] += nbytes
                self.stats["packed_bytes"] += ql.packed_nbytes()
                self.stats["layers"].append({"name": name, "bits": ql.bits, "rel_error": err, "escalated": esc})
            self.pending.clear()
            model.is_tensorshrink_quantized = True
            model.tensorshrink_stats = self.stats
            if self.quantization_config.verbose and self.stats["orig_bytes"]:
                r = self.stats["orig_bytes"] / max(1, self.stats["packed_bytes"])
                print(f"  tensorshrink: replaced {self.stats['n_replaced']} layers, "
                      f"{self.stats['orig_bytes'] / 1e6:.1f}MB -> {self.stats['packed_bytes'] / 1e6:.1f}MB "
                      f"({r:.2f}x)")
            return model

        def is_serializable(self, safe_serialization=None) -> bool:
            return False

        @property
        def is_trainable(self) -> bool:
            return False

    auto_mod.AUTO_QUANTIZATION_CONFIG_MAPPING[METHOD] = TensorShrinkConfig
    auto_mod.AUTO_QUANTIZER_MAPPING[METHOD] = TensorShrinkHfQuantizer
    globals()["TensorShrinkHfQuantizer"] = TensorShrinkHfQuantizer
    _INSTALLED = True
