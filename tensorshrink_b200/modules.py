"""`QuantLinear` and `quantize_module` backed by the sm_100a kernels.

Drop-in for tensorshrink modules.py:282-1026 and 1258-1455: same constructor
arguments, same registered buffers (names, dtypes, shapes, row-sorted
outlier tables), so reference state_dicts load unchanged. The forward pass is
one `ts_qlinear` call for fp16/bf16 activations at any M (decode GEMV or
prefill GEMM chosen inside the library), with the outlier correction and bias
fused. CUDA tensors always run the sm_100a kernels (a missing library
raises); a layer whose buffers and input are on the CPU runs the reference's
CPU algorithm (chunked dequantize + F.linear, modules.py:752-804, 924-940),
which never touches the GPU path.

Differences from the reference that callers can see:
* `cache`, `use_triton`, `fast_dequant`, `max_dequant_rows` are accepted and
  ignored (no dense-weight cache is needed; there is no Triton).
* One extra non-persistent buffer, `outlier_row_ptr` (int32 [rows+1]), holds
  the CSR row offsets of the row-sorted outlier tables.
* `from_linear` / `quantize_module` quantize on the GPU and build the layer's
  buffers on the device directly.
"""

from __future__ import annotations

from typing import Dict, Iterable, List, Optional, Tuple, Union

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _C, kernels
from .codec import (
    DEFAULT_DQ_GROUP_SIZE,
    DeviceQuant,
    LayerBitStats,
    QuantizedTensor,
    budget_allocate_bits,
    quantize_device,
    quantize_device_adaptive,
    relative_error,
)

DEFAULT_SKIP_PATTERNS = ("norm", "ln_", "embed", "lm_head", "shared", "position")
DEFAULT_MIN_NUMEL = 16384
DEFAULT_MAX_DEQUANT_ROWS = 4096
T5_EXTRA_SKIP_PATTERNS = (".wo",)


def suggest_max_dequant_rows(out_features: int, in_features: int, itemsize: int = 4, device=None,
                             vram_frac: float = 0.02, min_rows: int = 128, max_rows: int = 65536) -> int:
    """modules.py:64-116. Kept for API compatibility; the fused kernels never
    materialise dequantized rows, so the value does not affect them."""
    free = None
    if torch.cuda.is_available():
        try:
            free, _ = torch.cuda.mem_get_info(device or "cuda")
        except Exception:
            free = None
    if free is None:
        return DEFAULT_MAX_DEQUANT_ROWS
    rows = int(free * vram_frac // max(1, in_features * itemsize))
    return max(min_rows, min(rows, max_rows, out_features))


# ---------------------------------------------------------------------------
# host bookkeeping of the outlier tables (construction only)
# ---------------------------------------------------------------------------

def _unpack_codes_at(packed: np.ndarray, bits: int, row: np.ndarray, col: np.ndarray) -> np.ndarray:
    if bits == 4:
        b = packed[row, col // 2]
        return np.where(col % 2 == 1, (b >> 4) & 0xF, b & 0xF).astype(np.int64)
    if bits == 2:
        b = packed[row, col // 4]
        return ((b >> (2 * (col % 4))) & 0x3).astype(np.int64)
    return packed[row, col].astype(np.int64)


def _scale_gmin_f32(qt: QuantizedTensor) -> Tuple[np.ndarray, np.ndarray]:
    """fp32 [rows, n_groups] scale/gmin as QuantLinear._get_scale_gmin builds
    them (modules.py:558-583): DQ reconstruction code*meta_scale+meta_min in
    fp32, not rounded to fp16."""
    n = qt.rows * qt.n_groups
    if qt.dq_scale_codes is not None:
        def rec(codes, meta):
            ns = meta.shape[0]
            c = codes.astype(np.float32).reshape(ns, -1)
            m = meta.astype(np.float32)
            return (c * m[:, 0:1] + m[:, 1:2]).reshape(-1)[:n].reshape(qt.rows, qt.n_groups)
        return rec(qt.dq_scale_codes, qt.dq_scale_meta), rec(qt.dq_gmin_codes, qt.dq_gmin_meta)
    return qt.scale.astype(np.float32), qt.gmin.astype(np.float32)


def host_outlier_tables(qt: QuantizedTensor):
    """(row, col, delta, row_ptr) for a host QuantizedTensor: rows stable-sorted
    (modules.py:414-431), delta = f16(f32(val) - base) (modules.py:649-715)."""
    idx = qt.outlier_idx.astype(np.int64)
    if idx.size == 0:
        z = np.zeros(0, dtype=np.int32)
        return z, z, np.zeros(0, dtype=np.float16), np.zeros(qt.rows + 1, dtype=np.int32)
    row = idx // qt.cols
    col = idx % qt.cols
    perm = np.argsort(row, kind="stable")
    row, col, val = row[perm], col[perm], qt.outlier_val[perm]
    code = _unpack_codes_at(qt.packed, qt.bits, row, col)
    cv = qt.codebook.astype(np.float32)[code] if qt.codebook is not None else code.astype(np.float32)
    s, m = _scale_gmin_f32(qt)
    g = col // qt.group_size
    base = cv * s[row, g] + m[row, g]
    delta = (val.astype(np.float32) - base).astype(np.float16)
    row_ptr = np.searchsorted(row, np.arange(qt.rows + 1), side="left").astype(np.int32)
    return row.astype(np.int32), col.astype(np.int32), delta, row_ptr


# ---------------------------------------------------------------------------
# QuantLinear
# ---------------------------------------------------------------------------

class QuantLinear(nn.Module):
    """nn.Linear replacement whose weight lives as GOAP packed codes
    (tensorshrink modules.py:282-1026)."""

    def __init__(self, qt: Optional[QuantizedTensor], bias: Optional[torch.Tensor] = None,
                 max_dequant_rows: Union[int, str] = DEFAULT_MAX_DEQUANT_ROWS,
                 force_fp32_compute: bool = False, cache=None, fast_dequant: bool = True,
                 use_triton: bool = True, *, _device_quant: Optional[DeviceQuant] = None):
        super().__init__()
        src = qt if qt is not None else _device_quant
        if src is None:
            raise ValueError("QuantLinear needs a QuantizedTensor")
        if len(src.orig_shape) != 2:
            raise ValueError("QuantLinear requires a 2D weight (out_features, in_features)")
        if int(src.bits) == 6 or getattr(src, "smooth_scale", None) is not None:
            # as in the reference (modules.py:963-969): 6-bit RVQ and smooth-scaled
            # tensors are storage formats of the codec, not QuantLinear layouts
            raise ValueError("QuantLinear serves 2/4/8-bit unsmoothed weights; 6-bit RVQ and smooth-scaled "
                             "tensors are codec-level (quantize_tensor / dequantize_tensor)")
        self.out_features, self.in_features = int(src.orig_shape[0]), int(src.orig_shape[1])
        self.bits = int(src.bits)
        self.group_size = int(src.group_size)
        self.rows, self.cols = int(src.rows), int(src.cols)
        self.padded_cols, self.n_groups = int(src.padded_cols), int(src.n_groups)
        self.orig_dtype_str = src.orig_dtype
        self.max_dequant_rows = max_dequant_rows if isinstance(max_dequant_rows, int) else DEFAULT_MAX_DEQUANT_ROWS
        self.force_fp32_compute = force_fp32_compute
        self.cache = cache
        self.fast_dequant = fast_dequant
        self.use_triton = use_triton
        self._qw = None
        self._qw_key = None

        if _device_quant is not None:
            d = _device_quant
            self.register_buffer("packed", d.packed)
            self.double_quant = d.dq_scale_codes is not None
            if self.double_quant:
                self.dq_group_size = int(d.dq_group_size)
                for n in ("dq_scale_codes", "dq_scale_meta", "dq_gmin_codes", "dq_gmin_meta"):
                    self.register_buffer(n, getattr(d, n))
                self.scale = None
                self.gmin = None
            else:
                self.dq_group_size = 0
                self.register_buffer("scale", d.scale)
                self.register_buffer("gmin", d.gmin)
            self.companded = d.codebook_store is not None
            if self.companded:
                self.register_buffer("codebook", d.codebook_store.to(torch.float32))
            else:
                self.codebook = None
            self.register_buffer("outlier_row", d.outlier_row)
            self.register_buffer("outlier_col", d.outlier_col)
            self.register_buffer("outlier_delta", d.outlier_delta)
            self.register_buffer("outlier_row_ptr", d.outlier_row_ptr, persistent=False)
        else:
            t = lambda a: torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
            self.register_buffer("packed", t(qt.packed))
            self.double_quant = qt.dq_scale_codes is not None
            if self.double_quant:
                self.dq_group_size = int(qt.dq_scale_codes.shape[0] // qt.dq_scale_meta.shape[0])
                for n in ("dq_scale_codes", "dq_scale_meta", "dq_gmin_codes", "dq_gmin_meta"):
                    self.register_buffer(n, t(getattr(qt, n)))
                self.scale = None
                self.gmin = None
            else:
                self.dq_group_size = 0
                self.register_buffer("scale", t(qt.scale))
                self.register_buffer("gmin", t(qt.gmin))
            self.companded = qt.codebook is not None
            if self.companded:
                self.register_buffer("codebook", t(qt.codebook).to(torch.float32))
            else:
                self.codebook = None
            row, col, delta, row_ptr = host_outlier_tables(qt)
            self.register_buffer("outlier_row", t(row))
            self.register_buffer("outlier_col", t(col))
            self.register_buffer("outlier_delta", t(delta))
            self.register_buffer("outlier_row_ptr", t(row_ptr), persistent=False)
        if bias is not None:
            self.register_buffer("bias", bias.detach().clone())
        else:
            self.bias = None

    # -- device plumbing ------------------------------------------------------
    def __getstate__(self):
        # the cached ts_qweight holds raw device pointers: never copy or pickle it
        state = super().__getstate__() if hasattr(super(), "__getstate__") else self.__dict__.copy()
        state = dict(state)
        state["_qw"] = None
        state["_qw_key"] = None
        return state

    def _apply(self, fn, recurse=True):
        result = super()._apply(fn, recurse=recurse)
        self._qw = None
        self._qw_key = None
        return result

    def _load_from_state_dict(self, state_dict, prefix, *args, **kwargs):
        super()._load_from_state_dict(state_dict, prefix, *args, **kwargs)
        # outlier_row_ptr is derived, not serialized: rebuild it from the rows
        if self.outlier_row.numel():
            self.outlier_row_ptr = kernels.row_ptr_from_rows(self.outlier_row, self.rows) \
                if self.outlier_row.is_cuda else torch.from_numpy(
                    np.searchsorted(self.outlier_row.numpy(), np.arange(self.rows + 1)).astype(np.int32))
        self._qw = None

    def qweight(self):
        """The `ts_qweight` view of this layer's device buffers (cached)."""
        key = (self.packed.data_ptr(), self.outlier_delta.data_ptr(), self.outlier_row_ptr.data_ptr())
        if self._qw is None or self._qw_key != key:
            self._qw = kernels.make_qweight(
                packed=self.packed, scale=self.scale, gmin=self.gmin, bits=self.bits,
                group_size=self.group_size, cols=self.cols, out_features=self.out_features,
                n_groups=self.n_groups, codebook=self.codebook if self.companded else None,
                dq_scale_codes=getattr(self, "dq_scale_codes", None) if self.double_quant else None,
                dq_scale_meta=getattr(self, "dq_scale_meta", None) if self.double_quant else None,
                dq_gmin_codes=getattr(self, "dq_gmin_codes", None) if self.double_quant else None,
                dq_gmin_meta=getattr(self, "dq_gmin_meta", None) if self.double_quant else None,
                dq_group_size=self.dq_group_size, outlier_row_ptr=self.outlier_row_ptr,
                outlier_row=self.outlier_row, outlier_col=self.outlier_col,
                outlier_delta=self.outlier_delta)
            self._qw_key = key
        return self._qw

    # -- introspection ----------------------------------------------------------
    @property
    def weight(self) -> torch.Tensor:
        """Storage-free int8 'already quantized' sentinel (modules.py:527-541)."""
        return torch.empty(self.out_features, self.in_features, dtype=torch.int8, device="meta")

    def packed_nbytes(self) -> int:
        n = self.packed.numel() * self.packed.element_size()
        if self.double_quant:
            for b in (self.dq_scale_codes, self.dq_scale_meta, self.dq_gmin_codes, self.dq_gmin_meta):
                n += b.numel() * b.element_size()
        else:
            n += self.scale.numel() * self.scale.element_size() + self.gmin.numel() * self.gmin.element_size()
        for b in (self.outlier_row, self.outlier_col, self.outlier_delta):
            n += b.numel() * b.element_size()
        return n

    def dense_equiv_nbytes(self, itemsize: int = 2) -> int:
        return self.out_features * self.in_features * itemsize

    @staticmethod
    def estimate_resident_nbytes(qt) -> int:
        from .codec import estimate_resident_nbytes
        return estimate_resident_nbytes(qt)

    def _scale_gmin_f32(self) -> Tuple[torch.Tensor, torch.Tensor]:
        if not self.double_quant:
            return self.scale.to(torch.float32), self.gmin.to(torch.float32)
        n = self.rows * self.n_groups

        def rec(codes, meta):
            ns = meta.shape[0]
            c = codes.to(torch.float32).reshape(ns, -1)
            m = meta.to(torch.float32)
            return (c * m[:, 0:1] + m[:, 1:2]).reshape(-1)[:n].reshape(self.rows, self.n_groups)
        return rec(self.dq_scale_codes, self.dq_scale_meta), rec(self.dq_gmin_codes, self.dq_gmin_meta)

    def to_quantized_tensor(self) -> QuantizedTensor:
        """Host QuantizedTensor of this layer (modules.py:595-645):
        outlier_val = f16(base + delta)."""
        pk = self.packed.cpu().numpy()
        row = self.outlier_row.cpu().numpy().astype(np.int64)
        col = self.outlier_col.cpu().numpy().astype(np.int64)
        s, m = (a.cpu().numpy() for a in self._scale_gmin_f32())
        if row.size:
            code = _unpack_codes_at(pk, self.bits, row, col)
            cv = self.codebook.cpu().numpy()[code] if self.companded else code.astype(np.float32)
            g = col // self.group_size
            base = cv * s[row, g] + m[row, g]
            val = (base + self.outlier_delta.cpu().numpy().astype(np.float32)).astype(np.float16)
        else:
            val = np.zeros(0, dtype=np.float16)
        kw = dict(orig_shape=(self.out_features, self.in_features), orig_dtype=self.orig_dtype_str,
                  bits=self.bits, group_size=self.group_size, rows=self.rows, cols=self.cols,
                  padded_cols=self.padded_cols, n_groups=self.n_groups, packed=pk,
                  scale=s.astype(np.float16), gmin=m.astype(np.float16),
                  outlier_idx=(row * self.cols + col).astype(np.int32), outlier_val=val)
        if self.double_quant:
            kw.update(dq_scale_codes=self.dq_scale_codes.cpu().numpy(),
                      dq_scale_meta=self.dq_scale_meta.cpu().numpy(),
                      dq_gmin_codes=self.dq_gmin_codes.cpu().numpy(),
                      dq_gmin_meta=self.dq_gmin_meta.cpu().numpy())
        if self.companded:
            kw.update(codebook=self.codebook.cpu().numpy())
        return QuantizedTensor(**kw)

    # -- forward ------------------------------------------------------------------
    def dequantize(self, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """Dense W with outliers (base + delta), as modules.py:903-919 builds."""
        return kernels.dequantize_weight(
            self.packed, self.scale, self.gmin, self.bits, self.rows, self.cols, self.padded_cols,
            self.n_groups, self.group_size, dtype, codebook=self.codebook if self.companded else None,
            dq_scale_codes=getattr(self, "dq_scale_codes", None) if self.double_quant else None,
            dq_scale_meta=getattr(self, "dq_scale_meta", None) if self.double_quant else None,
            dq_gmin_codes=getattr(self, "dq_gmin_codes", None) if self.double_quant else None,
            dq_gmin_meta=getattr(self, "dq_gmin_meta", None) if self.double_quant else None,
            dq_group_size=self.dq_group_size, outlier_row=self.outlier_row,
            outlier_col=self.outlier_col, outlier_delta=self.outlier_delta)

    def _codes_rows(self, r0: int, r1: int) -> torch.Tensor:
        """Integer codes [r1 - r0, padded_cols] of rows [r0, r1) (CPU)."""
        pk = self.packed[r0:r1]
        if self.bits == 8:
            return pk
        per = 8 // self.bits
        shifts = torch.arange(per, dtype=torch.uint8) * self.bits
        mask = (1 << self.bits) - 1
        codes = (pk.unsqueeze(-1) >> shifts) & mask          # code j of byte b at [.., b, j]
        return codes.reshape(r1 - r0, -1)[:, : self.padded_cols]

    def _dequantize_rows_cpu(self, r0: int, r1: int, compute_dtype: torch.dtype) -> torch.Tensor:
        """Rows [r0, r1) of W on the CPU, the reference's chunked dequant
        (modules.py:752-804): codes (or codebook values) * scale + gmin in the
        compute dtype when fast_dequant and the compute dtype is 16-bit, else
        fp32; outlier positions get fp32(base) + delta, rounded once."""
        n = r1 - r0
        calc = compute_dtype if (self.fast_dequant and compute_dtype in (torch.float16, torch.bfloat16)) \
            else torch.float32
        s_full, g_full = self._scale_gmin_f32()
        sc = s_full[r0:r1].to(calc).unsqueeze(-1)
        gm = g_full[r0:r1].to(calc).unsqueeze(-1)
        codes = self._codes_rows(r0, r1).reshape(n, self.n_groups, self.group_size)
        if self.companded:
            vals = self.codebook.to(calc)[codes.long()]
        else:
            vals = codes.to(calc)
        w = (vals * sc + gm).reshape(n, self.padded_cols)[:, : self.cols].contiguous()
        lo = int(self.outlier_row_ptr[r0])
        hi = int(self.outlier_row_ptr[r1])
        if hi > lo:
            flat = w.view(-1)
            idx = (self.outlier_row[lo:hi].long() - r0) * self.cols + self.outlier_col[lo:hi].long()
            base = flat[idx].to(torch.float32)
            flat[idx] = (base + self.outlier_delta[lo:hi].to(torch.float32)).to(calc)
        return w.to(compute_dtype)

    def _forward_cpu(self, x: torch.Tensor) -> torch.Tensor:
        """The reference's CPU forward (modules.py:924-940): dequantize
        `max_dequant_rows` rows at a time and F.linear each chunk."""
        in_dtype = x.dtype
        compute_dtype = torch.float32 if self.force_fp32_compute else in_dtype
        x = x.to(compute_dtype)
        bias = self.bias.to(compute_dtype) if self.bias is not None else None
        step = max(1, int(self.max_dequant_rows))
        outs = []
        for r0 in range(0, self.rows, step):
            r1 = min(r0 + step, self.rows)
            b = bias[r0:r1] if bias is not None else None
            outs.append(F.linear(x, self._dequantize_rows_cpu(r0, r1, compute_dtype), b))
        out = outs[0] if len(outs) == 1 else torch.cat(outs, dim=-1)
        return out.to(in_dtype) if out.dtype != in_dtype else out

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.device.type == "cpu" and self.packed.device.type == "cpu":
            return self._forward_cpu(x)
        if not (x.is_cuda and self.packed.is_cuda):
            raise RuntimeError("QuantLinear: input on {} and weights on {} (both must be on one CUDA "
                               "device, or both on the CPU)".format(x.device, self.packed.device))
        in_dtype = x.dtype
        compute_dtype = torch.float32 if self.force_fp32_compute else in_dtype
        if compute_dtype in (torch.float16, torch.bfloat16):
            ops = _C.torch_ops()
            if ops is not None:
                # one dispatcher call: torch.ops.tensorshrink.qlinear over ts_qlinear
                dq = self.double_quant
                return ops.qlinear(
                    x, self.packed, self.scale, self.gmin,
                    self.dq_scale_codes if dq else None, self.dq_scale_meta if dq else None,
                    self.dq_gmin_codes if dq else None, self.dq_gmin_meta if dq else None,
                    self.codebook if self.companded else None, self.outlier_row_ptr, self.outlier_col,
                    self.outlier_delta, self.bias, self.bits, self.group_size, self.cols, self.out_features,
                    self.n_groups, self.dq_group_size, compute_dtype)
            x2d = x.reshape(-1, self.in_features)
            if not x2d.is_contiguous():
                x2d = x2d.contiguous()
            out = kernels.qlinear(x2d, self.qweight(), self.bias, compute_dtype)
            return out.reshape(*x.shape[:-1], self.out_features)
        # fp32 compute (force_fp32_compute or fp32 activations): dense fp32
        # reconstruction + fp32 matmul, modules.py:819-824 semantics
        w = self.dequantize(torch.float32)
        b = self.bias.to(torch.float32) if self.bias is not None else None
        out = F.linear(x.to(torch.float32), w, b)
        return out.to(in_dtype) if out.dtype != in_dtype else out

    # -- construction helpers ----------------------------------------------------------
    @classmethod
    def from_device_quant(cls, dq: DeviceQuant, bias: Optional[torch.Tensor] = None,
                          force_fp32_compute: bool = False) -> "QuantLinear":
        return cls(None, bias, force_fp32_compute=force_fp32_compute, _device_quant=dq)

    @classmethod
    def from_quantized_tensor(cls, qt: QuantizedTensor, bias: Optional[torch.Tensor] = None,
                              max_dequant_rows=DEFAULT_MAX_DEQUANT_ROWS, force_fp32_compute: bool = False,
                              cache=None, fast_dequant: bool = True, use_triton: bool = True) -> "QuantLinear":
        return cls(qt, bias, max_dequant_rows=max_dequant_rows, force_fp32_compute=force_fp32_compute,
                   cache=cache, fast_dequant=fast_dequant, use_triton=use_triton)

    @classmethod
    def from_linear(cls, linear: nn.Linear, bits: int = 4, group_size: int = 128,
                    outlier_frac: float = 0.001, adaptive: bool = False, error_threshold: float = 0.10,
                    max_dequant_rows=DEFAULT_MAX_DEQUANT_ROWS, force_fp32_compute: bool = False,
                    cache=None, fast_dequant: bool = True, use_triton: bool = True,
                    companded: bool = False, double_quant: bool = True,
                    dq_group_size: int = DEFAULT_DQ_GROUP_SIZE, nf_quant: bool = True,
                    ) -> Tuple["QuantLinear", float, bool]:
        """Quantize `linear.weight` on the GPU (modules.py:943-1003) and build
        the layer on the device; the layer ends up on `linear`'s device."""
        w = linear.weight.data
        kw = dict(group_size=group_size, outlier_frac=outlier_frac, double_quant=double_quant,
                  dq_group_size=dq_group_size, companded=companded, nf_quant=nf_quant and not companded)
        if adaptive:
            dq, err, esc = quantize_device_adaptive(w, error_threshold=error_threshold,
                                                    allowed_bits=(2, 4, 8), **kw)
        else:
            dq = quantize_device(w, bits=bits, **kw)
            err, esc = relative_error(w, dq), False
        bias = linear.bias.data if linear.bias is not None else None
        if bias is not None:
            bias = bias.to(dq.packed.device)
        ql = cls.from_device_quant(dq, bias, force_fp32_compute=force_fp32_compute)
        if w.device != dq.packed.device:
            ql = ql.to(w.device)
        return ql, err, esc

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bits={self.bits}, group_size={self.group_size}, "
                f"packed_kB={self.packed_nbytes() / 1024:.1f}, "
                f"dense_fp16_kB={self.dense_equiv_nbytes() / 1024:.1f}")


# ---------------------------------------------------------------------------
# whole-model helpers (modules.py:1033-1455)
# ---------------------------------------------------------------------------

def _set_module_by_name(root: nn.Module, dotted_name: str, new_module: nn.Module) -> None:
    """Replace the submodule at `dotted_name` (e.g. "layers.3.mlp.up_proj")."""
    parent_name, _, leaf = dotted_name.rpartition(".")
    parent = root.get_submodule(parent_name) if parent_name else root
    setattr(parent, leaf, new_module)


def _iter_target_linears(model: nn.Module, min_numel: int, skip_name_patterns: Iterable[str]):
    """(name, nn.Linear) pairs to quantize: plain Linear layers (not already
    QuantLinear) with at least `min_numel` weights whose lower-cased name
    contains none of the skip patterns (modules.py:1033-1051)."""
    skip = [p.lower() for p in skip_name_patterns]

    def eligible(name: str, mod: nn.Module) -> bool:
        if type(mod) is QuantLinear or not isinstance(mod, nn.Linear):
            return False
        lname = name.lower()
        return mod.weight.numel() >= min_numel and not any(p in lname for p in skip)

    return [(n, m) for n, m in model.named_modules() if eligible(n, m)]


def model_weight_bytes(model: nn.Module) -> int:
    total = sum(p.numel() * p.element_size() for p in model.parameters(recurse=True))
    return total + sum(b.numel() * b.element_size() for b in model.buffers(recurse=True))


def _resident_nbytes(dq: DeviceQuant) -> int:
    n = dq.packed.numel() + dq.outlier_idx.numel() * 10
    if dq.dq_scale_codes is not None:
        n += sum(t.numel() * t.element_size() for t in (dq.dq_scale_codes, dq.dq_scale_meta,
                                                        dq.dq_gmin_codes, dq.dq_gmin_meta))
    else:
        n += 2 * dq.scale.numel() * 2
    return int(n)


def quantize_module(
    model: nn.Module,
    bits: int = 4,
    group_size: int = 128,
    outlier_frac: float = 0.001,
    adaptive: bool = False,
    error_threshold: float = 0.10,
    min_numel: int = DEFAULT_MIN_NUMEL,
    skip_name_patterns: Iterable[str] = DEFAULT_SKIP_PATTERNS,
    max_dequant_rows=DEFAULT_MAX_DEQUANT_ROWS,
    force_fp32_patterns: Iterable[str] = (),
    cache_budget_mb: float = 0.0,
    host_cache_budget_mb: float = 0.0,
    fast_dequant: bool = True,
    use_triton: bool = True,
    vram_budget_mb: Optional[float] = None,
    quantize_workers: Optional[int] = 4,
    verbose: bool = True,
    companded: bool = False,
    double_quant: bool = True,
    dq_group_size: int = DEFAULT_DQ_GROUP_SIZE,
    nf_quant: bool = True,
) -> dict:
    """Swap every eligible nn.Linear of `model` for a QuantLinear, in place
    (modules.py:1258-1455). Layers are quantized one at a time on the GPU
    (`quantize_workers` is accepted and ignored); the stats dict has the
    reference's keys."""
    targets = list(_iter_target_linears(model, min_numel, skip_name_patterns))
    fp32_pats = tuple(p.lower() for p in force_fp32_patterns)
    stats = {"n_replaced": 0, "orig_bytes": 0, "packed_bytes": 0, "layers": [], "cache": None}
    kw = dict(group_size=group_size, outlier_frac=outlier_frac, double_quant=double_quant,
              dq_group_size=dq_group_size, companded=companded, nf_quant=nf_quant and not companded)

    plan: Dict[str, int] = {}
    if vram_budget_mb is not None:
        if companded:
            raise ValueError("companded=True is not yet supported with vram_budget_mb (budget-aware path)")
        layer_stats: List[LayerBitStats] = []
        for name, lin in targets:
            q4 = quantize_device(lin.weight.data, bits=4, **kw)
            q8 = quantize_device(lin.weight.data, bits=8, **kw)
            layer_stats.append(LayerBitStats(name, _resident_nbytes(q4), _resident_nbytes(q8),
                                             relative_error(lin.weight.data, q4),
                                             relative_error(lin.weight.data, q8)))
            del q4, q8
        plan = budget_allocate_bits(layer_stats, vram_budget_mb * 1024 * 1024)

    for i, (name, lin) in enumerate(targets):
        force_fp32 = any(p in name.lower() for p in fp32_pats)
        w = lin.weight.data
        if vram_budget_mb is not None:
            dq = quantize_device(w, bits=plan[name], **kw)
            err, esc = relative_error(w, dq), plan[name] == 8
        elif adaptive:
            dq, err, esc = quantize_device_adaptive(w, error_threshold=error_threshold,
                                                    allowed_bits=(2, 4, 8), **kw)
        else:
            dq = quantize_device(w, bits=bits, **kw)
            err, esc = relative_error(w, dq), False
        bias = lin.bias.data.to(dq.packed.device) if lin.bias is not None else None
        ql = QuantLinear.from_device_quant(dq, bias, force_fp32_compute=force_fp32)
        if w.device != dq.packed.device:
            ql = ql.to(w.device)
        _set_module_by_name(model, name, ql)
        targets[i] = None
        orig_bytes = ql.dense_equiv_nbytes(itemsize=w.element_size())
        packed_bytes = ql.packed_nbytes()
        stats["n_replaced"] += 1
        stats["orig_bytes"] += orig_bytes
        stats["packed_bytes"] += packed_bytes
        stats["layers"].append({"name": name, "bits": ql.bits, "rel_error": err, "escalated": esc,
                                "orig_bytes": orig_bytes, "packed_bytes": packed_bytes,
                                "force_fp32_compute": force_fp32})
        if verbose:
            flag = "*" if esc else " "
            print(f"  [{ql.bits}b{flag}{' fp32' if force_fp32 else ''}] {name:60s} err={err:.4f} "
                  f"{orig_bytes / 1e6:8.3f}MB -> {packed_bytes / 1e6:8.3f}MB")
    stats["ratio"] = stats["orig_bytes"] / max(1, stats["packed_bytes"]) if stats["orig_bytes"] else 1.0
    if vram_budget_mb is not None:
        stats["vram_budget_mb"] = vram_budget_mb
    return stats
