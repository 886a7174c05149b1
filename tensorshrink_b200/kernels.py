"""Torch-facing wrappers of the sm_100a kernels.

Drop-in replacement for the reference's `triton_kernels.py` dispatch layer:
`fused_quantized_linear`, `apply_outlier_correction` and `dequantize_weight`
keep the reference signatures (tensorshrink triton_kernels.py:714-739,
948-954, 1114-1126) and argument meanings. Differences, all deliberate:

* Unsupported CUDA inputs raise instead of returning None: there is no
  silent fallback to a slower path. CPU tensors raise too.
* The result is written straight in the compute dtype by the kernel (no fp32
  pool buffer + cast); `return_fp32=True` makes the kernel write fp32.
* Outliers must be row-sorted (QuantLinear guarantees it); the kernel walks
  CSR row offsets (`outlier_row_ptr`, derived from `outlier_row` when not
  given). `outliers_sorted=False` runs the standalone atomic correction pass
  after the GEMM, which is order-independent.
* Every launch goes to `torch.cuda.current_stream()`, so calls are CUDA-graph
  capturable.
"""

from __future__ import annotations

import ctypes as C
import threading
from typing import Dict, List, Optional, Tuple

import torch

from . import _C

SUPPORTED_BITS = (2, 4, 8)
_SUPPORTED_GROUP_SIZES = {64, 128}     # the reference's fused-path set; others run too
SUPPORTED_GROUP_SIZE = 128

_DTYPES = {torch.float16: _C.TS_F16, torch.bfloat16: _C.TS_BF16, torch.float32: _C.TS_F32}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPES[dt]
    except KeyError:
        raise NotImplementedError(f"dtype {dt} is not supported") from None


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*tensors: Optional[torch.Tensor], what: str) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(f"{what}: tensorshrink_b200 runs on CUDA tensors only (got {t.device})")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"{what}: tensors on different devices ({dev} vs {t.device})")
    if dev is None:
        raise RuntimeError(f"{what}: no CUDA tensor given")
    return dev


def _contig(t: Optional[torch.Tensor], name: str) -> Optional[torch.Tensor]:
    if t is not None and not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t


def row_ptr_from_rows(outlier_row: torch.Tensor, rows: int) -> torch.Tensor:
    """CSR offsets [rows+1] of a row-sorted int32 outlier_row table."""
    bounds = torch.arange(rows + 1, device=outlier_row.device, dtype=torch.int32)
    return torch.searchsorted(outlier_row.to(torch.int32), bounds, right=False).to(torch.int32)


def make_qweight(*, packed, scale, gmin, bits, group_size, cols, out_features, n_groups=None,
                 codebook=None, dq_scale_codes=None, dq_scale_meta=None, dq_gmin_codes=None,
                 dq_gmin_meta=None, dq_group_size=0, outlier_row_ptr=None, outlier_row=None,
                 outlier_col=None, outlier_delta=None) -> _C.TsQWeight:
    """Fill a `ts_qweight` from QuantLinear-layout tensors (they must stay
    alive while the struct is used)."""
    if n_groups is None:
        if scale is None:
            raise ValueError("n_groups is required when scale is None")
        n_groups = int(scale.shape[1])
    has_dq = dq_scale_codes is not None
    if has_dq and not (dq_scale_meta is not None and dq_gmin_codes is not None and dq_gmin_meta is not None):
        raise ValueError("dq_scale_codes/dq_scale_meta/dq_gmin_codes/dq_gmin_meta come all or none")
    if not has_dq and (scale is None or gmin is None):
        raise ValueError("scale and gmin are required without double quantization")
    for name, t in (("packed", packed), ("scale", scale), ("gmin", gmin), ("codebook", codebook),
                    ("dq_scale_codes", dq_scale_codes), ("dq_scale_meta", dq_scale_meta),
                    ("dq_gmin_codes", dq_gmin_codes), ("dq_gmin_meta", dq_gmin_meta),
                    ("outlier_row_ptr", outlier_row_ptr), ("outlier_col", outlier_col),
                    ("outlier_delta", outlier_delta)):
        _contig(t, name)
    if codebook is not None and codebook.dtype != torch.float32:
        raise ValueError("codebook must be float32")
    if packed.dtype != torch.uint8:
        raise ValueError("packed must be uint8")
    if scale is not None and (scale.dtype != torch.float16 or gmin.dtype != torch.float16):
        raise ValueError("scale/gmin must be float16")
    q = _C.TsQWeight()
    q.rows = int(out_features)
    q.cols = int(cols)
    q.n_groups = int(n_groups)
    q.padded_cols = int(n_groups) * int(group_size)
    q.packed_row_bytes = int(packed.stride(0)) if packed.dim() == 2 else q.padded_cols * bits // 8
    q.bits = int(bits)
    q.group_size = int(group_size)
    q.packed = _ptr(packed)
    q.scale = _ptr(scale) if not has_dq else None
    q.gmin = _ptr(gmin) if not has_dq else None
    q.dq_scale_codes = _ptr(dq_scale_codes)
    q.dq_scale_meta = _ptr(dq_scale_meta)
    q.dq_gmin_codes = _ptr(dq_gmin_codes)
    q.dq_gmin_meta = _ptr(dq_gmin_meta)
    q.dq_group_size = int(dq_group_size) if has_dq else 0
    q.codebook = _ptr(codebook)
    n = 0 if outlier_delta is None else int(outlier_delta.numel())
    q.n_outliers = n
    if n:
        q.outlier_row_ptr = _ptr(outlier_row_ptr)
        q.outlier_row = _ptr(outlier_row)
        q.outlier_col = _ptr(outlier_col)
        q.outlier_delta = _ptr(outlier_delta)
    return q


# ---------------------------------------------------------------------------
# workspaces
# ---------------------------------------------------------------------------

class _Workspaces:
    """Zero-filled scratch per (device, stream). Buffers are never freed
    while the process runs (a captured CUDA graph may still point at one);
    kernels leave their scratch zeroed again when they finish."""

    def __init__(self):
        self._lock = threading.Lock()
        self._cur: Dict[Tuple[int, int], torch.Tensor] = {}
        self._all: List[torch.Tensor] = []

    def get(self, device: torch.device, nbytes: int) -> torch.Tensor:
        key = (device.index if device.index is not None else torch.cuda.current_device(),
               torch.cuda.current_stream(device).cuda_stream)
        with self._lock:
            buf = self._cur.get(key)
            if buf is None or buf.numel() < nbytes:
                buf = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
                self._cur[key] = buf
                self._all.append(buf)
            return buf


    def on_device(self, index: int) -> List[torch.Tensor]:
        with self._lock:
            return [b for b in self._all if b.device.index == index]


_WORKSPACES = _Workspaces()


def device_status(device: Optional[torch.device] = None, clear: bool = True) -> None:
    """Raise RuntimeError if a bounded wait inside a qlinear kernel ran out
    on `device` since the last check (`ts_qlinear_status` over every cached
    workspace of the device). The call synchronizes the current stream; with
    `clear` the flags and the workspaces' counters are reset, so later calls
    run normally. A timed-out call's outputs are not valid."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    lib = _C.load()
    with torch.cuda.device(dev):
        stream = _stream_handle(dev)
        ops = _C.torch_ops()
        if ops is not None:       # the workspaces of torch.ops.tensorshrink.qlinear
            try:
                ops.device_status(dev.index, clear)
            except RuntimeError as e:
                raise RuntimeError(f"ts_qlinear_status: {e}") from None
        bufs = _WORKSPACES.on_device(dev.index) + [None]   # None: the no-alloc scratch
        for b in bufs:
            if b is None:
                rc = lib.ts_qlinear_status(None, 0, 1 if clear else 0, stream)
            else:
                rc = lib.ts_qlinear_status(b.data_ptr(), int(b.numel()), 1 if clear else 0, stream)
            _C.check(rc, "ts_qlinear_status")


def workspace_for(device: torch.device, nbytes: int) -> torch.Tensor:
    return _WORKSPACES.get(device, nbytes)


# ---------------------------------------------------------------------------
# public kernel entry points
# ---------------------------------------------------------------------------

def qlinear(x2d: torch.Tensor, qw: _C.TsQWeight, bias: Optional[torch.Tensor], out_dtype: torch.dtype,
            out: Optional[torch.Tensor] = None, workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out[M, rows] = x2d @ W^T (+outliers)(+bias) through `ts_qlinear`."""
    lib = _C.load()
    M = int(x2d.shape[0])
    if out is None:
        out = torch.empty((M, qw.rows), dtype=out_dtype, device=x2d.device)
    if M == 0:
        return out
    need = int(lib.ts_qlinear_workspace_size(qw, M))
    if workspace is None or workspace.numel() < need:
        workspace = workspace_for(x2d.device, need)
    rc = lib.ts_qlinear(qw, x2d.data_ptr(), dtype_code(x2d.dtype), M, int(x2d.stride(0)),
                        _ptr(bias), dtype_code(bias.dtype) if bias is not None else 0,
                        out.data_ptr(), dtype_code(out.dtype), int(out.stride(0)),
                        workspace.data_ptr(), int(workspace.numel()), _stream_handle(x2d.device))
    _C.check(rc, "ts_qlinear")
    return out


def qlinear_gated(gate_up: torch.Tensor, qw: _C.TsQWeight, bias: Optional[torch.Tensor], out_dtype: torch.dtype,
                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out[M, rows] = (silu(gate) * up) @ W^T for gate_up = [gate | up]
    ([M, 2 * cols], e.g. a fused gate/up projection's output): one
    `ts_qlinear_gated` launch for decode-sized M (the product is formed while
    the kernel stages its activations); F.silu(gate) * up then `ts_qlinear`
    for larger M."""
    lib = _C.load()
    M, K = int(gate_up.shape[0]), int(qw.cols)
    if gate_up.stride(-1) != 1:
        gate_up = gate_up.contiguous()
    if out is None:
        out = torch.empty((M, qw.rows), dtype=out_dtype, device=gate_up.device)
    if M == 0:
        return out
    workspace = workspace_for(gate_up.device, int(lib.ts_qlinear_workspace_size(qw, M)))
    rc = lib.ts_qlinear_gated(qw, gate_up.data_ptr(), dtype_code(gate_up.dtype), M, int(gate_up.stride(0)),
                              _ptr(bias), dtype_code(bias.dtype) if bias is not None else 0,
                              out.data_ptr(), dtype_code(out.dtype), int(out.stride(0)),
                              workspace.data_ptr(), int(workspace.numel()), _stream_handle(gate_up.device))
    if rc == -2:    # not a decode-sized call: the elementwise product, then the GEMM
        g, u = gate_up[:, :K], gate_up[:, K:2 * K]
        return qlinear((torch.nn.functional.silu(g) * u).contiguous(), qw, bias, out_dtype, out=out)
    _C.check(rc, "ts_qlinear_gated")
    return out


class ChainStep:
    """One layer of `qlinear_chain`: out = W x' (+ bias) (+ residual), with x'
    = x, or silu(gate) * up of x = [gate | up] (`gated`), or
    F.rms_norm(x, norm_weight, norm_eps) of fp32 rows (`norm_weight`),
    rounded to `act_dtype`. `residual` (fp32 [M, rows]) may be `out`."""

    __slots__ = ("qw", "x", "out", "bias", "gated", "norm_weight", "norm_eps", "act_dtype", "residual")

    def __init__(self, qw: _C.TsQWeight, x: torch.Tensor, out: torch.Tensor, bias: Optional[torch.Tensor] = None,
                 gated: bool = False, norm_weight: Optional[torch.Tensor] = None, norm_eps: float = 1e-5,
                 act_dtype: Optional[torch.dtype] = None, residual: Optional[torch.Tensor] = None):
        self.qw, self.x, self.out, self.bias = qw, x, out, bias
        self.gated, self.norm_weight, self.norm_eps = gated, norm_weight, norm_eps
        self.act_dtype = act_dtype if act_dtype is not None else (torch.bfloat16 if x.dtype == torch.float32
                                                                  else x.dtype)
        self.residual = residual

    def to_c(self) -> _C.TsQlinearOp:
        for t, name in ((self.x, "x"), (self.out, "out"), (self.residual, "residual")):
            if t is not None and (t.dim() != 2 or t.stride(-1) != 1):
                raise ValueError(f"chain step {name} must be a 2-D row-major tensor")
        if self.norm_weight is not None and (self.norm_weight.dtype != torch.float32
                                             or not self.norm_weight.is_contiguous()):
            raise ValueError("norm_weight must be a contiguous fp32 tensor")
        if self.residual is not None and self.residual.dtype != torch.float32:
            raise ValueError("residual must be fp32")
        op = _C.TsQlinearOp()
        op.w = C.pointer(self.qw)
        op.x = self.x.data_ptr()
        op.x_row_stride = int(self.x.stride(0))
        op.x_dtype = dtype_code(self.x.dtype)
        op.flags = (_C.OP_GATED if self.gated else 0) | (_C.OP_RMSNORM if self.norm_weight is not None else 0)
        op.bias = _ptr(self.bias)
        op.bias_dtype = dtype_code(self.bias.dtype) if self.bias is not None else 0
        op.out = self.out.data_ptr()
        op.out_dtype = dtype_code(self.out.dtype)
        op.out_row_stride = int(self.out.stride(0))
        op.norm_weight = _ptr(self.norm_weight)
        op.norm_eps = float(self.norm_eps)
        op.act_dtype = dtype_code(self.act_dtype)
        op.residual = _ptr(self.residual)
        op.residual_row_stride = int(self.residual.stride(0)) if self.residual is not None else 0
        return op

    def run_unfused(self) -> None:
        """The same layer from separate torch ops and `qlinear` (calls the
        decode kernel does not take)."""
        x = self.x
        if self.gated:
            K = int(self.qw.cols)
            x = (torch.nn.functional.silu(x[:, :K]) * x[:, K:2 * K]).to(self.act_dtype)
        elif self.norm_weight is not None:
            x = torch.nn.functional.rms_norm(x, (x.shape[-1],), self.norm_weight, self.norm_eps).to(self.act_dtype)
        if self.residual is None:
            qlinear(x.contiguous(), self.qw, self.bias, self.out.dtype, out=self.out)
        else:
            y = qlinear(x.contiguous(), self.qw, self.bias, torch.float32)
            self.out.copy_(self.residual + y)


def qlinear_chain(steps: List[ChainStep], persistent: bool = False) -> None:
    """Run `steps` in order (step i + 1 may read what step i wrote) through
    `ts_qlinear_chain`: decode-sized calls as one decode launch per step, or
    with `persistent` as one launch over every step when the layers share a
    code layout; calls the decode kernel does not take run unfused, step by
    step."""
    if not steps:
        return
    lib = _C.load()
    M = int(steps[0].x.shape[0])
    dev = steps[0].x.device
    if any(int(st.x.shape[0]) != M or int(st.out.shape[0]) != M for st in steps):
        raise ValueError("every chain step must have the same number of rows")
    need = max(int(lib.ts_qlinear_workspace_size(st.qw, M)) for st in steps)
    ws = workspace_for(dev, need)
    arr = (_C.TsQlinearOp * len(steps))(*[st.to_c() for st in steps])
    rc = lib.ts_qlinear_chain(arr, len(steps), M, 1 if persistent else 0, ws.data_ptr(), int(ws.numel()),
                              _stream_handle(dev))
    if rc == -2:      # validated before anything ran: run the layers unfused
        for st in steps:
            st.run_unfused()
        return
    _C.check(rc, "ts_qlinear_chain")


def decode_attention(qkv: torch.Tensor, n_q: int, n_kv: int, head_dim: int, pos: torch.Tensor,
                     rope_cos: torch.Tensor, rope_sin: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     attn_len: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One decode step of grouped-query attention (`ts_decode_attention`):
    ropes the new q/k of `qkv` ([B, (n_q + 2 n_kv) D] bf16) at position
    `pos` (int64 device tensor, one element), writes k/v into this layer's
    caches ([B', n_kv, max_seq, D] bf16, B' >= B) and attends over positions
    < min(attn_len, pos + 1). Returns [B, n_q D] bf16."""
    lib = _C.load()
    B = int(qkv.shape[0])
    if qkv.dtype != torch.bfloat16 or k_cache.dtype != torch.bfloat16 or v_cache.dtype != torch.bfloat16:
        raise ValueError("decode_attention takes bf16 q/k/v and caches")
    if k_cache.stride() != v_cache.stride() or k_cache.stride(-1) != 1 or k_cache.stride(-2) != head_dim:
        raise ValueError("the caches must share a [B, n_kv, max_seq, D] row-major layout")
    if pos.dtype != torch.int64 or rope_cos.dtype != torch.float32 or not rope_cos.is_contiguous() \
            or not rope_sin.is_contiguous():
        raise ValueError("pos must be int64, the rotary tables contiguous fp32")
    if out is None:
        out = torch.empty(B, n_q * head_dim, dtype=torch.bfloat16, device=qkv.device)
    rc = lib.ts_decode_attention(qkv.data_ptr(), int(qkv.stride(0)), B, n_q, n_kv, head_dim, pos.data_ptr(),
                                 rope_cos.data_ptr(), rope_sin.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                                 int(k_cache.stride(0)), int(k_cache.stride(1)), int(attn_len),
                                 int(k_cache.shape[2]), out.data_ptr(), int(out.stride(0)),
                                 _stream_handle(qkv.device))
    _C.check(rc, "ts_decode_attention")
    return out


def fused_quantized_linear(
    x: torch.Tensor,
    packed: torch.Tensor,
    scale: Optional[torch.Tensor],
    gmin: Optional[torch.Tensor],
    bias: Optional[torch.Tensor],
    bits: int,
    group_size: int,
    cols: int,
    out_features: int,
    compute_dtype: torch.dtype,
    return_fp32: bool = False,
    out: Optional[torch.Tensor] = None,
    outlier_row: Optional[torch.Tensor] = None,
    outlier_col: Optional[torch.Tensor] = None,
    outlier_delta: Optional[torch.Tensor] = None,
    outliers_sorted: bool = True,
    use_buffer_pool: bool = True,
    codebook: Optional[torch.Tensor] = None,
    dq_scale_codes: Optional[torch.Tensor] = None,
    dq_scale_meta: Optional[torch.Tensor] = None,
    dq_gmin_codes: Optional[torch.Tensor] = None,
    dq_gmin_meta: Optional[torch.Tensor] = None,
    dq_group_size: int = 0,
    n_groups: Optional[int] = None,
    outlier_row_ptr: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Fused unpack + group-affine dequant + GEMM (+ outlier correction + bias).

    Same contract as tensorshrink triton_kernels.py:714-793 except that it
    never returns None (see the module docstring). `use_buffer_pool` is
    accepted for signature compatibility; outputs come from torch's caching
    allocator (or `out=`, an fp32 [M, out_features] tensor).
    `outlier_row_ptr` (int32 [out_features+1]) may be passed to skip deriving
    the CSR offsets from `outlier_row`.
    """
    del use_buffer_pool
    if bits not in SUPPORTED_BITS:
        raise NotImplementedError(f"bits={bits} has no fused kernel (supported: {SUPPORTED_BITS})")
    if compute_dtype not in (torch.float16, torch.bfloat16):
        raise NotImplementedError("compute_dtype must be float16 or bfloat16")
    dev = _require_cuda(x, packed, scale, gmin, bias, codebook, dq_scale_codes, outlier_row,
                        what="fused_quantized_linear")
    orig_shape = x.shape
    x2d = x.reshape(-1, orig_shape[-1])
    if x2d.dtype != compute_dtype:
        x2d = x2d.to(compute_dtype)
    if not x2d.is_contiguous():
        x2d = x2d.contiguous()
    M = x2d.shape[0]
    N = int(out_features)
    n_out = 0 if outlier_row is None else int(outlier_row.numel())
    fuse = n_out > 0 and outliers_sorted
    if fuse and outlier_row_ptr is None:
        outlier_row_ptr = row_ptr_from_rows(outlier_row, N)
    if bias is not None and bias.dtype not in _DTYPES:
        raise ValueError("bias dtype not supported")
    qw = make_qweight(packed=packed, scale=scale, gmin=gmin, bits=bits, group_size=group_size, cols=cols,
                      out_features=N, n_groups=n_groups, codebook=codebook,
                      dq_scale_codes=dq_scale_codes, dq_scale_meta=dq_scale_meta,
                      dq_gmin_codes=dq_gmin_codes, dq_gmin_meta=dq_gmin_meta,
                      dq_group_size=dq_group_size,
                      outlier_row_ptr=outlier_row_ptr if fuse else None,
                      outlier_row=outlier_row if fuse else None,
                      outlier_col=outlier_col if fuse else None,
                      outlier_delta=outlier_delta if fuse else None)
    want_fp32 = return_fp32 or (n_out > 0 and not outliers_sorted)
    if out is not None and (tuple(out.shape) != (M, N) or out.dtype != torch.float32 or out.device != dev):
        out = None
    res = qlinear(x2d, qw, bias, torch.float32 if want_fp32 else compute_dtype,
                  out=out if want_fp32 else None)
    if n_out > 0 and not outliers_sorted:
        apply_outlier_correction(res, x2d, outlier_row, outlier_col, outlier_delta)
        if not return_fp32:
            res = res.to(compute_dtype)
    return res.reshape(*orig_shape[:-1], N)


def apply_outlier_correction(out: torch.Tensor, x2d: torch.Tensor, outlier_row: torch.Tensor,
                             outlier_col: torch.Tensor, outlier_delta: torch.Tensor) -> torch.Tensor:
    """out[m, row[k]] += x[m, col[k]] * delta[k] in place (fp32 `out`),
    tensorshrink triton_kernels.py:948-991."""
    dev = _require_cuda(out, x2d, outlier_row, what="apply_outlier_correction")
    if out.dtype != torch.float32:
        raise ValueError("apply_outlier_correction needs an fp32 `out`")
    n = int(outlier_row.numel())
    if n == 0:
        return out
    out2d = out.reshape(-1, out.shape[-1])
    if not out2d.is_contiguous():
        raise ValueError("out must be contiguous")
    x2d = x2d.reshape(-1, x2d.shape[-1])
    if not x2d.is_contiguous():
        x2d = x2d.contiguous()
    rc = _C.load().ts_apply_outlier_correction(
        out2d.data_ptr(), out2d.shape[0], out2d.shape[1], int(out2d.stride(0)), x2d.data_ptr(),
        dtype_code(x2d.dtype), int(x2d.stride(0)), outlier_row.data_ptr(),
        _contig(outlier_col, "outlier_col").data_ptr(), _contig(outlier_delta, "outlier_delta").data_ptr(),
        n, _stream_handle(dev))
    _C.check(rc, "ts_apply_outlier_correction")
    return out


def dequantize_weight(
    packed: torch.Tensor,
    scale: Optional[torch.Tensor],
    gmin: Optional[torch.Tensor],
    bits: int,
    rows: int,
    cols: int,
    padded_cols: int,
    n_groups: int,
    group_size: int = SUPPORTED_GROUP_SIZE,
    compute_dtype: torch.dtype = torch.float16,
    codebook: Optional[torch.Tensor] = None,
    dq_scale_codes: Optional[torch.Tensor] = None,
    dq_scale_meta: Optional[torch.Tensor] = None,
    dq_gmin_codes: Optional[torch.Tensor] = None,
    dq_gmin_meta: Optional[torch.Tensor] = None,
    dq_group_size: int = 0,
    outlier_row: Optional[torch.Tensor] = None,
    outlier_col: Optional[torch.Tensor] = None,
    outlier_delta: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Dense W [rows, cols] in `compute_dtype` (tensorshrink
    triton_kernels.py:1114-1186), for 2/4/8-bit and double-quantized
    metadata; with outlier tables the outlier positions hold base + delta."""
    dev = _require_cuda(packed, scale, dq_scale_codes, what="dequantize_weight")
    if padded_cols != n_groups * group_size:
        raise ValueError("padded_cols must equal n_groups * group_size")
    has_out = outlier_row is not None and outlier_row.numel() > 0
    qw = make_qweight(packed=packed, scale=scale, gmin=gmin, bits=bits, group_size=group_size, cols=cols,
                      out_features=rows, n_groups=n_groups, codebook=codebook,
                      dq_scale_codes=dq_scale_codes, dq_scale_meta=dq_scale_meta,
                      dq_gmin_codes=dq_gmin_codes, dq_gmin_meta=dq_gmin_meta, dq_group_size=dq_group_size,
                      outlier_row=outlier_row if has_out else None,
                      outlier_col=outlier_col if has_out else None,
                      outlier_delta=outlier_delta if has_out else None)
    out = torch.empty((rows, cols), dtype=compute_dtype, device=dev)
    rc = _C.load().ts_dequantize_weight(qw, out.data_ptr(), dtype_code(compute_dtype), cols,
                                        1 if has_out else 0, _stream_handle(dev))
    _C.check(rc, "ts_dequantize_weight")
    return out
