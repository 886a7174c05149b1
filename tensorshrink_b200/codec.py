"""GOAP codec API (tensorshrink codec.py) backed by the sm_100a quantize/pack
and dequantize kernels.

`QuantizedTensor` is field-for-field the reference dataclass
(codec.py:102-188), so objects flow between the two libraries unchanged.
`quantize_tensor` / `dequantize_tensor` keep the reference signatures
(codec.py:453-464, 761) but run on the GPU: a CPU input is copied to the
current CUDA device, and without a CUDA device they raise. Packed codes,
scale/gmin, double-quant codes/meta and outlier indices are bit-identical to
the reference codec (ties at the top-k threshold keep the lowest indices).

`quantize_device` is the device-resident entry: it returns the device
tensors QuantLinear needs (including its row-sorted outlier tables and
deltas) without a host round trip.
"""

from __future__ import annotations

import dataclasses
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

from . import _C
from .kernels import dequantize_weight as _dequantize_weight

DEFAULT_GROUP_SIZE = 128
DEFAULT_OUTLIER_FRAC = 0.001
DEFAULT_ERROR_THRESHOLD = 0.10
DEFAULT_DQ_GROUP_SIZE = 256
DEFAULT_SMOOTH_ALPHA = 0.5
DEFAULT_COMPAND_ITERS = 12
DEFAULT_COMPAND_SAMPLE_CAP = 300_000
_EPS = 1e-8


@dataclasses.dataclass
class QuantizedTensor:
    """One compressed weight tensor, numpy arrays on the host
    (tensorshrink codec.py:102-151)."""

    orig_shape: Tuple[int, ...]
    orig_dtype: str
    bits: int
    group_size: int
    rows: int
    cols: int
    padded_cols: int
    n_groups: int
    packed: np.ndarray
    scale: np.ndarray
    gmin: np.ndarray
    outlier_idx: np.ndarray
    outlier_val: np.ndarray
    dq_scale_codes: Optional[np.ndarray] = None
    dq_scale_meta: Optional[np.ndarray] = None
    dq_gmin_codes: Optional[np.ndarray] = None
    dq_gmin_meta: Optional[np.ndarray] = None
    smooth_scale: Optional[np.ndarray] = None
    stage2_packed: Optional[np.ndarray] = None
    stage2_scale: Optional[np.ndarray] = None
    stage2_gmin: Optional[np.ndarray] = None
    codebook: Optional[np.ndarray] = None

    def n_outliers(self) -> int:
        return int(self.outlier_idx.shape[0])

    def compressed_nbytes(self) -> int:
        """codec.py:156-181."""
        total = self.packed.nbytes + self.outlier_idx.nbytes + self.outlier_val.nbytes
        if self.dq_scale_codes is not None:
            total += self.dq_scale_codes.nbytes + self.dq_scale_meta.nbytes
            total += self.dq_gmin_codes.nbytes + self.dq_gmin_meta.nbytes
        else:
            total += self.scale.nbytes + self.gmin.nbytes
        if self.smooth_scale is not None:
            total += self.smooth_scale.nbytes
        if self.stage2_packed is not None:
            total += self.stage2_packed.nbytes + self.stage2_scale.nbytes + self.stage2_gmin.nbytes
        if self.codebook is not None:
            total += self.codebook.nbytes
        return total

    def orig_nbytes(self) -> int:
        itemsize = {"float16": 2, "bfloat16": 2, "float32": 4}.get(self.orig_dtype, 2)
        n = 1
        for d in self.orig_shape:
            n *= d
        return n * itemsize


# ---------------------------------------------------------------------------
# codebooks
# ---------------------------------------------------------------------------

_NF_CODEBOOKS: Dict[int, np.ndarray] = {}


def _get_nf_codebook(bits: int) -> np.ndarray:
    """Normal-float levels (codec.py:273-317): the centroid
    E[X | X in bin] of each of 2**bits equal-probability N(0,1) bins,
    rescaled to [0, 2**bits - 1]; bin-midpoint quantiles without scipy."""
    if bits not in _NF_CODEBOOKS:
        n = 1 << bits
        try:
            from scipy.stats import norm
            edges = np.linspace(0, 1, n + 1)
            cb = np.zeros(n, dtype=np.float32)
            for i in range(n):
                lo = norm.ppf(max(edges[i], 1e-10))
                hi = norm.ppf(min(edges[i + 1], 1 - 1e-10))
                cb[i] = (norm.pdf(lo) - norm.pdf(hi)) / max(edges[i + 1] - edges[i], 1e-10)
        except ImportError:  # pragma: no cover
            from statistics import NormalDist
            cb = np.array([NormalDist().inv_cdf((i + 0.5) / n) for i in range(n)], dtype=np.float32)
        lo_v, hi_v = cb.min(), cb.max()
        if hi_v > lo_v:
            cb = (cb - lo_v) / (hi_v - lo_v) * (n - 1)
        _NF_CODEBOOKS[bits] = cb.astype(np.float32)
    return _NF_CODEBOOKS[bits]


_NF_DEVICE: Dict[Tuple[int, int], torch.Tensor] = {}


def _nf_codebook_device(bits: int, device: torch.device) -> torch.Tensor:
    key = (bits, device.index if device.index is not None else torch.cuda.current_device())
    t = _NF_DEVICE.get(key)
    if t is None:
        t = torch.from_numpy(_get_nf_codebook(bits)).to(device)
        _NF_DEVICE[key] = t
    return t


# ---------------------------------------------------------------------------
# device quantize
# ---------------------------------------------------------------------------

@dataclasses.dataclass
class DeviceQuant:
    """Output of the GPU quantizer: QuantizedTensor fields plus QuantLinear's
    outlier tables, as device tensors."""

    orig_shape: Tuple[int, ...]
    orig_dtype: str
    bits: int
    group_size: int
    rows: int
    cols: int
    padded_cols: int
    n_groups: int
    packed: torch.Tensor
    scale: torch.Tensor            # fp16, DQ-reconstructed when double-quantized
    gmin: torch.Tensor
    outlier_idx: torch.Tensor      # int32 ascending
    outlier_val: torch.Tensor      # fp16
    outlier_row: torch.Tensor      # int32 (row-sorted: ascending flat index)
    outlier_col: torch.Tensor
    outlier_delta: torch.Tensor    # fp16
    outlier_row_ptr: torch.Tensor  # int32 [rows+1]
    threshold: torch.Tensor        # fp32 [1]
    dq_scale_codes: Optional[torch.Tensor] = None
    dq_scale_meta: Optional[torch.Tensor] = None
    dq_gmin_codes: Optional[torch.Tensor] = None
    dq_gmin_meta: Optional[torch.Tensor] = None
    dq_group_size: int = 0
    codebook_assign: Optional[torch.Tensor] = None  # fp32 levels the codes were assigned against
    codebook_store: Optional[torch.Tensor] = None   # what QuantizedTensor.codebook holds
    smooth_scale: Optional[torch.Tensor] = None     # fp16 [cols] column scales (smooth=True)
    stage2_packed: Optional[torch.Tensor] = None    # 6-bit RVQ: 2-bit residual stage
    stage2_scale: Optional[torch.Tensor] = None
    stage2_gmin: Optional[torch.Tensor] = None

    def to_quantized_tensor(self) -> QuantizedTensor:
        def h(t):
            return None if t is None else t.cpu().numpy()
        return QuantizedTensor(
            orig_shape=tuple(self.orig_shape), orig_dtype=self.orig_dtype, bits=self.bits,
            group_size=self.group_size, rows=self.rows, cols=self.cols,
            padded_cols=self.padded_cols, n_groups=self.n_groups,
            packed=h(self.packed), scale=h(self.scale), gmin=h(self.gmin),
            outlier_idx=h(self.outlier_idx), outlier_val=h(self.outlier_val),
            dq_scale_codes=h(self.dq_scale_codes), dq_scale_meta=h(self.dq_scale_meta),
            dq_gmin_codes=h(self.dq_gmin_codes), dq_gmin_meta=h(self.dq_gmin_meta),
            codebook=h(self.codebook_store), smooth_scale=h(self.smooth_scale),
            stage2_packed=h(self.stage2_packed), stage2_scale=h(self.stage2_scale),
            stage2_gmin=h(self.stage2_gmin))


def n_outliers_for(n_elem: int, outlier_frac: float) -> int:
    """codec.py:530."""
    return max(1, int(n_elem * outlier_frac)) if outlier_frac > 0 else 0


def _as_cuda(w: torch.Tensor) -> torch.Tensor:
    if w.is_cuda:
        return w
    if not torch.cuda.is_available():
        raise RuntimeError("tensorshrink_b200 quantizes on the GPU; no CUDA device is available")
    return w.to(torch.device("cuda", torch.cuda.current_device()))


def quantize_device(w: torch.Tensor, bits: int = 4, group_size: int = DEFAULT_GROUP_SIZE,
                    outlier_frac: float = DEFAULT_OUTLIER_FRAC, double_quant: bool = False,
                    dq_group_size: int = DEFAULT_DQ_GROUP_SIZE, companded: bool = False,
                    nf_quant: bool = False, codebook: Optional[torch.Tensor] = None,
                    lloyd_sample: Optional[torch.Tensor] = None,
                    lloyd_iters: int = DEFAULT_COMPAND_ITERS, smooth: bool = False,
                    smooth_alpha: float = DEFAULT_SMOOTH_ALPHA) -> DeviceQuant:
    """GOAP quantize on the GPU (codec.py:453-675 semantics; bits 2/4/8).

    companded=True fits a Lloyd-Max codebook on the device (codec.py:320-361)
    over every normalized value, or over `DEFAULT_COMPAND_SAMPLE_CAP` values
    drawn with `torch.randperm` on the weight's device when there are more
    (codec.py:329-333). `lloyd_sample` (int64 flat indices into the padded
    [rows, padded_cols] grid) or `codebook` (sorted fp32 levels to assign
    against, skipping the fit) override that.

    smooth=True (codec.py:519-525) divides each column by
    s_j = max(max_i |w_ij|, 1e-8) ** smooth_alpha before quantizing and keeps
    f16(s) as `smooth_scale`; the column maxima come from the device and the
    power is taken by torch on the host, as the reference computes it, so
    the scales (and the codes) are the reference's. bits=6 is the residual
    scheme of codec.py:678-737 (`quantize_rvq_device`).
    """
    if bits == 6:
        if companded:
            raise ValueError("companded=True is not supported with bits=6 (RVQ)")
        return quantize_rvq_device(w, group_size, outlier_frac, double_quant, dq_group_size, smooth, smooth_alpha)
    if bits not in (2, 4, 8):
        raise ValueError("bits must be 2, 4, 6, or 8")
    if w.dim() < 2:
        raise ValueError("quantize_tensor expects a tensor with ndim >= 2")
    w = _as_cuda(w)
    dev = w.device
    orig_shape = tuple(w.shape)
    orig_dtype = str(w.dtype).replace("torch.", "")
    rows = orig_shape[0]
    cols = int(np.prod(orig_shape[1:]))
    w2d = w.detach().reshape(rows, cols)
    if w2d.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        w2d = w2d.to(torch.float32)
    smooth16 = None
    if smooth:
        work = w2d.to(torch.float32)
        col_max = work.abs().amax(dim=0).clamp(min=_EPS)
        s_j = col_max.cpu().pow(smooth_alpha).to(dev)
        w2d = work / s_j.unsqueeze(0)
        smooth16 = s_j.to(torch.float16)
    w2d = w2d.contiguous()
    gs = int(group_size)
    padded_cols = (cols + gs - 1) // gs * gs
    n_groups = padded_cols // gs
    n = rows * cols
    k = n_outliers_for(n, outlier_frac)
    k_eff = k if 0 < k < n else 0
    L = 1 << bits

    p = _C.TsQuantParams()
    p.rows, p.cols, p.bits, p.group_size = rows, cols, bits, gs
    p.k_outliers = k
    p.double_quant = 1 if double_quant else 0
    p.dq_group_size = int(dq_group_size)
    p.lloyd_iters = int(lloyd_iters)
    cb_assign = None
    keep = []
    if companded and codebook is None:
        p.mode = _C.TS_QMODE_LLOYD
        n_fit = rows * padded_cols
        if lloyd_sample is None and n_fit > DEFAULT_COMPAND_SAMPLE_CAP:
            lloyd_sample = torch.randperm(n_fit, device=dev)[:DEFAULT_COMPAND_SAMPLE_CAP]
        if lloyd_sample is not None:
            lloyd_sample = lloyd_sample.to(device=dev, dtype=torch.int64).contiguous()
            keep.append(lloyd_sample)
            p.lloyd_sample = lloyd_sample.data_ptr()
            p.lloyd_n_sample = int(lloyd_sample.numel())
    elif companded or nf_quant or codebook is not None:
        p.mode = _C.TS_QMODE_CODEBOOK
        if codebook is None:
            cb_assign = _nf_codebook_device(bits, dev)
        else:
            cb_assign = codebook.to(device=dev, dtype=torch.float32).contiguous()
        p.codebook = cb_assign.data_ptr()
    else:
        p.mode = _C.TS_QMODE_UNIFORM

    u8, f16, i32 = torch.uint8, torch.float16, torch.int32
    packed = torch.empty((rows, padded_cols * bits // 8), dtype=u8, device=dev)
    scale = torch.empty((rows, n_groups), dtype=f16, device=dev)
    gmin = torch.empty((rows, n_groups), dtype=f16, device=dev)
    idx = torch.empty(k_eff, dtype=i32, device=dev)
    val = torch.empty(k_eff, dtype=f16, device=dev)
    orow = torch.empty(k_eff, dtype=i32, device=dev)
    ocol = torch.empty(k_eff, dtype=i32, device=dev)
    odelta = torch.empty(k_eff, dtype=f16, device=dev)
    optr = torch.empty(rows + 1, dtype=i32, device=dev)
    thr = torch.empty(1, dtype=torch.float32, device=dev)
    dq = {}
    if double_quant:
        n_super = (rows * n_groups + dq_group_size - 1) // dq_group_size
        for nm in ("scale", "gmin"):
            dq[f"dq_{nm}_codes"] = torch.empty(n_super * dq_group_size, dtype=u8, device=dev)
            dq[f"dq_{nm}_meta"] = torch.empty((n_super, 2), dtype=f16, device=dev)
    cb_out = torch.empty(L, dtype=torch.float32, device=dev) if p.mode != _C.TS_QMODE_UNIFORM else None
    cb16 = torch.empty(L, dtype=f16, device=dev) if companded else None

    o = _C.TsQuantOutputs()
    o.packed, o.scale, o.gmin = packed.data_ptr(), scale.data_ptr(), gmin.data_ptr()
    if double_quant:
        o.dq_scale_codes = dq["dq_scale_codes"].data_ptr()
        o.dq_scale_meta = dq["dq_scale_meta"].data_ptr()
        o.dq_gmin_codes = dq["dq_gmin_codes"].data_ptr()
        o.dq_gmin_meta = dq["dq_gmin_meta"].data_ptr()
    if cb_out is not None:
        o.codebook_out = cb_out.data_ptr()
    if cb16 is not None:
        o.codebook_f16 = cb16.data_ptr()
    if k_eff:
        o.outlier_idx, o.outlier_val = idx.data_ptr(), val.data_ptr()
        o.outlier_row, o.outlier_col, o.outlier_delta = orow.data_ptr(), ocol.data_ptr(), odelta.data_ptr()
    o.outlier_row_ptr = optr.data_ptr()
    o.threshold = thr.data_ptr()

    lib = _C.load()
    ws_bytes = int(lib.ts_quantize_workspace_size(p))
    ws = torch.empty(max(ws_bytes, 1), dtype=u8, device=dev)
    from .kernels import dtype_code
    rc = lib.ts_quantize_pack(w2d.data_ptr(), dtype_code(w2d.dtype), p, o, ws.data_ptr(), ws_bytes,
                              torch.cuda.current_stream(dev).cuda_stream)
    _C.check(rc, "ts_quantize_pack")
    del keep

    if p.mode == _C.TS_QMODE_LLOYD:
        cb_assign = cb_out
    cb_store = cb16 if companded else cb_assign   # Lloyd-Max levels are stored in fp16 (codec.py:596)
    return DeviceQuant(
        orig_shape=orig_shape, orig_dtype=orig_dtype, bits=bits, group_size=gs, rows=rows, cols=cols,
        padded_cols=padded_cols, n_groups=n_groups, packed=packed, scale=scale, gmin=gmin,
        outlier_idx=idx, outlier_val=val, outlier_row=orow, outlier_col=ocol, outlier_delta=odelta,
        outlier_row_ptr=optr, threshold=thr, dq_group_size=int(dq_group_size) if double_quant else 0,
        codebook_assign=cb_assign, codebook_store=cb_store, smooth_scale=smooth16, **dq)


def quantize_rvq_device(w: torch.Tensor, group_size: int = DEFAULT_GROUP_SIZE,
                        outlier_frac: float = DEFAULT_OUTLIER_FRAC, double_quant: bool = False,
                        dq_group_size: int = DEFAULT_DQ_GROUP_SIZE, smooth: bool = False,
                        smooth_alpha: float = DEFAULT_SMOOTH_ALPHA) -> DeviceQuant:
    """6-bit residual quantization on the GPU (codec.py:678-737): a 4-bit
    stage with outliers (and double quant / smoothing as asked), then the
    fp32 residual w - W4 quantized at 2 bits without outliers."""
    w = _as_cuda(w)
    d4 = quantize_device(w, bits=4, group_size=group_size, outlier_frac=outlier_frac, double_quant=double_quant,
                         dq_group_size=dq_group_size, smooth=smooth, smooth_alpha=smooth_alpha)
    residual = w.detach().reshape(d4.rows, d4.cols).to(torch.float32) - dequantize_device(d4).reshape(d4.rows, -1)
    d2 = quantize_device(residual, bits=2, group_size=group_size, outlier_frac=0.0)
    d4.bits = 6
    d4.stage2_packed, d4.stage2_scale, d4.stage2_gmin = d2.packed, d2.scale, d2.gmin
    return d4


def quantize_tensor(
    w: torch.Tensor,
    bits: int = 4,
    group_size: int = DEFAULT_GROUP_SIZE,
    outlier_frac: float = DEFAULT_OUTLIER_FRAC,
    double_quant: bool = False,
    dq_group_size: int = DEFAULT_DQ_GROUP_SIZE,
    smooth: bool = False,
    smooth_alpha: float = DEFAULT_SMOOTH_ALPHA,
    companded: bool = False,
    nf_quant: bool = False,
) -> QuantizedTensor:
    """GOAP quantize (codec.py:453-675) on the GPU, returning a host
    QuantizedTensor; smooth scaling and 6-bit RVQ included."""
    if bits == 6 and companded:
        raise ValueError("companded=True is not supported with bits=6 (RVQ)")
    if companded and nf_quant:
        nf_quant = False  # codec.py:582: nf_quant applies only when not companded
    dq = quantize_device(w, bits=bits, group_size=group_size, outlier_frac=outlier_frac,
                         double_quant=double_quant, dq_group_size=dq_group_size,
                         companded=companded, nf_quant=nf_quant, smooth=smooth, smooth_alpha=smooth_alpha)
    return dq.to_quantized_tensor()


# ---------------------------------------------------------------------------
# dequantize
# ---------------------------------------------------------------------------

def _qt_device_tensors(qt: QuantizedTensor, device: torch.device) -> dict:
    t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(device)  # noqa: E731
    d = dict(packed=t(qt.packed), codebook=None)
    if qt.codebook is not None:
        d["codebook"] = t(qt.codebook).to(torch.float32)
    if qt.dq_scale_codes is not None:
        d.update(scale=None, gmin=None, dq_scale_codes=t(qt.dq_scale_codes),
                 dq_scale_meta=t(qt.dq_scale_meta), dq_gmin_codes=t(qt.dq_gmin_codes),
                 dq_gmin_meta=t(qt.dq_gmin_meta),
                 dq_group_size=int(qt.dq_scale_codes.shape[0] // qt.dq_scale_meta.shape[0]))
    else:
        d.update(scale=t(qt.scale), gmin=t(qt.gmin))
    return d


def _reconstruct(bits, rows, cols, padded_cols, n_groups, group_size, packed, scale, gmin, codebook=None,
                 dq_scale_codes=None, dq_scale_meta=None, dq_gmin_codes=None, dq_gmin_meta=None,
                 dq_group_size=0, outlier_idx=None, outlier_val=None, smooth_scale=None, stage2=None):
    """fp32 W [rows, cols] on the device from device tensors: the group-affine
    stage (the 4-bit stage when bits == 6) with exact outlier values, columns
    multiplied back by the smooth scales, plus the 2-bit residual stage of a
    6-bit tensor (codec.py:761-847)."""
    dq = dq_scale_codes is not None
    W = _dequantize_weight(packed, None if dq else scale, None if dq else gmin, 4 if bits == 6 else bits, rows,
                           cols, padded_cols, n_groups, group_size, torch.float32, codebook=codebook,
                           dq_scale_codes=dq_scale_codes, dq_scale_meta=dq_scale_meta,
                           dq_gmin_codes=dq_gmin_codes, dq_gmin_meta=dq_gmin_meta, dq_group_size=dq_group_size)
    if outlier_idx is not None and outlier_idx.numel():
        W.view(-1)[outlier_idx.to(torch.int64)] = outlier_val.to(torch.float32)
    if smooth_scale is not None:
        W = W * smooth_scale.to(torch.float32).unsqueeze(0)
    if bits == 6:
        p2, s2, g2 = stage2
        W = W + _dequantize_weight(p2, s2, g2, 2, rows, cols, padded_cols, n_groups, group_size, torch.float32)
    return W


def dequantize_tensor(qt: QuantizedTensor, device=None, dtype=None) -> torch.Tensor:
    """codec.py:761-847 on the GPU: fp32 reconstruction (double-quant metadata
    in fp32), exact `outlier_val` at outlier positions, smooth scales and the
    6-bit residual stage applied, then cast to `dtype` and moved to `device`
    (default "cpu", as the reference)."""
    device = torch.device(device or "cpu")
    out_dtype = dtype or getattr(torch, qt.orig_dtype, torch.float16)
    gdev = device if device.type == "cuda" else torch.device("cuda", torch.cuda.current_device()) \
        if torch.cuda.is_available() else None
    if gdev is None:
        raise RuntimeError("tensorshrink_b200 dequantizes on the GPU; no CUDA device is available")
    d = _qt_device_tensors(qt, gdev)
    t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(gdev)  # noqa: E731
    stage2 = (t(qt.stage2_packed), t(qt.stage2_scale), t(qt.stage2_gmin)) if qt.bits == 6 else None
    W = _reconstruct(qt.bits, qt.rows, qt.cols, qt.padded_cols, qt.n_groups, qt.group_size, d["packed"],
                     d.get("scale"), d.get("gmin"), d["codebook"], d.get("dq_scale_codes"), d.get("dq_scale_meta"),
                     d.get("dq_gmin_codes"), d.get("dq_gmin_meta"), d.get("dq_group_size", 0),
                     t(qt.outlier_idx.astype(np.int64)), t(qt.outlier_val), t(qt.smooth_scale), stage2)
    return W.reshape(qt.orig_shape).to(device=device, dtype=out_dtype)


def dequantize_device(dq: DeviceQuant, dtype=torch.float32) -> torch.Tensor:
    """Dense reconstruction of a DeviceQuant (exact outlier values)."""
    W = _reconstruct(dq.bits, dq.rows, dq.cols, dq.padded_cols, dq.n_groups, dq.group_size, dq.packed, dq.scale,
                     dq.gmin, None if dq.codebook_store is None else dq.codebook_store.to(torch.float32),
                     dq.dq_scale_codes, dq.dq_scale_meta, dq.dq_gmin_codes, dq.dq_gmin_meta, dq.dq_group_size,
                     dq.outlier_idx, dq.outlier_val, dq.smooth_scale,
                     (dq.stage2_packed, dq.stage2_scale, dq.stage2_gmin) if dq.bits == 6 else None)
    return W.reshape(dq.orig_shape).to(dtype)


def relative_error(w: torch.Tensor, qt) -> float:
    """Relative Frobenius reconstruction error (codec.py:850-857)."""
    if isinstance(qt, DeviceQuant):
        deq = dequantize_device(qt)
        w32 = w.detach().to(device=deq.device, dtype=torch.float32)
    else:
        w32 = _as_cuda(w.detach()).to(torch.float32)
        deq = dequantize_tensor(qt, device=w32.device, dtype=torch.float32)
    num = torch.linalg.norm((w32 - deq).reshape(-1))
    den = torch.linalg.norm(w32.reshape(-1)).clamp(min=_EPS)
    return float((num / den).item())


DEFAULT_ADAPTIVE_BIT_CHAIN: Tuple[int, ...] = (2, 4, 6, 8)


def quantize_tensor_adaptive(
    w: torch.Tensor,
    group_size: int = DEFAULT_GROUP_SIZE,
    outlier_frac: float = DEFAULT_OUTLIER_FRAC,
    error_threshold: float = DEFAULT_ERROR_THRESHOLD,
    force_bits: Optional[int] = None,
    double_quant: bool = False,
    dq_group_size: int = DEFAULT_DQ_GROUP_SIZE,
    smooth: bool = False,
    smooth_alpha: float = DEFAULT_SMOOTH_ALPHA,
    allowed_bits: Sequence[int] = DEFAULT_ADAPTIVE_BIT_CHAIN,
    companded: bool = False,
    nf_quant: bool = False,
) -> Tuple[QuantizedTensor, float, bool]:
    """Lowest bit width whose error is within `error_threshold`
    (codec.py:863-931)."""
    qd, err, esc = quantize_device_adaptive(
        w, group_size=group_size, outlier_frac=outlier_frac, error_threshold=error_threshold,
        force_bits=force_bits, double_quant=double_quant, dq_group_size=dq_group_size,
        smooth=smooth, smooth_alpha=smooth_alpha, allowed_bits=allowed_bits, companded=companded,
        nf_quant=nf_quant)
    return qd.to_quantized_tensor(), err, esc


def quantize_device_adaptive(w, group_size=DEFAULT_GROUP_SIZE, outlier_frac=DEFAULT_OUTLIER_FRAC,
                             error_threshold=DEFAULT_ERROR_THRESHOLD, force_bits=None,
                             double_quant=False, dq_group_size=DEFAULT_DQ_GROUP_SIZE, smooth=False,
                             allowed_bits=DEFAULT_ADAPTIVE_BIT_CHAIN, companded=False, nf_quant=False,
                             smooth_alpha=DEFAULT_SMOOTH_ALPHA):
    """Device-resident variant of quantize_tensor_adaptive."""
    if companded and (force_bits == 6 or 6 in tuple(allowed_bits)):
        raise ValueError("companded=True is not supported with bits=6 (RVQ)")
    kw = dict(group_size=group_size, outlier_frac=outlier_frac, double_quant=double_quant,
              dq_group_size=dq_group_size, companded=companded, nf_quant=nf_quant and not companded,
              smooth=smooth, smooth_alpha=smooth_alpha)
    if force_bits is not None:
        qd = quantize_device(w, bits=force_bits, **kw)
        return qd, relative_error(w, qd), False
    chain = sorted(set(allowed_bits))
    if not chain or any(b not in (2, 4, 6, 8) for b in chain):
        raise ValueError(f"allowed_bits must be a non-empty subset of (2, 4, 6, 8), got {allowed_bits!r}")
    for i, b in enumerate(chain):
        qd = quantize_device(w, bits=b, **kw)
        err = relative_error(w, qd)
        if err <= error_threshold or i == len(chain) - 1:
            return qd, err, i > 0
    raise AssertionError("unreachable")


# ---------------------------------------------------------------------------
# host-side planning (codec.py:934-1033), unchanged semantics
# ---------------------------------------------------------------------------

def estimate_resident_nbytes(qt) -> int:
    """Bytes a QuantLinear built from `qt` keeps resident (codec.py:934-979)."""
    n_out = int(qt.outlier_idx.shape[0])
    total = int(qt.packed.nbytes) + n_out * 10
    if qt.dq_scale_codes is not None:
        total += sum(int(a.nbytes) for a in (qt.dq_scale_codes, qt.dq_scale_meta, qt.dq_gmin_codes,
                                             qt.dq_gmin_meta))
    else:
        total += int(qt.scale.nbytes) + int(qt.gmin.nbytes)
    return total


@dataclasses.dataclass
class LayerBitStats:
    name: str
    bytes4: int
    bytes8: int
    err4: float
    err8: float


def budget_allocate_bits(stats: Sequence[LayerBitStats], budget_bytes: float) -> Dict[str, int]:
    """Bit plan under a byte budget (same plan as tensorshrink codec.py:997-1033).

    All layers start at 4 bits; the budget left over is spent on 8-bit
    upgrades in decreasing order of error removed per extra byte (equal
    ratios keep the order of `stats`), skipping any upgrade that no longer
    fits. Layers whose 8-bit form is not both larger and more accurate are
    never upgraded."""
    plan = {s.name: 4 for s in stats}
    left = budget_bytes - sum(s.bytes4 for s in stats)
    gains = [((s.err4 - s.err8) / (s.bytes8 - s.bytes4), s) for s in stats
             if s.bytes8 > s.bytes4 and s.err4 > s.err8]
    gains.sort(key=lambda g: g[0], reverse=True)   # stable: ties stay in input order
    for _, s in gains:
        extra = s.bytes8 - s.bytes4
        if extra <= left:
            plan[s.name] = 8
            left -= extra
    return plan
