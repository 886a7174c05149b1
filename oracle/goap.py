"""numpy restatement of tensorshrink's GOAP codec and QuantLinear math.

TEST INFRASTRUCTURE ONLY (see `oracle/__init__.py`): the checker the CUDA
kernels are compared against, never imported by the product package.

Every function cites the reference lines it restates (paths are relative to
the tensorshrink repository root). Floating-point steps are written in the
reference's order with float32 operands so that every rounding happens where
the reference's does: codes, packed bytes, double-quant codes/meta and outlier
deltas come out bit-identical to the reference on the same input.

The one deliberate difference is the top-k tie rule (`codec.py:530-534`): when
several elements tie at the threshold magnitude, `torch.topk` picks an
unspecified subset; this oracle (and the CUDA kernel) keep the lowest flat
indices. Tied elements are clamped to +-threshold either way, so codes do not
depend on the choice.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, Optional, Tuple

import numpy as np

F32 = np.float32
EPS = F32(1e-8)                     # codec.py:99 `_EPS`, compared in float32
DQ_EPS = F32(1e-8)                  # codec.py:397 np.maximum(meta_scale, 1e-8)


# ---------------------------------------------------------------------------
# codebooks
# ---------------------------------------------------------------------------

_NF_CACHE: Dict[int, np.ndarray] = {}


def nf_codebook(bits: int) -> np.ndarray:
    """Normal-float codebook, codec.py:273-317.

    Entry i is E[X | X in bin i] for 2**bits equal-probability bins of N(0,1),
    i.e. (pdf(ppf(a)) - pdf(ppf(b))) / (b - a), then rescaled linearly to
    [0, 2**bits - 1]. With scipy absent the reference uses the erfinv
    bin-midpoint approximation instead (codec.py:303-316); so does this.
    """
    if bits in _NF_CACHE:
        return _NF_CACHE[bits]
    n = 1 << bits
    try:
        from scipy.stats import norm
        bounds = np.linspace(0, 1, n + 1)
        cb = np.zeros(n, dtype=np.float32)
        for i in range(n):
            a, b = bounds[i], bounds[i + 1]
            qa = norm.ppf(max(a, 1e-10))
            qb = norm.ppf(min(b, 1 - 1e-10))
            cb[i] = (norm.pdf(qa) - norm.pdf(qb)) / max(b - a, 1e-10)
        lo, hi = cb.min(), cb.max()
        if hi > lo:
            cb = (cb - lo) / (hi - lo) * (n - 1)
        cb = cb.astype(np.float32)
    except ImportError:  # pragma: no cover - scipy is in the image
        # bin-midpoint quantiles sqrt(2)*erfinv(2p-1) of codec.py:303-316
        from statistics import NormalDist
        cb = np.array([NormalDist().inv_cdf((i + 0.5) / n) for i in range(n)],
                      dtype=np.float32)
        lo, hi = cb.min(), cb.max()
        if hi > lo:
            cb = (cb - lo) / (hi - lo) * (n - 1)
    _NF_CACHE[bits] = cb
    return cb


def _torch_linspace_f32(start: float, end: float, steps: int) -> np.ndarray:
    """float32 linspace computed the way ATen's CPU kernel does (symmetric
    halves: start + i*step below the midpoint, end - (steps-1-i)*step above)."""
    out = np.empty(steps, dtype=np.float32)
    if steps == 1:
        out[0] = F32(start)
        return out
    s, e = F32(start), F32(end)
    step = (e - s) / F32(steps - 1)
    half = steps // 2
    for i in range(steps):
        if i < half:
            out[i] = s + step * F32(i)
        else:
            out[i] = e - step * F32(steps - i - 1)
    return out


def lloyd_fit(fit_vals: np.ndarray, n_levels: int, iters: int = 12) -> np.ndarray:
    """1-D Lloyd-Max fit, codec.py:320-361, on an already-drawn sample.

    The reference draws the sample with `torch.randperm` when there are more
    than 300,000 values (codec.py:329-333); callers pass the sample they want
    fitted. Sums are accumulated sequentially in float32 (np.add.at), which
    is what `index_add_` does on CPU.
    """
    fit_vals = np.ascontiguousarray(fit_vals, dtype=np.float32).reshape(-1)
    m = fit_vals.shape[0]
    n_levels = max(1, min(n_levels, m))
    cent = _torch_linspace_f32(float(fit_vals.min()), float(fit_vals.max()), n_levels)
    for _ in range(iters):
        order = np.argsort(cent, kind="stable")
        cs = cent[order]
        if n_levels > 1:
            mids = (cs[:-1] + cs[1:]) / F32(2)
            assign_sorted = np.searchsorted(mids, fit_vals, side="left")
        else:
            assign_sorted = np.zeros(m, dtype=np.int64)
        assign = order[assign_sorted]
        newc = np.zeros(n_levels, dtype=np.float32)
        cnt = np.zeros(n_levels, dtype=np.float32)
        np.add.at(newc, assign, fit_vals)
        np.add.at(cnt, assign, F32(1))
        empty = cnt == 0
        cnt = np.maximum(cnt, F32(1))
        newc = newc / cnt
        newc[empty] = cent[empty]
        cent = newc
    return np.sort(cent).astype(np.float32)


def codebook_mids(cb: np.ndarray) -> np.ndarray:
    """Decision boundaries of nearest-entry assignment, codec.py:370."""
    cb = cb.astype(np.float32)
    return (cb[:-1] + cb[1:]) / F32(2)


def companded_assign(v: np.ndarray, cb: np.ndarray) -> np.ndarray:
    """codec.py:364-373: searchsorted(mids, v) (left side), clamped."""
    k = cb.shape[0]
    if k <= 1:
        return np.zeros(v.shape, dtype=np.int64)
    return np.clip(np.searchsorted(codebook_mids(cb), v, side="left"), 0, k - 1)


# ---------------------------------------------------------------------------
# bit packing, codec.py:195-240
# ---------------------------------------------------------------------------

def pack_codes(codes: np.ndarray, bits: int) -> np.ndarray:
    """codes uint8 [rows, padded_cols] -> packed bytes (codec.py:612-634)."""
    rows, pc = codes.shape
    if bits == 2:
        extra = (-pc) % 4
        if extra:
            codes = np.concatenate([codes, np.repeat(codes[:, -1:], extra, axis=1)], axis=1)
        c = codes.astype(np.uint8)
        return (c[:, 0::4] | (c[:, 1::4] << 2) | (c[:, 2::4] << 4) | (c[:, 3::4] << 6)).astype(np.uint8)
    if bits == 4:
        if pc % 2:
            codes = np.concatenate([codes, codes[:, -1:]], axis=1)
        c = codes.astype(np.uint8)
        return (c[:, 0::2] | (c[:, 1::2] << 4)).astype(np.uint8)
    return np.ascontiguousarray(codes.astype(np.uint8))


def unpack_codes(packed: np.ndarray, bits: int, n: int) -> np.ndarray:
    """Inverse of pack_codes (codec.py:205-240), sliced to n columns."""
    if bits == 2:
        out = np.empty((packed.shape[0], packed.shape[1] * 4), dtype=np.uint8)
        for j in range(4):
            out[:, j::4] = (packed >> (2 * j)) & 0x3
        return out[:, :n]
    if bits == 4:
        out = np.empty((packed.shape[0], packed.shape[1] * 2), dtype=np.uint8)
        out[:, 0::2] = packed & 0xF
        out[:, 1::2] = (packed >> 4) & 0xF
        return out[:, :n]
    return packed[:, :n]


# ---------------------------------------------------------------------------
# double quantization, codec.py:380-435
# ---------------------------------------------------------------------------

def double_quantize(values_f16: np.ndarray, dq_group_size: int) -> Tuple[np.ndarray, np.ndarray]:
    """codec.py:380-401 -> (codes uint8 [n_super*dq_gs], meta fp16 [n_super, 2])."""
    flat = values_f16.astype(np.float32).ravel()
    pad = (-flat.shape[0]) % dq_group_size
    if pad:
        flat = np.concatenate([flat, np.full(pad, flat[-1], dtype=np.float32)])
    g = flat.reshape(-1, dq_group_size)
    mn = g.min(axis=1)
    mx = g.max(axis=1)
    ms = (mx - mn) / F32(255.0)
    ms = np.maximum(ms, DQ_EPS)
    codes = np.round((g - mn[:, None]) / ms[:, None])
    codes = codes.clip(0, 255).astype(np.uint8)
    meta = np.stack([ms, mn], axis=1).astype(np.float16)
    return codes.ravel(), meta


def double_dequantize_f32(codes: np.ndarray, meta: np.ndarray, n: int) -> np.ndarray:
    """fp32 reconstruction used by dequantize_tensor and QuantLinear
    (codec.py:420-435, modules.py:573-580): code*meta_scale + meta_min."""
    n_super = meta.shape[0]
    c = codes.astype(np.float32).reshape(n_super, -1)
    m = meta.astype(np.float32)
    rec = c * m[:, 0:1] + m[:, 1:2]
    return rec.reshape(-1)[:n]


def double_dequantize_f16(codes: np.ndarray, meta: np.ndarray, n: int) -> np.ndarray:
    """codec.py:404-417 (the fp16 `qt.scale`/`qt.gmin` stored after DQ)."""
    return double_dequantize_f32(codes, meta, n).astype(np.float16)


# ---------------------------------------------------------------------------
# quantize, codec.py:453-675
# ---------------------------------------------------------------------------

@dataclass
class QT:
    """Field-for-field mirror of codec.QuantizedTensor (codec.py:102-151)."""
    rows: int
    cols: int
    bits: int
    group_size: int
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
    codebook: Optional[np.ndarray] = None
    smooth_scale: Optional[np.ndarray] = None
    stage2_packed: Optional[np.ndarray] = None
    stage2_scale: Optional[np.ndarray] = None
    stage2_gmin: Optional[np.ndarray] = None
    # by-products the CUDA quantizer also returns (not QuantizedTensor fields)
    codes: Optional[np.ndarray] = field(default=None, repr=False)
    threshold: Optional[float] = None
    assign_codebook_f32: Optional[np.ndarray] = field(default=None, repr=False)


def n_outliers_for(n_elem: int, outlier_frac: float) -> int:
    """codec.py:530: k = max(1, int(n*frac)) if frac > 0 else 0."""
    return max(1, int(n_elem * outlier_frac)) if outlier_frac > 0 else 0


def topk_outliers(flat: np.ndarray, k: int) -> Tuple[np.ndarray, Optional[np.float32]]:
    """Top-k by |w| (codec.py:532-543) with the lowest-index tie rule.
    Returns (indices ascending, threshold) or (empty, None) when no clipping."""
    n = flat.shape[0]
    if not (0 < k < n):
        return np.zeros(0, dtype=np.int64), None
    a = np.abs(flat)
    thr = np.partition(a, n - k)[n - k]
    gt = np.flatnonzero(a > thr)
    need = k - gt.shape[0]
    eq = np.flatnonzero(a == thr)[:need]
    idx = np.sort(np.concatenate([gt, eq]))
    return idx.astype(np.int64), F32(thr)


def smooth_scales(work: np.ndarray, alpha: float) -> np.ndarray:
    """codec.py:519-523: s_j = max(max_i |w_ij|, 1e-8) ** alpha in float32."""
    col_max = np.maximum(np.abs(work).max(axis=0), EPS)
    return np.power(col_max, F32(alpha)).astype(np.float32)


def quantize(w: np.ndarray, bits: int = 4, group_size: int = 128, outlier_frac: float = 0.001,
             double_quant: bool = False, dq_group_size: int = 256, mode: str = "uniform",
             codebook: Optional[np.ndarray] = None, lloyd_sample: Optional[np.ndarray] = None,
             smooth: bool = False, smooth_alpha: float = 0.5) -> QT:
    """GOAP quantize (codec.py:453-675) of a 2-D array.

    mode: "uniform" (round-half-even grid), "nf" (nf_quant=True) or "lloyd"
    (companded=True). For "lloyd" pass either `codebook` (the float32 levels
    to assign against, e.g. the reference's own fit) or `lloyd_sample`
    (flat indices of the normalized values to fit on; all of them when the
    tensor has at most 300,000 elements, as the reference does).
    """
    if bits == 6:
        return quantize_rvq(w, group_size, outlier_frac, double_quant, dq_group_size, smooth, smooth_alpha)
    if bits not in (2, 4, 8):
        raise ValueError("bits must be 2, 4, 6 or 8")
    w = np.asarray(w)
    rows, cols = w.shape
    work2 = w.astype(np.float32)                                    # codec.py:517
    s_smooth = None
    if smooth:                                                       # codec.py:519-525
        s_smooth = smooth_scales(work2, smooth_alpha)
        work2 = work2 / s_smooth[None, :]
    work = work2.reshape(-1).copy()
    k = n_outliers_for(work.shape[0], outlier_frac)
    idx, thr = topk_outliers(work, k)
    if thr is not None:
        vals = work[idx].copy()
        np.clip(work, -thr, thr, out=work)                           # codec.py:543
    else:
        vals = np.zeros(0, dtype=np.float32)
    clipped = work.reshape(rows, cols)
    pad = (-cols) % group_size                                       # codec.py:555-562
    padded = np.concatenate([clipped, np.repeat(clipped[:, -1:], pad, axis=1)], axis=1) if pad else clipped
    padded_cols = cols + pad
    n_groups = padded_cols // group_size
    g = padded.reshape(rows, n_groups, group_size)
    gmin = g.min(axis=-1)                                            # codec.py:567-571
    gmax = g.max(axis=-1)
    levels = (1 << bits) - 1
    scale = (gmax - gmin) / F32(levels)
    scale = np.maximum(scale, EPS)
    v = (g - gmin[..., None]) / scale[..., None]                    # codec.py:579-580
    cb_store = None
    cb_assign = None
    if mode == "nf":                                                 # codec.py:582-590
        cb_assign = nf_codebook(bits)
        codes = companded_assign(v, cb_assign).astype(np.uint8)
        cb_store = cb_assign
    elif mode == "lloyd":                                            # codec.py:591-596
        if codebook is None:
            flatv = v.reshape(-1)
            sample = flatv if lloyd_sample is None else flatv[lloyd_sample]
            codebook = lloyd_fit(sample, 1 << bits)
        cb_assign = np.asarray(codebook, dtype=np.float32)
        codes = companded_assign(v, cb_assign).astype(np.uint8)
        cb_store = cb_assign.astype(np.float16)
    elif mode == "uniform":                                          # codec.py:597-600
        codes = np.clip(np.rint(v), 0, levels).astype(np.uint8)
    else:
        raise ValueError(f"unknown mode {mode!r}")
    codes = codes.reshape(rows, padded_cols)
    packed = pack_codes(codes, bits)
    scale16 = scale.astype(np.float16)                               # codec.py:637-638
    gmin16 = gmin.astype(np.float16)
    q = QT(rows=rows, cols=cols, bits=bits, group_size=group_size, padded_cols=padded_cols,
           n_groups=n_groups, packed=packed, scale=scale16, gmin=gmin16,
           outlier_idx=idx.astype(np.int32), outlier_val=vals.astype(np.float16),
           codebook=cb_store, codes=codes, threshold=None if thr is None else float(thr),
           assign_codebook_f32=cb_assign,
           smooth_scale=None if s_smooth is None else s_smooth.astype(np.float16))
    if double_quant:                                                 # codec.py:644-652
        q.dq_scale_codes, q.dq_scale_meta = double_quantize(scale16, dq_group_size)
        q.dq_gmin_codes, q.dq_gmin_meta = double_quantize(gmin16, dq_group_size)
        n = rows * n_groups
        q.scale = double_dequantize_f16(q.dq_scale_codes, q.dq_scale_meta, n).reshape(rows, n_groups)
        q.gmin = double_dequantize_f16(q.dq_gmin_codes, q.dq_gmin_meta, n).reshape(rows, n_groups)
    return q


# ---------------------------------------------------------------------------
# dequantize and QuantLinear math
# ---------------------------------------------------------------------------

def resolve_scale_gmin(q) -> Tuple[np.ndarray, np.ndarray]:
    """fp32 [rows, n_groups] scale/gmin, codec.py:740-758 and
    modules.py:558-583 (DQ reconstruction kept in fp32, not rounded to fp16)."""
    n = q.rows * q.n_groups
    if getattr(q, "dq_scale_codes", None) is not None:
        s = double_dequantize_f32(q.dq_scale_codes, q.dq_scale_meta, n)
        m = double_dequantize_f32(q.dq_gmin_codes, q.dq_gmin_meta, n)
        return s.reshape(q.rows, q.n_groups), m.reshape(q.rows, q.n_groups)
    return q.scale.astype(np.float32), q.gmin.astype(np.float32)


def code_values(q) -> np.ndarray:
    """Reconstruction level of every code (codebook[code] or code), fp32."""
    codes = unpack_codes(q.packed, q.bits, q.padded_cols)
    if getattr(q, "codebook", None) is not None:
        return q.codebook.astype(np.float32)[codes]
    return codes.astype(np.float32)


def quantize_rvq(w: np.ndarray, group_size: int = 128, outlier_frac: float = 0.001, double_quant: bool = False,
                 dq_group_size: int = 256, smooth: bool = False, smooth_alpha: float = 0.5) -> QT:
    """6-bit residual quantization, codec.py:678-737: 4-bit stage (outliers,
    double quant and smoothing as asked), then the fp32 residual w - W4 at
    2 bits with no outliers, no smoothing and no double quant."""
    q4 = quantize(w, 4, group_size, outlier_frac, double_quant, dq_group_size, smooth=smooth,
                  smooth_alpha=smooth_alpha)
    res = np.asarray(w).astype(np.float32) - dequantize(q4)
    q2 = quantize(res, 2, group_size, 0.0)
    q4.bits = 6
    q4.stage2_packed, q4.stage2_scale, q4.stage2_gmin = q2.packed, q2.scale, q2.gmin
    return q4


def dequantize(q, exact_outliers: bool = True) -> np.ndarray:
    """codec.py:761-807, 810-847: fp32 W [rows, cols]; outlier positions hold
    the exact stored `outlier_val` (the oracle definition of the weight);
    columns multiplied back by the smooth scales; 6-bit: plus the 2-bit
    residual stage."""
    if q.bits == 6:
        s1 = QT(rows=q.rows, cols=q.cols, bits=4, group_size=q.group_size, padded_cols=q.padded_cols,
                n_groups=q.n_groups, packed=q.packed, scale=q.scale, gmin=q.gmin, outlier_idx=q.outlier_idx,
                outlier_val=q.outlier_val, dq_scale_codes=q.dq_scale_codes, dq_scale_meta=q.dq_scale_meta,
                dq_gmin_codes=q.dq_gmin_codes, dq_gmin_meta=q.dq_gmin_meta, smooth_scale=q.smooth_scale)
        s2 = QT(rows=q.rows, cols=q.cols, bits=2, group_size=q.group_size, padded_cols=q.padded_cols,
                n_groups=q.n_groups, packed=q.stage2_packed, scale=q.stage2_scale, gmin=q.stage2_gmin,
                outlier_idx=np.zeros(0, np.int32), outlier_val=np.zeros(0, np.float16))
        return dequantize(s1, exact_outliers) + dequantize(s2)
    cv = code_values(q).reshape(q.rows, q.n_groups, q.group_size)
    s, m = resolve_scale_gmin(q)
    deq = (cv * s[..., None] + m[..., None]).reshape(q.rows, q.padded_cols)[:, : q.cols]
    flat = deq.reshape(-1).copy()
    if exact_outliers and q.outlier_idx.shape[0]:
        flat[q.outlier_idx.astype(np.int64)] = q.outlier_val.astype(np.float32)
    out = flat.reshape(q.rows, q.cols)
    if getattr(q, "smooth_scale", None) is not None:
        out = out * q.smooth_scale.astype(np.float32)[None, :]
    return out


@dataclass
class OutlierTables:
    row: np.ndarray      # int32, stable-sorted by row (modules.py:414-431)
    col: np.ndarray      # int32
    val: np.ndarray      # fp16, in the same order
    delta: np.ndarray    # fp16 (modules.py:649-715)
    row_ptr: np.ndarray  # int32 [rows + 1] CSR offsets into the sorted tables


def outlier_tables(q) -> OutlierTables:
    """QuantLinear's outlier buffers (modules.py:414-448) plus the CSR row
    offsets the CUDA epilogue walks. delta = f16(f32(val) - base) where base
    is the plain group-affine value at (row, col), modules.py:649-715."""
    idx = q.outlier_idx.astype(np.int64)
    if idx.shape[0] == 0:
        z = np.zeros(0, dtype=np.int32)
        return OutlierTables(z, z, np.zeros(0, np.float16), np.zeros(0, np.float16),
                             np.zeros(q.rows + 1, dtype=np.int32))
    row = idx // q.cols
    col = idx % q.cols
    perm = np.argsort(row, kind="stable")
    row, col = row[perm], col[perm]
    val = q.outlier_val[perm]
    codes = unpack_codes(q.packed, q.bits, q.padded_cols)[row, col]
    if getattr(q, "codebook", None) is not None:
        cv = q.codebook.astype(np.float32)[codes]
    else:
        cv = codes.astype(np.float32)
    s, m = resolve_scale_gmin(q)
    grp = col // q.group_size
    base = cv * s[row, grp] + m[row, grp]
    delta = (val.astype(np.float32) - base).astype(np.float16)
    row_ptr = np.searchsorted(row, np.arange(q.rows + 1), side="left").astype(np.int32)
    return OutlierTables(row.astype(np.int32), col.astype(np.int32), val, delta, row_ptr)


def qlinear(x: np.ndarray, q, bias: Optional[np.ndarray] = None) -> np.ndarray:
    """The GEMM oracle: fp32 x @ dequantize(q).T (+ bias)."""
    W = dequantize(q)
    y = x.astype(np.float32).reshape(-1, q.cols) @ W.T
    if bias is not None:
        y = y + bias.astype(np.float32)
    return y.reshape(*x.shape[:-1], q.rows)


def qlinear_rows(x: np.ndarray, q, r0: int, r1: int) -> np.ndarray:
    """fp32 x @ W[r0:r1].T for a row block of the weight (exact outliers);
    the chunked form of the reference's CPU forward (modules.py:924-938)."""
    codes = unpack_codes(q.packed[r0:r1], q.bits, q.padded_cols)
    cv = q.codebook.astype(np.float32)[codes] if getattr(q, "codebook", None) is not None \
        else codes.astype(np.float32)
    s, m = resolve_scale_gmin(q)
    n = r1 - r0
    W = (cv.reshape(n, q.n_groups, q.group_size) * s[r0:r1, :, None]
         + m[r0:r1, :, None]).reshape(n, q.padded_cols)[:, : q.cols]
    idx = q.outlier_idx.astype(np.int64)
    sel = (idx >= r0 * q.cols) & (idx < r1 * q.cols)
    if sel.any():
        W = np.ascontiguousarray(W)
        W.reshape(-1)[idx[sel] - r0 * q.cols] = q.outlier_val[sel].astype(np.float32)
    return x.astype(np.float32).reshape(-1, q.cols) @ W.T


def qlinear_threaded(x: np.ndarray, q, threads: int, chunk_rows: int = 1024,
                     rows: Optional[int] = None) -> np.ndarray:
    """qlinear over the first `rows` weight rows (all by default), row chunks
    dequantized and multiplied on `threads` host threads (numpy releases the
    GIL). Used only as the timed CPU baseline."""
    from concurrent.futures import ThreadPoolExecutor
    rows = q.rows if rows is None else rows
    spans = [(r, min(r + chunk_rows, rows)) for r in range(0, rows, chunk_rows)]
    with ThreadPoolExecutor(max_workers=threads) as ex:
        parts = list(ex.map(lambda s: qlinear_rows(x, q, *s), spans))
    return np.concatenate(parts, axis=-1)


def max_rel_error(y: np.ndarray, y_ref: np.ndarray) -> float:
    """max|y - y_ref| / max|y_ref|: the GEMM tolerance metric used by tests."""
    y = np.asarray(y, dtype=np.float64)
    r = np.asarray(y_ref, dtype=np.float64)
    return float(np.abs(y - r).max() / max(np.abs(r).max(), 1e-30))


def student_t_weights(shape, seed: int, std: float = 0.02, dtype=np.float16) -> np.ndarray:
    """Seeded synthetic weights: Student-t(df=4) rescaled to `std`."""
    rng = np.random.default_rng(seed)
    w = rng.standard_t(4, size=shape).astype(np.float32)
    w *= std / max(float(w.std()), 1e-12)
    return w.astype(dtype)

