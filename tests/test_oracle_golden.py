"""Pin the numpy oracle against the reference's own outputs (golden fixtures).

These run on CPU. Codes, packed bytes, double-quant codes/meta, outlier
indices and outlier deltas must be bit-identical; the top-k tie rule is
checked as: same count, identical set of strictly-above-threshold indices,
every remaining chosen index ties at the threshold.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import goap
from tests.conftest import golden_case_list, load_case


def _quantize_case(c):
    bits, gs, dq, _ = (int(v) for v in c["params"])
    mode = str(c["mode"])
    cb = c["lloyd_cb32"] if mode == "lloyd" else None
    return goap.quantize(c["w"], bits=bits, group_size=gs, outlier_frac=float(c["frac"]),
                         double_quant=bool(dq), mode=mode, codebook=cb)


def _check_outlier_set(idx_ours, idx_ref, w):
    a = np.abs(w.astype(np.float32).reshape(-1))
    assert idx_ours.shape == idx_ref.shape
    if idx_ref.shape[0] == 0:
        return
    thr = a[idx_ref].min()
    assert a[idx_ours].min() == thr
    above_ours = set(idx_ours[a[idx_ours] > thr].tolist())
    above_ref = set(idx_ref[a[idx_ref] > thr].tolist())
    assert above_ours == above_ref == set(np.flatnonzero(a > thr).tolist())
    assert np.all(a[idx_ours] >= thr)


@pytest.mark.parametrize("name", golden_case_list())
def test_quantize_matches_reference(golden, name):
    c = load_case(golden, name)
    q = _quantize_case(c)
    np.testing.assert_array_equal(q.packed, c["packed"])
    np.testing.assert_array_equal(q.scale.view(np.uint16), c["scale"].view(np.uint16))
    np.testing.assert_array_equal(q.gmin.view(np.uint16), c["gmin"].view(np.uint16))
    if "dq_scale_codes" in c:
        for f in ("dq_scale_codes", "dq_gmin_codes"):
            np.testing.assert_array_equal(getattr(q, f), c[f])
        for f in ("dq_scale_meta", "dq_gmin_meta"):
            np.testing.assert_array_equal(getattr(q, f).view(np.uint16), c[f].view(np.uint16))
    else:
        assert q.dq_scale_codes is None
    if "codebook" in c:
        np.testing.assert_array_equal(q.codebook, c["codebook"])
    _check_outlier_set(q.outlier_idx.astype(np.int64), c["outlier_idx"].astype(np.int64), c["w"])


@pytest.mark.parametrize("name", golden_case_list())
def test_outlier_tables_match_reference(golden, name):
    c = load_case(golden, name)
    q = _quantize_case(c)
    ref_idx = c["outlier_idx"].astype(np.int64)
    # Build the tables from the reference's own outlier choice so ties do not
    # change membership; compare per row as sets of (col, delta).
    q.outlier_idx = c["outlier_idx"]
    q.outlier_val = c["outlier_val"]
    t = goap.outlier_tables(q)
    assert np.all(np.diff(t.row) >= 0)
    np.testing.assert_array_equal(t.row, c["ql_outlier_row"])
    ours = sorted(zip(t.row.tolist(), t.col.tolist(), t.delta.view(np.uint16).tolist()))
    ref = sorted(zip(c["ql_outlier_row"].tolist(), c["ql_outlier_col"].tolist(),
                     c["ql_outlier_delta"].view(np.uint16).tolist()))
    assert ours == ref
    assert t.row_ptr[-1] == ref_idx.shape[0]


@pytest.mark.parametrize("name", golden_case_list())
def test_qlinear_oracle_matches_reference(golden, name):
    c = load_case(golden, name)
    q = _quantize_case(c)
    q.outlier_idx, q.outlier_val = c["outlier_idx"], c["outlier_val"]
    y = goap.qlinear(c["x"], q, c.get("bias"))
    np.testing.assert_allclose(y, c["y_ref"], rtol=1e-5, atol=1e-5)


def test_nf_codebooks(golden):
    for bits in (2, 4, 8):
        np.testing.assert_array_equal(goap.nf_codebook(bits), golden[f"nf_codebook/{bits}"])


def test_double_quant_roundtrip(golden):
    codes, meta = goap.double_quantize(golden["dq/vals"], 256)
    np.testing.assert_array_equal(codes, golden["dq/codes"])
    np.testing.assert_array_equal(meta.view(np.uint16), golden["dq/meta"].view(np.uint16))
    rec = goap.double_dequantize_f16(codes, meta, golden["dq/vals"].shape[0])
    np.testing.assert_array_equal(rec.view(np.uint16), golden["dq/recon16"].view(np.uint16))


@pytest.mark.parametrize("name", ["lloyd2_g64", "lloyd4_g128"])
def test_lloyd_fit_unsampled_case(golden, name):
    """Below the 300,000-value cap the reference fits on every normalized
    value, so the oracle's fit must reproduce its float32 levels exactly."""
    c = load_case(golden, name)
    bits, gs, _, _ = (int(v) for v in c["params"])
    q = goap.quantize(c["w"], bits=bits, group_size=gs, outlier_frac=float(c["frac"]), mode="lloyd")
    np.testing.assert_array_equal(q.assign_codebook_f32, c["lloyd_cb32"])
    np.testing.assert_array_equal(q.packed, c["packed"])


@pytest.mark.parametrize("levels", [4, 16])
def test_lloyd_fit(golden, levels):
    cent = goap.lloyd_fit(golden["lloyd/sample"], levels)
    np.testing.assert_array_equal(cent, golden[f"lloyd/cent{levels}"])


def test_oracle_smooth_and_rvq_match_reference():
    """The oracle's smoothing and 6-bit RVQ against the reference's outputs."""
    from pathlib import Path
    z = np.load(Path(__file__).resolve().parent / "golden" / "golden_rvq.npz")
    for name in z["cases"]:
        p = f"{name}/"
        bits, gs, dq, sm, nf = (int(v) for v in z[p + "params"])
        q = goap.quantize(z[p + "w"], bits=bits, group_size=gs, outlier_frac=float(z[p + "frac"]),
                          double_quant=bool(dq), mode="nf" if nf else "uniform", smooth=bool(sm),
                          smooth_alpha=float(z[p + "alpha"]))
        for f in ("packed", "scale", "gmin", "smooth_scale", "stage2_packed", "stage2_scale", "stage2_gmin",
                  "dq_scale_codes", "dq_gmin_meta"):
            if p + f in z.files:
                np.testing.assert_array_equal(getattr(q, f).view(np.uint8), z[p + f].view(np.uint8),
                                              err_msg=f"{name} {f}")
        W, ref = goap.dequantize(q), z[p + "W"]
        tied = ~np.isin(q.outlier_idx, z[p + "outlier_idx"])
        assert tied.sum() <= 2, name
        np.testing.assert_allclose(W, ref, rtol=0, atol=1e-3 * np.abs(ref).max())
