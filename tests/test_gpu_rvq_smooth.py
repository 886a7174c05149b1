"""Smooth-scaled and 6-bit RVQ quantization on the GPU against the
reference's own outputs (tests/golden/golden_rvq.npz, made by
tests/golden/make_golden_rvq.py) and the oracle: codes, scales, the smooth
scales and the residual stage bit for bit; the reconstruction to fp32
rounding (outlier positions may differ only at a top-k tie)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import goap

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden" / "golden_rvq.npz"


@pytest.fixture(scope="module")
def gold():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    with np.load(GOLD) as z:
        return {k: z[k] for k in z.files}


@pytest.mark.parametrize("name", ["smooth_u4", "smooth_nf4_dq", "rvq6", "rvq6_dq_smooth"])
def test_matches_reference(gold, name):
    import tensorshrink_b200 as ts
    p = name + "/"
    bits, gs, dq, sm, nf = (int(v) for v in gold[p + "params"])
    qt = ts.quantize_tensor(torch.from_numpy(gold[p + "w"]).cuda(), bits=bits, group_size=gs,
                            outlier_frac=float(gold[p + "frac"]), double_quant=bool(dq), smooth=bool(sm),
                            smooth_alpha=float(gold[p + "alpha"]), nf_quant=bool(nf))
    assert qt.bits == bits
    for f in ("packed", "scale", "gmin", "smooth_scale", "stage2_packed", "stage2_scale", "stage2_gmin",
              "dq_scale_codes", "dq_scale_meta", "codebook"):
        if p + f in gold:
            np.testing.assert_array_equal(getattr(qt, f).view(np.uint8), gold[p + f].view(np.uint8), err_msg=f)
    o = np.argsort(gold[p + "outlier_idx"])
    ref_idx = gold[p + "outlier_idx"][o]
    same = np.isin(qt.outlier_idx, ref_idx)
    assert same.mean() >= 0.95                      # top-k ties may pick other indices
    W = ts.dequantize_tensor(qt, dtype=torch.float32).numpy()
    q = goap.quantize(gold[p + "w"], bits=bits, group_size=gs, outlier_frac=float(gold[p + "frac"]),
                      double_quant=bool(dq), mode="nf" if nf else "uniform", smooth=bool(sm),
                      smooth_alpha=float(gold[p + "alpha"]))
    np.testing.assert_array_equal(qt.outlier_idx, q.outlier_idx)
    np.testing.assert_allclose(W, goap.dequantize(q), rtol=0, atol=1e-6)
    np.testing.assert_allclose(W, gold[p + "W"], rtol=0, atol=2e-3 * np.abs(gold[p + "W"]).max())


def test_rvq_beats_4bit_and_rejected_by_quantlinear(gold):
    import tensorshrink_b200 as ts
    w = torch.from_numpy(gold["rvq6/w"]).cuda()
    e4 = ts.relative_error(w, ts.quantize_device(w, bits=4, outlier_frac=0.003))
    d6 = ts.quantize_device(w, bits=6, outlier_frac=0.003)
    assert ts.relative_error(w, d6) < 0.5 * e4
    with pytest.raises(ValueError, match="RVQ"):
        ts.QuantLinear.from_device_quant(d6)
