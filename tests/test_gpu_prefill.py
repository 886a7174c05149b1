"""GPU parity of the prefill-shaped (M >= 65) tensor-core dequant-GEMM.

Reference: y_ref = x.float() @ W.T (+bias) in fp32, W the oracle's (or, for
the largest shapes, the dense fp32 reconstruction kernel's, itself checked
bit-exactly against the oracle in test_gpu_parity.py) dequantized weight
with exact outlier values. Bar: max|y - y_ref| / max|y_ref| <= 1e-2.
"""

from __future__ import annotations

import pytest
import torch

from oracle import goap
from tests.conftest import load_case
from tests.test_host_cpu import qt_from_case

pytestmark = pytest.mark.gpu

TOL = 1e-2


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import tensorshrink_b200._C as C
    C.load()
    yield


def _layer(rows, cols, bits, gs, mode, dq, seed, frac=0.002):
    import tensorshrink_b200 as ts
    w = torch.from_numpy(goap.student_t_weights((rows, cols), seed=seed)).cuda()
    return ts.quantize_device(w, bits=bits, group_size=gs, outlier_frac=frac, double_quant=dq,
                              nf_quant=mode == "nf", companded=mode == "lloyd")


def _ref(x, W, bias=None):
    y = x.float() @ W.T
    return y + bias.float() if bias is not None else y


def _rel(y, ref):
    return ((y.float() - ref).abs().max() / ref.abs().max()).item()


@pytest.mark.parametrize("bits,gs,mode,dq", [
    (4, 128, "uniform", False), (4, 128, "nf", True), (4, 64, "uniform", True), (4, 32, "uniform", False),
    (4, 16, "nf", False), (2, 64, "lloyd", False), (2, 128, "uniform", True), (2, 32, "nf", False),
    (8, 128, "uniform", False), (8, 64, "nf", True)])
@pytest.mark.parametrize("xdt", [torch.bfloat16, torch.float16])
def test_prefill_modes(bits, gs, mode, dq, xdt):
    import tensorshrink_b200 as ts
    rows, cols = 1000, 1000          # ragged against the 128/256-row tiles and 64-column stages
    d = _layer(rows, cols, bits, gs, mode, dq, seed=bits * 100 + gs)
    W = torch.from_numpy(goap.dequantize(d.to_quantized_tensor())).cuda()
    bias = (torch.randn(rows, device="cuda") * 0.1).to(xdt)
    ql = ts.QuantLinear.from_device_quant(d, bias)
    for M in (65, 128, 300):
        x = torch.randn(M, cols, device="cuda").to(xdt)
        y = ql(x)
        assert y.dtype == xdt and y.shape == (M, rows)
        err = _rel(y, _ref(x, W, bias))
        assert err <= TOL, (M, err)


def test_prefill_out_fp32_and_strided_out():
    import tensorshrink_b200 as ts
    from tensorshrink_b200 import kernels
    d = _layer(512, 768, 4, 128, "uniform", False, seed=3)
    ql = ts.QuantLinear.from_device_quant(d)
    W = torch.from_numpy(goap.dequantize(d.to_quantized_tensor())).cuda()
    x = torch.randn(200, 768, device="cuda", dtype=torch.bfloat16)
    y = kernels.qlinear(x, ql.qweight(), None, torch.float32)
    assert y.dtype == torch.float32
    assert _rel(y, _ref(x, W)) <= TOL
    big = torch.zeros(200, 600, device="cuda", dtype=torch.float16)
    kernels.qlinear(x.half(), ql.qweight(), None, torch.float16, out=big[:, :512])
    assert _rel(big[:, :512], _ref(x.half(), W)) <= TOL
    assert torch.all(big[:, 512:] == 0)


@pytest.mark.parametrize("name", ["nf4_dq_g128", "u4_g128_pad", "lloyd2_g64", "u8_dq_g128", "u4_ties"])
def test_prefill_reference_ordered_outliers(golden, name):
    """QuantLinear buffers exactly as the reference builds them (outliers in
    top-k order within a row) on the tensor-core path."""
    import tensorshrink_b200 as ts
    c = load_case(golden, name)
    qt = qt_from_case(c)
    bias = torch.from_numpy(c["bias"]) if "bias" in c else None
    ql = ts.QuantLinear(qt, bias).cuda()
    W = torch.from_numpy(goap.dequantize(qt)).cuda()
    x = torch.randn(150, qt.cols, device="cuda", dtype=torch.float16)
    y = ql(x)
    err = _rel(y, _ref(x, W, bias.cuda() if bias is not None else None))
    assert err <= TOL, err


def test_prefill_deterministic():
    import tensorshrink_b200 as ts
    d = _layer(2048, 2048, 4, 128, "nf", True, seed=11)
    ql = ts.QuantLinear.from_device_quant(d)
    x = torch.randn(512, 2048, device="cuda", dtype=torch.bfloat16)
    y0 = ql(x)
    for _ in range(3):
        assert torch.equal(ql(x), y0)


@pytest.mark.parametrize("M", [256, 2048])
def test_prefill_config3_8192(M):
    """Config 3: 2-bit Lloyd-Max, group 64, outliers 1e-3, [8192, 8192], bf16."""
    import tensorshrink_b200 as ts
    d = _layer(8192, 8192, 2, 64, "lloyd", False, seed=31, frac=0.001)
    W = ts.dequantize_device(d)
    ql = ts.QuantLinear.from_device_quant(d)
    x = torch.randn(M, 8192, device="cuda", dtype=torch.bfloat16)
    err = _rel(ql(x), _ref(x, W))
    assert err <= TOL, err


def test_prefill_config3_28672():
    import tensorshrink_b200 as ts
    d = _layer(28672, 8192, 2, 64, "lloyd", False, seed=32, frac=0.001)
    W = ts.dequantize_device(d)
    ql = ts.QuantLinear.from_device_quant(d)
    x = torch.randn(256, 8192, device="cuda", dtype=torch.bfloat16)
    err = _rel(ql(x), _ref(x, W))
    assert err <= TOL, err


def test_prefill_large_k_4bit():
    """Down-projection shape [4096, 14336], 4-bit g128 uniform, M = 2048."""
    import tensorshrink_b200 as ts
    d = _layer(4096, 14336, 4, 128, "uniform", False, seed=41, frac=0.001)
    W = ts.dequantize_device(d)
    ql = ts.QuantLinear.from_device_quant(d)
    x = torch.randn(2048, 14336, device="cuda", dtype=torch.bfloat16)
    err = _rel(ql(x), _ref(x, W))
    assert err <= TOL, err


@pytest.mark.parametrize("shuffle", [False, True])
def test_tensor_core_dense_outliers(shuffle):
    """5% outliers (about 100 per row, far more than a dequantizer's outlier
    queue holds, so it refills) in column order and in a shuffled order
    within rows, on the prefill tiles and on the split decode plan."""
    import numpy as np
    import tensorshrink_b200 as ts
    d = _layer(300, 2048, 4, 128, "uniform", False, seed=11, frac=0.05)
    qt = d.to_quantized_tensor()
    if shuffle:
        perm = np.random.default_rng(0).permutation(qt.outlier_idx.shape[0])
        qt.outlier_idx = qt.outlier_idx[perm]
        qt.outlier_val = qt.outlier_val[perm]
    ql = ts.QuantLinear(qt).cuda()
    W = torch.from_numpy(goap.dequantize(qt)).cuda()
    for M in (20, 64, 100, 300):
        x = torch.randn(M, 2048, device="cuda", dtype=torch.bfloat16)
        err = _rel(ql(x), _ref(x, W))
        assert err <= TOL, (M, err)
