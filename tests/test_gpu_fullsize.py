"""Full-size parity of the GPU quantizer and the fused dequant-GEMM on the
shapes of every benchmark config, against the oracle (pinned to the
reference by tests/test_oracle_golden.py).

* config 2: Llama MLP gate/up [14336, 4096] and down [4096, 14336], 4-bit g128
  uniform + 0.1% outliers;
* config 3: [8192, 8192] and [28672, 8192], 2-bit Lloyd-Max g64 + 0.1%
  outliers, the levels fitted on the device from a 300,000-value sample;
* config 4: Llama-3-8B projections with per-layer forced bit widths 2/4/8;
* config 5: a Llama-70B up projection [28672, 8192], 4-bit g128 NF with
  double quantization (the reference's quantize_module defaults);
* adaptive escalation (codec.py:863-931) against the oracle's errors.

Codes, packed bytes, metadata, outlier indices/values, outlier tables and
fitted levels must be bit-identical; GEMM outputs within 1e-2 max-relative
of the fp32 dequant-matmul.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import goap
from tests.test_gpu_parity import assert_device_quant_equals_oracle

pytestmark = pytest.mark.gpu

TOL = 1e-2


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import tensorshrink_b200._C as C
    C.load()
    yield


def _check_gemm(ql, q, Ms, dtype=torch.bfloat16, seed=0):
    """GEMM outputs at each M against x @ W_oracle^T in fp32 (rows sampled for
    the reference product when M is large, to keep the CPU work bounded)."""
    W = goap.dequantize(q)
    g = torch.Generator(device="cuda").manual_seed(seed)
    for M in Ms:
        x = torch.randn(M, ql.in_features, device="cuda", generator=g).to(dtype)
        y = ql(x).float().cpu().numpy()
        rows = np.arange(M) if M <= 64 else np.linspace(0, M - 1, 64).astype(np.int64)
        ref = x.float().cpu().numpy()[rows] @ W.T
        err = goap.max_rel_error(y[rows], ref)
        assert err <= TOL, (M, err)


@pytest.mark.parametrize("shape", [(14336, 4096), (4096, 14336)])
def test_config2_mlp_full_size(shape):
    import tensorshrink_b200 as ts
    w_np = goap.student_t_weights(shape, seed=sum(shape))
    d = ts.quantize_device(torch.from_numpy(w_np).cuda(), bits=4, group_size=128, outlier_frac=0.001,
                           double_quant=False, nf_quant=False)
    q = goap.quantize(w_np, bits=4, group_size=128, outlier_frac=0.001, mode="uniform")
    assert_device_quant_equals_oracle(d, q)
    _check_gemm(ts.QuantLinear.from_device_quant(d), q, (1, 8, 32, 64, 256))


@pytest.mark.parametrize("shape", [(8192, 8192), (28672, 8192)])
def test_config3_lloyd2_full_size(shape):
    """The reference fits its levels on torch.randperm(n)[:300000] of the
    normalized values (codec.py:329-333); the same sample goes to the device
    fit and to the oracle's fit, and the levels must agree bit for bit."""
    import tensorshrink_b200 as ts
    rows, cols = shape
    w_np = goap.student_t_weights(shape, seed=rows // 1024)
    gen = torch.Generator().manual_seed(rows)
    sample = torch.randperm(rows * cols, generator=gen)[:300_000]
    d = ts.quantize_device(torch.from_numpy(w_np).cuda(), bits=2, group_size=64, outlier_frac=0.001,
                           companded=True, lloyd_sample=sample.cuda())
    q = goap.quantize(w_np, bits=2, group_size=64, outlier_frac=0.001, mode="lloyd",
                      lloyd_sample=sample.numpy())
    np.testing.assert_array_equal(d.codebook_assign.cpu().numpy(), q.assign_codebook_f32)
    assert_device_quant_equals_oracle(d, q)
    _check_gemm(ts.QuantLinear.from_device_quant(d), q, (1, 256, 2048))


@pytest.mark.parametrize("shape,bits", [((4096, 4096), 2), ((1024, 4096), 8), ((14336, 4096), 4),
                                        ((4096, 14336), 8)])
def test_config4_forced_bits(shape, bits):
    """quantize_tensor_adaptive(force_bits=b) per layer, as the decoder's
    seeded per-layer draw uses it (g128, uniform + outliers)."""
    import tensorshrink_b200 as ts
    w_np = goap.student_t_weights(shape, seed=bits + shape[0])
    d, err, esc = ts.quantize_device_adaptive(torch.from_numpy(w_np).cuda(), group_size=128,
                                              outlier_frac=0.001, force_bits=bits)
    assert not esc
    q = goap.quantize(w_np, bits=bits, group_size=128, outlier_frac=0.001, mode="uniform")
    assert_device_quant_equals_oracle(d, q)
    w64 = w_np.astype(np.float64)
    ref_err = np.linalg.norm(w64 - goap.dequantize(q)) / np.linalg.norm(w64)
    assert abs(err - ref_err) <= 1e-4 * ref_err   # the device sums fp32 squares
    _check_gemm(ts.QuantLinear.from_device_quant(d), q, (1, 16, 128))


def test_config5_llama70b_up_full_size():
    import tensorshrink_b200 as ts
    w_np = goap.student_t_weights((28672, 8192), seed=70)
    d = ts.quantize_device(torch.from_numpy(w_np).cuda(), bits=4, group_size=128, outlier_frac=0.001,
                           double_quant=True, nf_quant=True)
    q = goap.quantize(w_np, bits=4, group_size=128, outlier_frac=0.001, double_quant=True, mode="nf")
    assert_device_quant_equals_oracle(d, q)
    _check_gemm(ts.QuantLinear.from_device_quant(d), q, (1, 32))


def test_adaptive_escalation_matches_oracle():
    """2 -> 4 -> 8 escalation (codec.py:863-931): the first width whose
    relative Frobenius error is within the threshold, the last one always."""
    import tensorshrink_b200 as ts
    w_np = goap.student_t_weights((1024, 2048), seed=99)
    w64 = w_np.astype(np.float64)
    errs = {}
    for b in (2, 4, 8):
        q = goap.quantize(w_np, bits=b, group_size=128, outlier_frac=0.001, mode="uniform")
        errs[b] = np.linalg.norm(w64 - goap.dequantize(q)) / np.linalg.norm(w64)
    assert errs[2] > errs[4] > errs[8]
    w = torch.from_numpy(w_np).cuda()
    cases = [(0.5 * (errs[2] + errs[4]), 4, True),      # 2-bit too coarse, 4-bit accepted
             (2.0 * errs[2], 2, False),                  # 2-bit accepted at once
             (0.5 * errs[8], 8, True)]                   # nothing within: the last width
    for thr, want_bits, want_esc in cases:
        qt, err, esc = ts.quantize_tensor_adaptive(w, group_size=128, outlier_frac=0.001,
                                                   error_threshold=thr, allowed_bits=(2, 4, 8))
        assert (qt.bits, esc) == (want_bits, want_esc), thr
        assert abs(err - errs[want_bits]) <= 1e-4 * errs[want_bits]
        q = goap.quantize(w_np, bits=want_bits, group_size=128, outlier_frac=0.001, mode="uniform")
        np.testing.assert_array_equal(qt.packed, q.packed)
        np.testing.assert_array_equal(qt.outlier_idx, q.outlier_idx)
