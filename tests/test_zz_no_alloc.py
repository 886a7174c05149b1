"""ts_qlinear_noalloc, the allocation-free decode entry point, called through
the C ABI: its output must match ts_qlinear (caller workspace) on the same
inputs bit for bit, on two calls in a row (the second call relies on the
first having left the library's fixed scratch array zeroed again), and stay
within the parity tolerance of the oracle; decode calls with weights whose
scratch need exceeds the fixed size must be rejected with an error.

The file name sorts last so that it also runs after every other GPU test
in one session; it passes alone as well.
"""

from __future__ import annotations

import ctypes as C

import pytest
import torch

from oracle import goap

pytestmark = pytest.mark.gpu

TOL = 1e-2  # max relative error against the oracle (fp32 dequant-matmul)


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import tensorshrink_b200._C as _C
    return _C.load()


def _layer(rows, cols, bits, mode, dq, seed):
    import tensorshrink_b200 as ts
    w = torch.from_numpy(goap.student_t_weights((rows, cols), seed=seed)).cuda()
    d = ts.quantize_device(w, bits=bits, group_size=128, outlier_frac=0.001, double_quant=dq,
                           nf_quant=mode == "nf")
    return ts.QuantLinear.from_device_quant(d)


def _noalloc(lib, qw, x, out, bias=None):
    from tensorshrink_b200.kernels import dtype_code
    s = torch.cuda.current_stream().cuda_stream
    return lib.ts_qlinear_noalloc(C.byref(qw), x.data_ptr(), dtype_code(x.dtype), x.shape[0],
                                  x.stride(0), bias.data_ptr() if bias is not None else None,
                                  dtype_code(bias.dtype) if bias is not None else 0,
                                  out.data_ptr(), dtype_code(out.dtype), out.stride(0), s)


@pytest.mark.parametrize("rows,cols,bits,mode,dq,M", [
    (4096, 4096, 4, "nf", True, 1),
    (14336, 4096, 4, "uniform", False, 1),
    (4096, 14336, 4, "uniform", False, 8),
    (1000, 768, 2, "nf", True, 3),
    (512, 1024, 8, "uniform", True, 16),
])
def test_noalloc_matches_workspace_entry(lib, rows, cols, bits, mode, dq, M):
    """Bit-identical to ts_qlinear given a caller workspace of the same size
    as the fixed array (same kernel, same partition, only the scratch's
    owner differs) on two calls in a row, and within the parity tolerance
    of the oracle's fp32 dequant-matmul."""
    from tensorshrink_b200 import kernels
    ql = _layer(rows, cols, bits, mode, dq, seed=rows + cols + bits)
    qw = ql.qweight()
    limit = int(lib.ts_qlinear_noalloc_max_scratch())
    assert lib.ts_qlinear_workspace_size(C.byref(qw), 1) <= limit
    x = torch.randn(M, cols, device="cuda").to(torch.bfloat16)
    bias = torch.randn(rows, device="cuda").to(torch.bfloat16) * 0.1
    ws = torch.zeros(limit, dtype=torch.uint8, device="cuda")
    ref = kernels.qlinear(x, qw, bias, torch.float32, workspace=ws)
    W = goap.dequantize(ql.to_quantized_tensor())
    y_oracle = x.float().cpu().numpy() @ W.T + bias.float().cpu().numpy()
    for _ in range(2):
        out = torch.full((M, rows), float("nan"), device="cuda", dtype=torch.float32)
        rc = _noalloc(lib, qw, x, out, bias)
        assert rc == 0, lib.ts_last_error().decode()
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
        assert goap.max_rel_error(out.cpu().numpy(), y_oracle) <= TOL
    assert lib.ts_qlinear_status(None, 0, 1, torch.cuda.current_stream().cuda_stream) == 0


def test_noalloc_rejects_oversized_weight(lib):
    """A weight whose split-row counters do not fit the fixed array."""
    from tensorshrink_b200 import kernels
    limit = int(lib.ts_qlinear_noalloc_max_scratch())
    rows = 1 << 20   # 65536 row blocks of counters (256 KiB) after ~296 KiB of partial sums
    cols = 128
    packed = torch.zeros((rows, cols // 2), dtype=torch.uint8, device="cuda")
    scale = torch.ones((rows, 1), dtype=torch.float16, device="cuda")
    gmin = torch.zeros((rows, 1), dtype=torch.float16, device="cuda")
    qw = kernels.make_qweight(packed=packed, scale=scale, gmin=gmin, bits=4, group_size=128, cols=cols,
                              out_features=rows)
    assert lib.ts_qlinear_workspace_size(C.byref(qw), 1) > limit
    x = torch.zeros((1, cols), dtype=torch.float16, device="cuda")
    out = torch.zeros((1, rows), dtype=torch.float16, device="cuda")
    rc = _noalloc(lib, qw, x, out)
    assert rc == -2   # TS_ERR_UNSUPPORTED
    assert b"scratch" in lib.ts_last_error()
    # the tensor-core kernel needs no scratch: a prefill-sized call is taken
    M = 128
    x = torch.randn((M, cols), device="cuda").to(torch.float16)
    out = torch.empty((M, rows), dtype=torch.float16, device="cuda")
    rc = _noalloc(lib, qw, x, out)
    assert rc == 0, lib.ts_last_error().decode()
    torch.cuda.synchronize()
    # codes 0, scale 1, min 0: every weight is 0
    assert not out.any()
