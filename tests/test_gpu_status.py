"""Device error status of the qlinear kernels, through the C ABI.

Every barrier wait inside the kernels is bounded. `ts_test_inject_stall`
makes the next launch run with its copy producer disabled and a 1 ms wait
limit: the barriers it waits on are never completed by anyone, the waits run
out, the kernel unwinds and records its code, and `ts_qlinear_status`
reports TS_ERR_TIMEOUT. Nothing faults or hangs. After the status call has
cleared the flags, the same workspace gives the same results as before the
stall (the row-block counters were reset).
"""

from __future__ import annotations

import ctypes as C

import pytest
import torch

from oracle import goap

pytestmark = pytest.mark.gpu

TS_ERR_TIMEOUT = -5
STALL_NS = 1_000_000   # 1 ms


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import tensorshrink_b200._C as _C
    return _C.load()


def _layer(rows, cols, seed, **kw):
    import tensorshrink_b200 as ts
    w = torch.from_numpy(goap.student_t_weights((rows, cols), seed=seed)).cuda()
    return ts.QuantLinear.from_device_quant(ts.quantize_device(w, **kw))


def _stream():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("M", [1, 8, 32, 256])   # decode GEMV x2, split tensor-core kernel x2
def test_stalled_call_reports_timeout_then_recovers(lib, M):
    from tensorshrink_b200 import kernels
    ql = _layer(2048, 4096, seed=M, bits=4, group_size=128, outlier_frac=0.001, double_quant=False,
                nf_quant=False)
    qw = ql.qweight()
    x = torch.randn(M, 4096, device="cuda").to(torch.bfloat16)
    ws = kernels.workspace_for(x.device, int(lib.ts_qlinear_workspace_size(C.byref(qw), M)))
    assert lib.ts_qlinear_status(ws.data_ptr(), ws.numel(), 1, _stream()) == 0
    good = kernels.qlinear(x, qw, None, torch.float32, workspace=ws)
    assert lib.ts_qlinear_status(ws.data_ptr(), ws.numel(), 1, _stream()) == 0

    assert lib.ts_test_inject_stall(STALL_NS) == 0
    kernels.qlinear(x, qw, None, torch.float32, workspace=ws)
    rc = lib.ts_qlinear_status(ws.data_ptr(), ws.numel(), 1, _stream())
    assert rc == TS_ERR_TIMEOUT
    assert b"bounded wait" in lib.ts_last_error()
    # cleared: the flags read zero, and the workspace works again
    assert lib.ts_qlinear_status(ws.data_ptr(), ws.numel(), 0, _stream()) == 0
    again = kernels.qlinear(x, qw, None, torch.float32, workspace=ws)
    assert lib.ts_qlinear_status(ws.data_ptr(), ws.numel(), 1, _stream()) == 0
    assert torch.equal(again, good)


def test_device_status_helper_raises(lib):
    """kernels.device_status checks every cached workspace of the device."""
    from tensorshrink_b200 import kernels
    ql = _layer(1024, 1024, seed=5, bits=4, group_size=128, outlier_frac=0.001)
    x = torch.randn(1, 1024, device="cuda").to(torch.float16)
    ql(x)
    kernels.device_status()
    assert lib.ts_test_inject_stall(STALL_NS) == 0
    ql(x)
    with pytest.raises(RuntimeError, match="bounded wait"):
        kernels.device_status()
    kernels.device_status()
    y = ql(x)
    torch.cuda.synchronize()
    assert torch.isfinite(y.float()).all()


def test_inject_stall_rejects_bad_limit(lib):
    assert lib.ts_test_inject_stall(0) == -1
    assert lib.ts_test_inject_stall(3_000_000_000) == -1
