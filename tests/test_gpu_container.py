"""Container entries loaded straight into device QuantLinear buffers
(`ContainerReader.to_quantlinear`, `ts_outlier_tables_from_stream`): the
outlier tables built on the device equal the host build from the reference
reader's QuantizedTensor bit for bit, and the layers compute the same
outputs; also the 32-bit index stream and a whole-module save/load.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from tensorshrink_b200 import container as ct
from tensorshrink_b200.modules import QuantLinear, host_outlier_tables

pytestmark = pytest.mark.gpu
TSK = Path(__file__).resolve().parent / "golden" / "ref_container.tsk"


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _same_tables(ql, qt):
    row, col, delta, ptr = host_outlier_tables(qt)
    np.testing.assert_array_equal(ql.outlier_row.cpu().numpy(), row)
    np.testing.assert_array_equal(ql.outlier_col.cpu().numpy(), col)
    np.testing.assert_array_equal(ql.outlier_delta.cpu().numpy().view(np.uint16), delta.view(np.uint16))
    np.testing.assert_array_equal(ql.outlier_row_ptr.cpu().numpy(), ptr)


def test_reference_entries_to_device():
    with ct.ContainerReader(TSK) as rd:
        for name in rd.names():
            if rd.kind(name) != "quant":
                continue
            qt = rd.get_quantized(name)
            ql = rd.to_quantlinear(name, "cuda")
            _same_tables(ql, qt)
            ref = QuantLinear(qt).cuda()
            x = torch.randn(5, qt.cols, device="cuda").to(torch.float16)
            torch.testing.assert_close(ql(x), ref(x), rtol=0, atol=0)


def test_wide_index_stream_and_double_quant(tmp_path):
    """cols > 65535 forces 32-bit indices; double-quant parts round trip."""
    import tensorshrink_b200 as ts
    g = torch.Generator(device="cuda").manual_seed(0)
    w = (torch.randn(64, 70016, device="cuda", generator=g) * 0.02).half()
    d = ts.quantize_device(w, bits=4, group_size=128, outlier_frac=0.002, double_quant=True, nf_quant=True)
    src = QuantLinear.from_device_quant(d)
    p = tmp_path / "w.tsk"
    with ct.ContainerWriter(p) as wr:
        wr.add_quantized("w", src)
    with ct.ContainerReader(p) as rd:
        assert rd.entry("w")["segments_v2"]["parts"]["outlier_col"]["np_dtype"] == "uint32"
        ql = rd.to_quantlinear("w", "cuda")
    for b in ("packed", "dq_scale_codes", "dq_scale_meta", "outlier_row", "outlier_col", "outlier_row_ptr"):
        assert torch.equal(getattr(ql, b), getattr(src, b)), b
    assert torch.equal(ql.outlier_delta.view(torch.int16), src.outlier_delta.view(torch.int16))
    x = torch.randn(3, 70016, device="cuda").to(torch.bfloat16)
    assert torch.equal(ql(x), src(x))


def test_save_and_load_module(tmp_path):
    import tensorshrink_b200 as ts
    torch.manual_seed(0)
    model = torch.nn.Sequential(torch.nn.Linear(512, 1024), torch.nn.LayerNorm(1024),
                                torch.nn.Linear(1024, 256)).cuda().half()
    ts.quantize_module(model, min_numel=1, verbose=False)
    p = tmp_path / "m.tsk"
    ct.save_quant_module(model, p, verbose=False)
    fresh = torch.nn.Sequential(torch.nn.Linear(512, 1024), torch.nn.LayerNorm(1024),
                                torch.nn.Linear(1024, 256)).cuda().half()
    with ct.ContainerReader(p) as rd:
        st = ct.load_quantized_module(fresh, rd, device="cuda", verbose=False)
    assert st["n_quant_replaced"] == 2
    x = torch.randn(4, 512, device="cuda").half()
    assert torch.equal(model(x), fresh(x))
