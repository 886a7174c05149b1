"""Host-side logic on CPU: QuantLinear built from the reference's own
QuantizedTensors has the reference's buffers (names, dtypes, values), and
the product refuses to run the hot path on CPU."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tensorshrink_b200 import QuantLinear, QuantizedTensor
from tensorshrink_b200.codec import budget_allocate_bits, LayerBitStats, n_outliers_for
from tests.conftest import golden_case_list, load_case


def qt_from_case(c) -> QuantizedTensor:
    bits, gs, dq, _ = (int(v) for v in c["params"])
    rows, cols = c["w"].shape
    padded = (cols + gs - 1) // gs * gs
    return QuantizedTensor(
        orig_shape=(rows, cols), orig_dtype=str(c["w_dtype"]), bits=bits, group_size=gs, rows=rows,
        cols=cols, padded_cols=padded, n_groups=padded // gs, packed=c["packed"], scale=c["scale"],
        gmin=c["gmin"], outlier_idx=c["outlier_idx"], outlier_val=c["outlier_val"],
        dq_scale_codes=c.get("dq_scale_codes"), dq_scale_meta=c.get("dq_scale_meta"),
        dq_gmin_codes=c.get("dq_gmin_codes"), dq_gmin_meta=c.get("dq_gmin_meta"),
        codebook=c.get("codebook"))


@pytest.mark.parametrize("name", golden_case_list())
def test_quantlinear_buffers_match_reference(golden, name):
    c = load_case(golden, name)
    bias = torch.from_numpy(c["bias"]) if "bias" in c else None
    ql = QuantLinear(qt_from_case(c), bias)
    np.testing.assert_array_equal(ql.outlier_row.numpy(), c["ql_outlier_row"])
    np.testing.assert_array_equal(ql.outlier_col.numpy(), c["ql_outlier_col"])
    np.testing.assert_array_equal(ql.outlier_delta.numpy().view(np.uint16),
                                  c["ql_outlier_delta"].view(np.uint16))
    ptr = ql.outlier_row_ptr.numpy()
    assert ptr[0] == 0 and ptr[-1] == len(c["ql_outlier_row"])
    for r in range(ql.rows):
        assert np.all(ql.outlier_row.numpy()[ptr[r]:ptr[r + 1]] == r)
    keys = set(ql.state_dict().keys())
    expect = {"packed", "outlier_row", "outlier_col", "outlier_delta"}
    expect |= ({"dq_scale_codes", "dq_scale_meta", "dq_gmin_codes", "dq_gmin_meta"}
               if "dq_scale_codes" in c else {"scale", "gmin"})
    if "codebook" in c:
        expect.add("codebook")
    if bias is not None:
        expect.add("bias")
    assert keys == expect
    assert ql.weight.dtype == torch.int8 and ql.weight.device.type == "meta"


@pytest.mark.parametrize("name", ["nf4_dq_g128", "u4_g128_pad", "lloyd2_g64"])
def test_to_quantized_tensor_roundtrip(golden, name):
    c = load_case(golden, name)
    qt = qt_from_case(c)
    back = QuantLinear(qt).to_quantized_tensor()
    np.testing.assert_array_equal(back.packed, qt.packed)
    order = np.argsort(back.outlier_idx)
    ref_order = np.argsort(qt.outlier_idx)
    np.testing.assert_array_equal(back.outlier_idx[order], qt.outlier_idx[ref_order])
    # val -> delta -> val is exact up to the fp16 rounding of delta
    np.testing.assert_allclose(back.outlier_val[order].astype(np.float32),
                               qt.outlier_val[ref_order].astype(np.float32), rtol=2e-3, atol=1e-4)


@pytest.mark.parametrize("name", golden_case_list())
def test_cpu_forward_matches_reference(golden, name):
    """A QuantLinear on the CPU runs the reference's CPU algorithm: its output
    equals the reference QuantLinear.forward output bit for bit."""
    c = load_case(golden, name)
    bias = torch.from_numpy(c["bias"]) if "bias" in c else None
    ql = QuantLinear(qt_from_case(c), bias=bias)
    x = torch.from_numpy(c["x"]).to(getattr(torch, str(c["x_dtype"])))
    y = ql(x)
    assert y.dtype == x.dtype
    np.testing.assert_array_equal(y.float().numpy(), c["y_cpu"].astype(np.float32))


def test_cpu_forward_rejects_mixed_devices(golden):
    c = load_case(golden, "nf4_dq_g128")
    ql = QuantLinear(qt_from_case(c))
    x = torch.zeros(1, ql.in_features, dtype=torch.float16, device="meta")
    with pytest.raises(RuntimeError, match="CUDA device, or both on the CPU"):
        ql(x)


def test_state_dict_roundtrip_rebuilds_row_ptr(golden):
    c = load_case(golden, "u4_g128_pad")
    a = QuantLinear(qt_from_case(c))
    b = QuantLinear(qt_from_case(c))
    b.outlier_row_ptr.zero_()
    b.load_state_dict(a.state_dict())
    np.testing.assert_array_equal(a.outlier_row_ptr.numpy(), b.outlier_row_ptr.numpy())


def test_n_outliers_rule():
    assert n_outliers_for(4096 * 4096, 0.001) == 16777
    assert n_outliers_for(10, 0.001) == 1
    assert n_outliers_for(10, 0.0) == 0


def test_budget_allocator():
    stats = [LayerBitStats("a", 100, 200, 0.1, 0.01), LayerBitStats("b", 100, 200, 0.1, 0.09)]
    assert budget_allocate_bits(stats, 300) == {"a": 8, "b": 4}
    assert budget_allocate_bits(stats, 200) == {"a": 4, "b": 4}
    assert budget_allocate_bits(stats, 1000) == {"a": 8, "b": 8}


def test_hf_config_registered_and_round_trips():
    from transformers.quantizers.auto import AutoHfQuantizer
    from tensorshrink_b200.hf_integration import TensorShrinkConfig
    c = TensorShrinkConfig(bits=8, adaptive=True, modules_to_not_convert=["lm_head"])
    assert AutoHfQuantizer.supports_quant_method(c.to_dict())
    back = TensorShrinkConfig.from_dict(c.to_dict())
    assert back.to_dict() == c.to_dict()
    assert type(AutoHfQuantizer.from_config(c)).__name__ == "TensorShrinkHfQuantizer"
    with pytest.raises(ValueError):
        TensorShrinkConfig(bits=6)
    with pytest.raises(NotImplementedError):
        TensorShrinkConfig(vram_budget_mb=100)


def test_budget_ties_keep_input_order():
    """Equal error-per-byte ratios are upgraded in the order given, as the
    reference's stable sort on the ratio alone does (codec.py:1025)."""
    stats = [LayerBitStats("z", 100, 200, 0.2, 0.1), LayerBitStats("a", 100, 200, 0.2, 0.1)]
    assert budget_allocate_bits(stats, 300) == {"z": 8, "a": 4}
