"""Fused MLP pieces: q/k/v-style row concatenation (`tp.concat_rows`) and
the gated down projection (`ts_qlinear_gated`: silu(gate) * up formed while
the decode kernel stages its activations) against the unfused computation
and the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import goap

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mlp():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import tensorshrink_b200 as ts
    out = []
    for j, shape in enumerate(((1536, 1024), (1536, 1024), (1024, 1536))):
        w = torch.from_numpy(goap.student_t_weights(shape, seed=40 + j)).cuda()
        out.append(ts.QuantLinear.from_device_quant(ts.quantize_device(w, bits=4, group_size=128,
                                                                       outlier_frac=0.002)))
    return out


def test_concat_rows_equals_separate(mlp):
    from tensorshrink_b200 import tp
    gate, up, _ = mlp
    fused = tp.concat_rows([gate, up])
    for M in (1, 5, 40, 300):
        x = torch.randn(M, 1024, device="cuda").to(torch.bfloat16)
        y, ref = fused(x), torch.cat([gate(x), up(x)], dim=-1)
        if M == 40:
            # split-K tensor-core plan: the K ranges of a row are cut where the
            # stage count of the whole layer puts them, so fp32 partial sums
            # of the fused and the separate layers are added in other groupings
            assert ((y.float() - ref.float()).abs().max() / ref.float().abs().max()).item() < 1e-2
        else:
            assert torch.equal(y, ref)


@pytest.mark.parametrize("M", [1, 3, 8, 12, 40])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_gated_down_matches_unfused_and_oracle(mlp, M, dtype):
    from tensorshrink_b200 import kernels, tp
    gate, up, down = mlp
    fused = tp.concat_rows([gate, up])
    x = torch.randn(M, 1024, device="cuda").to(dtype)
    gu = fused(x)
    y = kernels.qlinear_gated(gu, down.qweight(), None, torch.float32)
    m = F.silu(gu[:, :1536]) * gu[:, 1536:]
    ref = kernels.qlinear(m.contiguous(), down.qweight(), None, torch.float32)
    # silu's exp may differ by an ulp before the rounding to the activation dtype
    assert ((y - ref).abs().max() / ref.abs().max()).item() < 2e-3
    W = goap.dequantize(down.to_quantized_tensor())
    y_or = m.float().cpu().numpy() @ W.T
    assert goap.max_rel_error(y.cpu().numpy(), y_or) <= 1e-2


def test_torch_op_matches_c_abi(mlp):
    """QuantLinear.forward through torch.ops.tensorshrink.qlinear gives the
    C ABI's result bit for bit, and the operator has a Meta shape function."""
    from tensorshrink_b200 import _C, kernels
    ops = _C.torch_ops()
    assert ops is not None, "libtensorshrink_torch.so was not built"
    gate, _, down = mlp
    for ql in (gate, down):
        for M in (1, 20, 100):
            x = torch.randn(M, ql.in_features, device="cuda").to(torch.bfloat16)
            assert torch.equal(ql(x), kernels.qlinear(x, ql.qweight(), None, torch.bfloat16))
    xm = torch.empty(3, 7, 1024, device="meta", dtype=torch.float16)
    y = ops.qlinear(xm, gate.packed.to("meta"), None, None, None, None, None, None, None, None, None, None, None,
                    4, 128, 1024, 1536, 8, 0, torch.float32)
    assert y.shape == (3, 7, 1536) and y.dtype == torch.float32
