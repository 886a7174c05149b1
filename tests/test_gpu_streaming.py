"""StreamingQuantModel: a stack of QuantLinear layers (uniform, NF4 with
double quantization, Lloyd-Max, with biases) run with their buffers
streamed from pinned host memory gives bit-identical outputs to the same
layers resident on the device, for prefetch depths 1 and 2, across repeated
forwards; disable() restores host-resident layers."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def stack():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import tensorshrink_b200 as ts
    torch.manual_seed(0)
    dims = [1024, 2048, 1536, 1024, 512]
    kinds = [dict(nf_quant=False, double_quant=False), dict(nf_quant=True, double_quant=True),
             dict(companded=True, bits=2, group_size=64), dict(nf_quant=False, double_quant=True, bits=8)]
    layers = []
    for i, kw in enumerate(kinds):
        w = (torch.randn(dims[i + 1], dims[i], device="cuda") * 0.02).half()
        kw = dict(dict(bits=4, group_size=128, outlier_frac=0.002), **kw)
        d = ts.quantize_device(w, **kw)
        layers.append(ts.QuantLinear.from_device_quant(d, bias=torch.randn(dims[i + 1], device="cuda").half()))
    return torch.nn.Sequential(*layers)


def _clone(model):
    import copy
    return copy.deepcopy(model)


@pytest.mark.parametrize("depth", [1, 2])
def test_streamed_equals_resident(stack, depth):
    from tensorshrink_b200.streaming import stream_offload_module
    x = torch.randn(3, 1024, device="cuda").half()
    ref = stack(x)
    model = _clone(stack)
    st = stream_offload_module(model, prefetch_depth=depth, verbose=False)
    assert all(not m.packed.is_cuda for m in model)
    for _ in range(3):
        y = model(x)
        assert torch.equal(y, ref)
    s = st.stats()
    assert s["n_layers"] == 4 and s["layers_currently_on_gpu"] <= depth
    st.disable()
    assert all(not m.packed.is_cuda for m in model)
    assert all(m.packed.is_pinned() for m in model)
