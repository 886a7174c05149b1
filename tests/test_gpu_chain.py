"""Fused decode calls (`ts_qlinear_ex`, `ts_qlinear_chain`): RMSNorm staged
in the decode kernel, the residual add in its epilogue, and chains of layers
run as one persistent launch, against the same layers run one call at a
time, the unfused torch ops and the oracle."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from oracle import goap

pytestmark = pytest.mark.gpu

H, I = 1024, 1536


def _layer(shape, seed, bits=4, **kw):
    import tensorshrink_b200 as ts
    w = torch.from_numpy(goap.student_t_weights(shape, seed=seed)).cuda()
    kw.setdefault("outlier_frac", 0.002)
    return ts.QuantLinear.from_device_quant(ts.quantize_device(w, bits=bits, group_size=128, **kw))


@pytest.fixture(scope="module")
def blocks():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from tensorshrink_b200 import tp
    out = []
    for b in range(4):
        gate, up, down = (_layer(s, 60 + 3 * b + j) for j, s in enumerate(((I, H), (I, H), (H, I))))
        out.append((tp.concat_rows([gate, up]), down))
    return out


def _sequential(blocks, x):
    """The blocks one ts_qlinear call at a time (gated down projection)."""
    from tensorshrink_b200 import kernels
    for gu_l, down in blocks:
        gu = kernels.qlinear(x, gu_l.qweight(), None, x.dtype)
        x = kernels.qlinear_gated(gu, down.qweight(), None, x.dtype)
    return x


def _chain_steps(blocks, x, outs):
    from tensorshrink_b200.kernels import ChainStep
    steps = []
    cur = x
    for (gu_l, down), (gu, y) in zip(blocks, outs):
        steps.append(ChainStep(gu_l.qweight(), cur, gu))
        steps.append(ChainStep(down.qweight(), gu, y, gated=True))
        cur = y
    return steps


@pytest.mark.parametrize("M", [1, 2, 5, 8])
@pytest.mark.parametrize("n_blocks", [1, 4])
def test_chain_equals_separate_launches(blocks, M, n_blocks):
    from tensorshrink_b200 import kernels
    bl = blocks[:n_blocks]
    x = torch.randn(M, H, device="cuda").to(torch.bfloat16)
    outs = [(torch.empty(M, 2 * I, device="cuda", dtype=torch.bfloat16),
             torch.empty(M, H, device="cuda", dtype=torch.bfloat16)) for _ in bl]
    before = kernels._C.load().ts_launch_count(1)
    kernels.qlinear_chain(_chain_steps(bl, x, outs), persistent=True)
    launches = kernels._C.load().ts_launch_count(1)
    assert launches == 1, f"a chain of {2 * n_blocks} layers took {launches} launches"
    del before
    ref = _sequential(bl, x)
    torch.cuda.synchronize()
    # one launch runs every layer in one build of the decode kernel, while
    # single calls pick the build per layer (one or two CTAs per SM, whose
    # warps split K differently): equal up to the fp32 summation order
    got = outs[-1][1].float()
    assert ((got - ref.float()).abs().max() / ref.float().abs().max()).item() < 1e-2
    # one launch per layer: the same calls as the sequential reference
    kernels.qlinear_chain(_chain_steps(bl, x, outs))
    assert torch.equal(outs[-1][1], ref)
    kernels.device_status()


def test_chain_repeats_and_replays_in_a_graph(blocks):
    """The chain counters return to zero after every launch: repeated calls
    and CUDA-graph replays give the same result."""
    from tensorshrink_b200 import kernels
    x = torch.randn(1, H, device="cuda").to(torch.bfloat16)
    outs = [(torch.empty(1, 2 * I, device="cuda", dtype=torch.bfloat16),
             torch.empty(1, H, device="cuda", dtype=torch.bfloat16)) for _ in blocks]
    steps = _chain_steps(blocks, x, outs)
    kernels.qlinear_chain(steps, persistent=True)
    first = outs[-1][1].clone()
    for _ in range(3):
        kernels.qlinear_chain(steps, persistent=True)
        assert torch.equal(outs[-1][1], first)
    kernels.qlinear_chain(steps)            # one launch per layer
    assert ((outs[-1][1].float() - first.float()).abs().max() / first.float().abs().max()).item() < 1e-2
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        kernels.qlinear_chain(steps, persistent=True)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        kernels.qlinear_chain(steps, persistent=True)
    for _ in range(5):
        outs[-1][1].zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(outs[-1][1], first)
    kernels.device_status()


def test_chain_of_mixed_layouts_runs_layer_by_layer():
    """A 2-bit layer then a 4-bit one cannot share one launch: the chain
    runs them as two launches with the same results."""
    from tensorshrink_b200 import kernels
    from tensorshrink_b200.kernels import ChainStep
    a = _layer((768, H), 90, bits=2)
    b = _layer((H, 768), 91, bits=4)
    x = torch.randn(3, H, device="cuda").to(torch.float16)
    t = torch.empty(3, 768, device="cuda", dtype=torch.float16)
    y = torch.empty(3, H, device="cuda", dtype=torch.float16)
    kernels._C.load().ts_launch_count(1)
    kernels.qlinear_chain([ChainStep(a.qweight(), x, t), ChainStep(b.qweight(), t, y)], persistent=True)
    assert kernels._C.load().ts_launch_count(1) == 2
    ref = kernels.qlinear(kernels.qlinear(x, a.qweight(), None, torch.float16), b.qweight(), None, torch.float16)
    assert torch.equal(y, ref)


@pytest.mark.parametrize("M", [1, 4, 8])
def test_rmsnorm_staging_matches_torch_and_oracle(blocks, M):
    from tensorshrink_b200 import kernels
    from tensorshrink_b200.kernels import ChainStep
    gu_l = blocks[0][0]
    h = torch.randn(M, H, device="cuda") * 3.0
    wn = torch.rand(H, device="cuda") + 0.5
    out = torch.empty(M, 2 * I, device="cuda", dtype=torch.float32)
    kernels.qlinear_chain([ChainStep(gu_l.qweight(), h, out, norm_weight=wn, norm_eps=1e-5,
                                     act_dtype=torch.bfloat16)])
    xn = F.rms_norm(h, (H,), wn, 1e-5).to(torch.bfloat16)
    ref = kernels.qlinear(xn, gu_l.qweight(), None, torch.float32)
    # the kernel's mean square is summed in another order than torch's: an
    # input can round to the neighbouring bf16 value
    assert ((out - ref).abs().max() / ref.abs().max()).item() < 5e-3
    W = goap.dequantize(gu_l.to_quantized_tensor())
    assert goap.max_rel_error(out.cpu().numpy(), xn.float().cpu().numpy() @ W.T) <= 1e-2


@pytest.mark.parametrize("M", [1, 6])
def test_residual_epilogue_in_place(blocks, M):
    from tensorshrink_b200 import kernels
    from tensorshrink_b200.kernels import ChainStep
    gu_l, down = blocks[1]
    gu = torch.randn(M, 2 * I, device="cuda").to(torch.bfloat16)
    h = torch.randn(M, H, device="cuda")
    h0 = h.clone()
    kernels.qlinear_chain([ChainStep(down.qweight(), gu, h, gated=True, residual=h)])
    y = kernels.qlinear_gated(gu, down.qweight(), None, torch.float32)
    assert torch.equal(h, h0 + y)


def test_decoder_mlp_chain_matches_unfused(blocks):
    """norm -> gate_up -> gated down + residual as one chain equals the
    unfused torch + qlinear sequence."""
    from tensorshrink_b200 import kernels
    from tensorshrink_b200.kernels import ChainStep
    gu_l, down = blocks[2]
    h = torch.randn(2, H, device="cuda")
    wn = torch.rand(H, device="cuda") + 0.5
    gu = torch.empty(2, 2 * I, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(2, H, device="cuda")
    kernels.qlinear_chain([ChainStep(gu_l.qweight(), h, gu, norm_weight=wn, act_dtype=torch.bfloat16),
                           ChainStep(down.qweight(), gu, out, gated=True, residual=h)])
    xn = F.rms_norm(h, (H,), wn, 1e-5).to(torch.bfloat16)
    gu_ref = kernels.qlinear(xn, gu_l.qweight(), None, torch.bfloat16)
    ref = h + kernels.qlinear_gated(gu_ref, down.qweight(), None, torch.float32)
    assert ((out - ref).abs().max() / ref.abs().max()).item() < 5e-3


def test_chain_wait_timeout_is_reported(blocks):
    """A stalled chain (test hook: the first layer's copies are never issued)
    runs its bounded waits out, returns, and reports through the status
    call; the next chain runs normally."""
    from tensorshrink_b200 import _C, kernels
    lib = _C.load()
    x = torch.randn(1, H, device="cuda").to(torch.bfloat16)
    outs = [(torch.empty(1, 2 * I, device="cuda", dtype=torch.bfloat16),
             torch.empty(1, H, device="cuda", dtype=torch.bfloat16)) for _ in blocks[:2]]
    steps = _chain_steps(blocks[:2], x, outs)
    _C.check(lib.ts_test_inject_stall(20_000_000), "stall")
    kernels.qlinear_chain(steps, persistent=True)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="bounded wait"):
        kernels.device_status()
    kernels.qlinear_chain(steps, persistent=True)
    torch.cuda.synchronize()
    kernels.device_status()
    ref = _sequential(blocks[:2], x).float()
    assert ((outs[-1][1].float() - ref).abs().max() / ref.abs().max()).item() < 1e-2
