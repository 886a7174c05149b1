"""The Llama-shaped QuantDecoder (the decode tok/s workload) on a small
shape: its prefill and decode steps against a dense fp32 restatement of the
same network built from the layers' oracle-dequantized weights, and the CUDA
graph decode loop against eager decode steps.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from tensorshrink_b200.decoder import DecoderConfig, QuantDecoder
    cfg = DecoderConfig(n_layers=3, hidden=512, n_heads=8, n_kv_heads=2, intermediate=1024, vocab=3000,
                        layer_bits=[2, 4, 8], seed=3)
    return QuantDecoder(cfg, "cuda", max_batch=2, max_seq=64)


def _dense_forward(m, tokens):
    """fp32 reference: same network, dequantized weights, full causal attention."""
    cfg = m.cfg
    D = cfg.head_dim
    B, T = tokens.shape
    h = m.embed[tokens].float()
    pos = torch.arange(T, device=tokens.device)
    cos, sin = m.rope_cos[pos][None, :, None, :], m.rope_sin[pos][None, :, None, :]

    def rope(x):
        x1, x2 = x.chunk(2, dim=-1)
        return torch.cat([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1)

    def norm(x, w):
        return x * torch.rsqrt(x.square().mean(-1, keepdim=True) + cfg.rms_eps) * w.float()

    def W(p):
        return p.local.dequantize(torch.float32)

    for layer in m.layers:
        x = norm(h, layer.input_norm)
        Wq, Wk, Wv = W(layer.qkv).split(layer.splits_qkv, dim=0)
        q = rope((x @ Wq.T).view(B, T, -1, D))
        k = rope((x @ Wk.T).view(B, T, -1, D))
        v = (x @ Wv.T).view(B, T, -1, D)
        a = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                           is_causal=True, enable_gqa=True)
        h = h + a.transpose(1, 2).reshape(B, T, -1) @ W(layer.o_proj).T
        x = norm(h, layer.post_norm)
        Wg, Wu = W(layer.gate_up).split([layer.split_gate] * 2, dim=0)
        h = h + (F.silu(x @ Wg.T) * (x @ Wu.T)) @ W(layer.down_proj).T
    x = norm(h[:, -1], m.final_norm)
    return x @ m.lm_head.float().T


def test_layer_bits_are_the_seeded_draw(model):
    assert model.layer_bits == [2, 4, 8]
    assert [layer.qkv.local.bits for layer in model.layers] == [2, 4, 8]
    from tensorshrink_b200.decoder import DecoderConfig
    a, b = DecoderConfig(seed=5).bits_per_layer(), DecoderConfig(seed=5).bits_per_layer()
    assert a == b and len(a) == 32 and set(a) <= {2, 4, 8}


def test_prefill_matches_dense_reference(model):
    g = torch.Generator(device="cuda").manual_seed(0)
    tokens = torch.randint(0, model.cfg.vocab, (2, 12), device="cuda", generator=g)
    ref_logits = _dense_forward(model, tokens)
    nxt = model.prefill(tokens)
    ref_top2 = ref_logits.topk(2, dim=-1)
    for b in range(2):
        # bf16 activations: accept the reference's runner-up when the two are within noise
        gap = (ref_top2.values[b, 0] - ref_top2.values[b, 1]).item()
        assert nxt[b].item() == ref_top2.indices[b, 0].item() or gap < 0.05 * ref_logits[b].abs().max().item()


def test_decode_steps_match_prefill(model):
    """Prefill T-1 tokens then one decode step at position T-1 sees the same
    context as a prefill of all T tokens."""
    g = torch.Generator(device="cuda").manual_seed(1)
    tokens = torch.randint(0, model.cfg.vocab, (2, 9), device="cuda", generator=g)
    full = model.prefill(tokens, return_logits=True)
    model.prefill(tokens[:, :-1])
    step = model.decode_step(tokens[:, -1].contiguous(), torch.tensor([8], device="cuda"), return_logits=True)
    # prefill and decode run different kernels (18 vs 2 token rows): bf16-level agreement
    assert ((full - step).abs().max() / full.abs().max()).item() < 2e-2


def test_cuda_graph_decode_matches_eager(model):
    from tensorshrink_b200.decoder import CUDAGraphDecoder
    g = torch.Generator(device="cuda").manual_seed(2)
    tokens = torch.randint(0, model.cfg.vocab, (2, 6), device="cuda", generator=g)
    first = model.prefill(tokens)
    eager = [first]
    pos = 6
    cur = first
    for _ in range(4):
        cur = model.decode_step(cur, torch.tensor([pos], device="cuda"))
        eager.append(cur)
        pos += 1
    model.prefill(tokens)
    runner = CUDAGraphDecoder(model, batch=2)
    model.prefill(tokens)            # the warm-up inside the runner wrote the cache
    runner.start(first, 6)
    got = [first.clone()]
    for _ in range(4):
        runner.step()
        got.append(runner.tokens.clone())
    torch.cuda.synchronize()
    for a, b in zip(eager, got):
        assert torch.equal(a, b)


def test_fused_decode_matches_unfused(model):
    """The fused decode step (norms staged in the projections, residual
    epilogues, the attention kernel, chained MLP) against the plain torch +
    qlinear step on the same cache contents."""
    g = torch.Generator(device="cuda").manual_seed(4)
    tokens = torch.randint(0, model.cfg.vocab, (2, 7), device="cuda", generator=g)
    pos = torch.tensor([7], device="cuda")
    nxt = torch.randint(0, model.cfg.vocab, (2,), device="cuda", generator=g)
    model.prefill(tokens)
    model.fused_decode = False
    try:
        ref = model.decode_step(nxt, pos, attn_len=16, return_logits=True)
    finally:
        model.fused_decode = True
    model.prefill(tokens)
    got = model.decode_step(nxt, pos, attn_len=16, return_logits=True)
    assert ((got - ref).abs().max() / ref.abs().max()).item() < 1e-2


@pytest.mark.parametrize("B,nq,nkv,pos,L", [(1, 8, 2, 0, 8), (2, 8, 2, 5, 16), (3, 4, 4, 20, 16), (1, 16, 2, 40, 64)])
def test_decode_attention_kernel_matches_sdpa(B, nq, nkv, pos, L):
    from tensorshrink_b200.kernels import decode_attention
    D, S = 64, 64
    g = torch.Generator(device="cuda").manual_seed(B * 100 + pos)
    qkv = torch.randn(B, (nq + 2 * nkv) * D, device="cuda", generator=g).to(torch.bfloat16)
    kc = torch.randn(B, nkv, S, D, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(B, nkv, S, D, device="cuda", generator=g).to(torch.bfloat16)
    inv = 1.0 / (10000.0 ** (torch.arange(0, D, 2, device="cuda", dtype=torch.float32) / D))
    ang = torch.outer(torch.arange(S, device="cuda", dtype=torch.float32), inv)
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    kref, vref = kc.clone(), vc.clone()

    def rope(x):   # x [B, h, D] at position pos
        x1, x2 = x.float().chunk(2, dim=-1)
        c, s = cos[pos], sin[pos]
        return torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1).to(torch.bfloat16)

    q = rope(qkv[:, :nq * D].view(B, nq, D))
    k = rope(qkv[:, nq * D:(nq + nkv) * D].view(B, nkv, D))
    v = qkv[:, (nq + nkv) * D:].view(B, nkv, D)
    kref[:, :, pos] = k
    vref[:, :, pos] = v
    mask = (torch.arange(L, device="cuda") <= pos)[None, None, None, :]
    ref = F.scaled_dot_product_attention(q[:, :, None].float(), kref[:, :, :L].float(), vref[:, :, :L].float(),
                                         attn_mask=mask, enable_gqa=True)[:, :, 0].reshape(B, nq * D)
    out = decode_attention(qkv, nq, nkv, D, torch.tensor([pos], device="cuda"), cos, sin, kc, vc, L)
    assert torch.equal(kc, kref) and torch.equal(vc, vref)
    assert ((out.float() - ref).abs().max()).item() < 2e-2
