"""A Llama-shaped decoder whose projections are QuantLinear layers: the
caller of the hot path that the decode tok/s and tensor-parallel
measurements run through.

The reference quantizes the projections of a Hugging Face Llama
(`quantize_module`, modules.py:1258-1455, skipping embed/lm_head/norms by
name, modules.py:62) and serves it through `CUDAGraphQuantModel`
(modules.py:1589-1691). This module builds the same structure directly on
the device with random weights (no checkpoint): seeded Student-t(df=4)
projection weights with std 0.02, quantized on the GPU with a seeded
per-layer bit width, plus plain-torch RMSNorm, rotary embeddings and
grouped-query attention over a static KV cache, so one decode step is
capturable in a CUDA graph.

Tensor parallelism (one process per GPU): q/k/v and gate/up are
column-parallel (whole heads per rank), o and down row-parallel with one
all-reduce each per layer, the lm_head is split over the vocabulary and the
next token is the global argmax of the per-rank maxima. The all-reduce is
the library's one-shot NVLink kernel when a `PeerExchange` is given, else
torch.distributed (NCCL).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import numpy as np
import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import nn

from .codec import quantize_device
from .modules import QuantLinear


@dataclass
class DecoderConfig:
    n_layers: int = 32
    hidden: int = 4096
    n_heads: int = 32
    n_kv_heads: int = 8
    intermediate: int = 14336
    vocab: int = 128256
    rope_theta: float = 500000.0
    rms_eps: float = 1e-5
    group_size: int = 128
    outlier_frac: float = 0.001
    bits_choices: Sequence[int] = (2, 4, 8)
    double_quant: bool = False
    nf_quant: bool = False
    seed: int = 0
    layer_bits: Optional[List[int]] = field(default=None)

    @property
    def head_dim(self) -> int:
        return self.hidden // self.n_heads

    def bits_per_layer(self) -> List[int]:
        """The seeded per-layer bit widths (a fixed draw over bits_choices)."""
        if self.layer_bits is not None:
            return list(self.layer_bits)
        rng = np.random.default_rng(self.seed)
        return [int(b) for b in rng.choice(np.asarray(self.bits_choices), size=self.n_layers)]


def llama3_8b_config(**kw) -> DecoderConfig:
    """Llama-3-8B shapes, per-layer bits drawn from 2/4/8."""
    return DecoderConfig(**kw)


def llama_70b_config(**kw) -> DecoderConfig:
    """Llama-70B shapes, 4-bit g128 double-quant NF4."""
    base = dict(n_layers=80, hidden=8192, n_heads=64, n_kv_heads=8, intermediate=28672,
                bits_choices=(4,), double_quant=True, nf_quant=True)
    base.update(kw)
    return DecoderConfig(**base)


def student_t_weight(shape, seed: int, device, std: float = 0.02) -> torch.Tensor:
    """Seeded Student-t(df=4) fp16 weights rescaled to `std`, drawn on the device."""
    g = torch.Generator(device=device).manual_seed(int(seed))
    z = torch.randn(shape, generator=g, device=device)
    chi = torch.zeros(shape, device=device)
    for _ in range(4):
        chi += torch.randn(shape, generator=g, device=device).square()
    w = z / torch.sqrt(chi / 4.0)
    w *= std / w.std()
    return w.to(torch.float16)


def _group_info(group):
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(group), dist.get_rank(group)
    return 1, 0


def _rms_norm(h: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm of the fp32 residual stream `h` with fp32 weights, to bf16
    (the projections' activation dtype)."""
    return F.rms_norm(h, (h.shape[-1],), w, eps).to(torch.bfloat16)


class ShardedProjection(nn.Module):
    """A QuantLinear shard: this rank's output rows [r0, r1) (column-parallel)
    or input columns [c0, c1) (row-parallel: the caller all-reduces)."""

    def __init__(self, ql: QuantLinear, world: int, rank: int, kind: str, align: int = 1):
        super().__init__()
        from . import tp
        self.kind = kind
        if world == 1:
            self.local = ql
            self.lo, self.hi = 0, ql.rows if kind == "column" else ql.cols
        elif kind == "column":
            self.lo, self.hi = tp.shard_bounds(ql.rows, world, rank, align)
            self.local = tp.shard_rows(ql, self.lo, self.hi)
        else:
            c0, c1 = tp.shard_bounds(ql.padded_cols, world, rank, ql.group_size)
            self.lo, self.hi = c0, min(c1, ql.cols)
            self.local = tp.shard_cols(ql, self.lo, self.hi)

    def forward(self, x: torch.Tensor, out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
        from . import kernels
        x2d = x.reshape(-1, x.shape[-1])
        if not x2d.is_contiguous():
            x2d = x2d.contiguous()
        y = kernels.qlinear(x2d, self.local.qweight(), self.local.bias, out_dtype or x.dtype)
        return y.reshape(*x.shape[:-1], y.shape[-1])


def _gated(self, gate_up: torch.Tensor, out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """This layer applied to silu(gate) * up, gate_up = [gate | up] (the
    output of the fused gate/up projection): one fused launch at decode."""
    from . import kernels
    g2d = gate_up.reshape(-1, gate_up.shape[-1])
    y = kernels.qlinear_gated(g2d, self.local.qweight(), self.local.bias, out_dtype or gate_up.dtype)
    return y.reshape(*gate_up.shape[:-1], y.shape[-1])


ShardedProjection.gated = _gated


class FusedProjection(nn.Module):
    """A QuantLinear called through kernels.qlinear (rows of several
    projections)."""

    def __init__(self, ql: QuantLinear):
        super().__init__()
        self.local = ql

    def forward(self, x: torch.Tensor, out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
        from . import kernels
        x2d = x.reshape(-1, x.shape[-1])
        if not x2d.is_contiguous():
            x2d = x2d.contiguous()
        y = kernels.qlinear(x2d, self.local.qweight(), self.local.bias, out_dtype or x.dtype)
        return y.reshape(*x.shape[:-1], y.shape[-1])


class QuantDecoderLayer(nn.Module):
    def __init__(self, cfg: DecoderConfig, layer_idx: int, bits: int, device, world: int = 1, rank: int = 0):
        super().__init__()
        self.cfg = cfg
        self.world, self.rank = world, rank
        H, D, F_ = cfg.hidden, cfg.head_dim, cfg.intermediate
        shapes = {"q_proj": (cfg.n_heads * D, H), "k_proj": (cfg.n_kv_heads * D, H),
                  "v_proj": (cfg.n_kv_heads * D, H), "o_proj": (H, cfg.n_heads * D),
                  "gate_proj": (F_, H), "up_proj": (F_, H), "down_proj": (H, F_)}
        kinds = {"q_proj": "column", "k_proj": "column", "v_proj": "column", "o_proj": "row",
                 "gate_proj": "column", "up_proj": "column", "down_proj": "row"}
        self.bits = bits
        for j, (name, shape) in enumerate(shapes.items()):
            w = student_t_weight(shape, seed=cfg.seed * 100003 + layer_idx * 16 + j, device=device)
            dq = quantize_device(w, bits=bits, group_size=cfg.group_size, outlier_frac=cfg.outlier_frac,
                                 double_quant=cfg.double_quant, nf_quant=cfg.nf_quant)
            del w
            ql = QuantLinear.from_device_quant(dq)
            align = D if name in ("q_proj", "k_proj", "v_proj") else 1
            setattr(self, name, ShardedProjection(ql, world, rank, kinds[name], align))
            del ql, dq
        self.n_heads_local = cfg.n_heads // world
        self.n_kv_local = cfg.n_kv_heads // world
        # this rank's q/k/v and gate/up shards fused into one launch each
        # (rows concatenated; every row reconstructs exactly as before)
        from .tp import concat_rows
        self.qkv = FusedProjection(concat_rows([self.q_proj.local, self.k_proj.local, self.v_proj.local]))
        self.gate_up = FusedProjection(concat_rows([self.gate_proj.local, self.up_proj.local]))
        self.splits_qkv = [self.q_proj.local.rows, self.k_proj.local.rows, self.v_proj.local.rows]
        self.split_gate = self.gate_proj.local.rows
        del self.q_proj, self.k_proj, self.v_proj, self.gate_proj, self.up_proj
        self.input_norm = nn.Parameter(torch.ones(H, dtype=torch.float32, device=device), requires_grad=False)
        self.post_norm = nn.Parameter(torch.ones(H, dtype=torch.float32, device=device), requires_grad=False)

    def projections(self):
        """The layers one forward runs (fused q/k/v and gate/up)."""
        return [self.qkv, self.o_proj, self.gate_up, self.down_proj]


class QuantDecoder(nn.Module):
    """Llama-shaped decoder over QuantLinear projections (see module doc)."""

    def __init__(self, cfg: DecoderConfig, device, group=None, exchange=None, max_batch: int = 1,
                 max_seq: int = 2048):
        super().__init__()
        self.cfg = cfg
        self.group = group
        self.exchange = exchange
        self.world, self.rank = _group_info(group)
        if cfg.n_heads % self.world or cfg.n_kv_heads % self.world:
            raise ValueError(f"{self.world} ranks do not divide {cfg.n_heads} q / {cfg.n_kv_heads} kv heads")
        self.device = torch.device(device)
        H, D = cfg.hidden, cfg.head_dim
        g = torch.Generator(device=self.device).manual_seed(cfg.seed + 7)
        # embed / lm_head stay unquantized (the reference skips them by name)
        self.embed = (torch.randn(cfg.vocab, H, generator=g, device=self.device) * 0.02).to(torch.bfloat16)
        v0, v1 = self._vocab_bounds(self.rank)
        # every rank draws the whole head and keeps its vocabulary slice, so
        # the sharded model is the unsharded one cut up
        full = (torch.randn(cfg.vocab, H, generator=g, device=self.device) * 0.02).to(torch.bfloat16)
        self.lm_head = full[v0:v1].contiguous()
        del full
        self.final_norm = torch.ones(H, dtype=torch.float32, device=self.device)
        self.layer_bits = cfg.bits_per_layer()
        self.layers = nn.ModuleList(
            QuantDecoderLayer(cfg, i, b, self.device, self.world, self.rank) for i, b in enumerate(self.layer_bits))
        # rotary tables
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, D, 2, device=self.device, dtype=torch.float32) / D))
        t = torch.arange(max_seq, device=self.device, dtype=torch.float32)
        ang = torch.outer(t, inv)
        self.rope_cos, self.rope_sin = ang.cos(), ang.sin()
        self.max_batch, self.max_seq = max_batch, max_seq
        nkv = cfg.n_kv_heads // self.world
        shape = (cfg.n_layers, max_batch, nkv, max_seq, D)
        self.k_cache = torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
        self.v_cache = torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
        # decode steps through the fused kernels (RMSNorm staged in the
        # projections, residual adds in their epilogues, one attention kernel,
        # the MLP as one chained launch); False: the plain torch + qlinear ops
        self.fused_decode = True
        self._dbufs = {}

    def _vocab_bounds(self, rank):
        per = -(-self.cfg.vocab // self.world)
        return rank * per, min(self.cfg.vocab, (rank + 1) * per)

    # -- accounting -------------------------------------------------------------------
    def packed_nbytes(self) -> int:
        """Quantized bytes this rank streams per decode step."""
        return sum(p.local.packed_nbytes() for layer in self.layers for p in layer.projections())

    # -- pieces -------------------------------------------------------------------------
    def _reduce_add(self, partial: torch.Tensor, h: torch.Tensor) -> torch.Tensor:
        """h + the sum over ranks of a row-parallel fp32 partial."""
        if self.world == 1:
            return h + partial
        if self.exchange is not None and partial.numel() <= self.exchange.cap:
            # decode-sized exchanges: the one-shot kernel (residual add fused)
            return self.exchange.all_reduce(partial.contiguous(), residual=h.contiguous())
        dist.all_reduce(partial, group=self.group)
        return h + partial

    def _rope(self, x: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        # x [B, T, h, D]; pos [T] absolute positions
        cos = self.rope_cos[pos][None, :, None, :]
        sin = self.rope_sin[pos][None, :, None, :]
        x1, x2 = x.float().chunk(2, dim=-1)
        return torch.cat([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1).to(x.dtype)

    def _layer(self, i: int, layer: QuantDecoderLayer, h: torch.Tensor, pos: torch.Tensor,
               mask: Optional[torch.Tensor], attn_len: int = 0) -> torch.Tensor:
        cfg = self.cfg
        B, T, _ = h.shape
        D = cfg.head_dim
        x = _rms_norm(h, layer.input_norm, cfg.rms_eps)
        q, k, v = layer.qkv(x).split(layer.splits_qkv, dim=-1)
        q = self._rope(q.view(B, T, layer.n_heads_local, D), pos)
        k = self._rope(k.view(B, T, layer.n_kv_local, D), pos)
        v = v.view(B, T, layer.n_kv_local, D)
        kc, vc = self.k_cache[i, :B], self.v_cache[i, :B]
        kc.index_copy_(2, pos, k.transpose(1, 2))
        vc.index_copy_(2, pos, v.transpose(1, 2))
        if mask is None:
            # prefill from position 0: causal attention over the T new tokens
            a = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                               is_causal=True, enable_gqa=True)
        else:
            # decode: attend to the first L cache positions, masked to < pos + 1
            # (a device-side mask, so every position replays the same graph)
            L = mask.shape[-1]
            a = F.scaled_dot_product_attention(q.transpose(1, 2), kc[:, :, :L], vc[:, :, :L], attn_mask=mask,
                                               enable_gqa=True)
        a = a.transpose(1, 2).reshape(B, T, layer.n_heads_local * D)
        h = self._reduce_add(layer.o_proj(a, torch.float32), h)
        x = _rms_norm(h, layer.post_norm, cfg.rms_eps)
        gu = layer.gate_up(x)
        return self._reduce_add(layer.down_proj.gated(gu, torch.float32), h)

    def _decode_buffers(self, B: int) -> dict:
        bufs = self._dbufs.get(B)
        if bufs is None:
            l0 = self.layers[0]
            D, dev = self.cfg.head_dim, self.device
            bufs = {"qkv": torch.empty(B, sum(l0.splits_qkv), dtype=torch.bfloat16, device=dev),
                    "attn": torch.empty(B, l0.n_heads_local * D, dtype=torch.bfloat16, device=dev),
                    "gu": torch.empty(B, 2 * l0.split_gate, dtype=torch.bfloat16, device=dev),
                    "part": torch.empty(B, self.cfg.hidden, dtype=torch.float32, device=dev)}
            self._dbufs[B] = bufs
        return bufs

    def _layer_decode(self, i: int, layer: QuantDecoderLayer, h: torch.Tensor, pos: torch.Tensor,
                      attn_len: int) -> torch.Tensor:
        """One layer of a decode step on the fp32 residual stream h [B, H],
        updated in place: q/k/v projection with the input RMSNorm staged in
        its kernel, the attention kernel (rope + cache append + GQA), then
        o_proj (+ residual), gate/up (post RMSNorm staged) and the gated down
        projection (+ residual) as one chained launch. With tensor
        parallelism the row-parallel partials go through the exchange (or
        NCCL) with the residual add fused there."""
        from .kernels import ChainStep, decode_attention, qlinear_chain
        cfg = self.cfg
        b = self._decode_buffers(h.shape[0])
        bf16 = torch.bfloat16
        qkv, gu = layer.qkv.local, layer.gate_up.local
        qlinear_chain([ChainStep(qkv.qweight(), h, b["qkv"], bias=qkv.bias, norm_weight=layer.input_norm,
                                 norm_eps=cfg.rms_eps, act_dtype=bf16)])
        decode_attention(b["qkv"], layer.n_heads_local, layer.n_kv_local, cfg.head_dim, pos, self.rope_cos,
                         self.rope_sin, self.k_cache[i], self.v_cache[i], attn_len, out=b["attn"])
        o, down = layer.o_proj.local, layer.down_proj.local

        def up_steps(h_in):
            # gate/up read the residual stream after the attention block's add
            return [ChainStep(gu.qweight(), h_in, b["gu"], bias=gu.bias, norm_weight=layer.post_norm,
                              norm_eps=cfg.rms_eps, act_dtype=bf16)]
        if self.world == 1:
            # o_proj adds into h in place, so the chain's later steps see it
            qlinear_chain([ChainStep(o.qweight(), b["attn"], h, bias=o.bias, residual=h)] + up_steps(h)
                          + [ChainStep(down.qweight(), b["gu"], h, bias=down.bias, gated=True, residual=h)])
            return h
        qlinear_chain([ChainStep(o.qweight(), b["attn"], b["part"], bias=o.bias if self.rank == 0 else None)])
        # the reduction returns a new residual tensor: gate/up must read that one
        h = self._reduce_add(b["part"], h)
        qlinear_chain(up_steps(h) + [ChainStep(down.qweight(), b["gu"], b["part"],
                                            bias=down.bias if self.rank == 0 else None, gated=True)])
        return self._reduce_add(b["part"], h)

    def _next_token(self, h_last: torch.Tensor) -> torch.Tensor:
        """Greedy next token: global argmax over the vocabulary shards."""
        x = _rms_norm(h_last, self.final_norm, self.cfg.rms_eps)
        logits = F.linear(x, self.lm_head).float()              # [B, local vocab]
        val, idx = logits.max(dim=-1)
        if self.world == 1:
            return idx
        v0, _ = self._vocab_bounds(self.rank)
        pair = torch.stack([val, (idx + v0).float()], dim=-1)   # [B, 2]
        parts = [torch.empty_like(pair) for _ in range(self.world)]
        dist.all_gather(parts, pair, group=self.group)
        allp = torch.stack(parts, dim=0)                         # [world, B, 2]
        best = allp[..., 0].argmax(dim=0)                        # first rank wins ties
        return allp[best, torch.arange(pair.shape[0], device=pair.device), 1].long()

    # -- entry points ------------------------------------------------------------------
    def _logits(self, h_last: torch.Tensor) -> torch.Tensor:
        """fp32 logits [B, vocab] of the last position (gathered over the
        vocabulary shards)."""
        x = _rms_norm(h_last, self.final_norm, self.cfg.rms_eps)
        logits = F.linear(x, self.lm_head).float()
        if self.world == 1:
            return logits
        per = -(-self.cfg.vocab // self.world)
        pad = per - logits.shape[-1]
        lp = F.pad(logits, (0, pad)) if pad else logits
        parts = [torch.empty_like(lp) for _ in range(self.world)]
        dist.all_gather(parts, lp.contiguous(), group=self.group)
        return torch.cat(parts, dim=-1)[:, : self.cfg.vocab]

    @torch.no_grad()
    def prefill(self, tokens: torch.Tensor, return_logits: bool = False) -> torch.Tensor:
        """Run `tokens` [B, T] from position 0; fills the KV cache; returns the
        greedy next token [B], or with `return_logits` the last position's
        fp32 logits [B, vocab]."""
        B, T = tokens.shape
        pos = torch.arange(T, device=tokens.device)
        h = self.embed[tokens].float()
        for i, layer in enumerate(self.layers):
            h = self._layer(i, layer, h, pos, None)
        return self._logits(h[:, -1]) if return_logits else self._next_token(h[:, -1])

    @torch.no_grad()
    def decode_step(self, tokens: torch.Tensor, pos: torch.Tensor, attn_len: int = 0,
                    return_logits: bool = False) -> torch.Tensor:
        """One token per sequence: `tokens` [B] at position `pos` (a one-element
        int64 device tensor, advanced by the caller). Attention reads the first
        `attn_len` cache positions (default all), masked to those <= pos.
        Returns the next tokens (or the fp32 logits)."""
        L = attn_len or self.max_seq
        if self.fused_decode:
            h = self.embed[tokens].float()
            for i, layer in enumerate(self.layers):
                h = self._layer_decode(i, layer, h, pos, L)
            return self._logits(h) if return_logits else self._next_token(h)
        h = self.embed[tokens][:, None, :].float()
        mask = (torch.arange(L, device=h.device) <= pos)[None, None, None, :]
        for i, layer in enumerate(self.layers):
            h = self._layer(i, layer, h, pos, mask, L)
        return self._logits(h[:, 0]) if return_logits else self._next_token(h[:, 0])


class CUDAGraphDecoder:
    """One decode step of a QuantDecoder captured as a CUDA graph
    (the role of the reference's CUDAGraphQuantModel, modules.py:1589-1691):
    static token and position buffers, replayed once per generated token."""

    def __init__(self, model: QuantDecoder, batch: int, warmup: int = 2, attn_len: int = 0):
        self.model = model
        dev = model.device
        self.tokens = torch.zeros(batch, dtype=torch.long, device=dev)
        self.pos = torch.zeros(1, dtype=torch.long, device=dev)
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(warmup):
                model.decode_step(self.tokens, self.pos, attn_len)
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.next_tokens = model.decode_step(self.tokens, self.pos, attn_len)
            self.tokens.copy_(self.next_tokens)
            self.pos.add_(1)

    def start(self, tokens: torch.Tensor, pos: int) -> None:
        self.tokens.copy_(tokens)
        self.pos.fill_(pos)

    def step(self) -> None:
        self.graph.replay()
