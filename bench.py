"""Benchmark of the QuantLinear hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--M 1] [--blocks 4]

Workload: Llama-style MLP blocks, hidden 4096,
intermediate 14336 (gate/up [14336, 4096], down [4096, 14336], SiLU-gated),
weights Student-t(df=4) std 0.02 quantized on the GPU to 4-bit g128 uniform
+ 0.1% outliers, bf16 activations, decode M=1. One step = one forward of the
activations through `--blocks` distinct MLP blocks (4 blocks = 381 MB of
packed weights, 3x the 126 MB L2, so every step streams from HBM).

Metric: packed-weight HBM GB/s = algorithmic bytes per step (packed codes +
scale/gmin + outlier tables + activations in/out) / step time. `value` is
measured device-side over a CUDA-graph replay of K steps; `e2e` runs the same
steps through the public module API with the input copied from pinned host
memory and the output copied back inside the timed region.

Multi-GPU (torchrun, one process per GPU): the blocks are tensor-parallel
(gate/up column-parallel, down row-parallel with its fp32 partial sums summed
by the library's one-shot NVLink all-reduce kernel, or NCCL with --nccl), so
the total work is fixed ("scaling": "strong"); time is the max over ranks.

The same JSON line carries a `prefill` object: TFLOP/s of the BASELINE
configs[2] layer ([8192, 8192], 2-bit Lloyd-Max g64, 0.1% outliers) at M=2048
bf16 on the tensor-core kernel, each launch timed alone after an L2 flush,
and a `quantize` object: fp16-input GB/s of the GPU quantize/pack on the
BASELINE configs[4] [28672, 8192] shape (4-bit g128, double quant).

--impl reference times the unmodified reference (installed into baseline/_ref
by baseline/install_ref.py): its QuantLinear.forward CPU path on one full MLP
block on all host threads as `value`, and, on a GPU host, its own CUDA/Triton
path on the same blocks as `gpu_anchor`. Without the install it falls back to
the oracle's numpy port of the CPU path.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "QuantLinear packed-weight HBM GB/s (M=1) & TFLOP/s (M=2048); decode tok/s"
HIDDEN, INTER = 4096, 14336
# DRAM bytes per launch (read + write) measured by ncu on this workload
QGEMV_TRAFFIC_BYTES = 31_679_488
# whether the timed one-GPU step runs as one persistent chained launch (see
# mlp_step); measured slower than one launch per layer, so kept off
STEP_CHAIN = False
QGEMM_TRAFFIC_BYTES = 56_665_088 + 8_519_168


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


# ---------------------------------------------------------------------------
# clocks: NVML polled from a thread during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nvml = None
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for bit, name in self.REASONS.items():
                    if r & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self._nvml is not None:
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._nvml is not None:
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------

def student_t_cuda(shape, seed, device):
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    z = torch.randn(shape, generator=g, device=device)
    chi = torch.zeros(shape, device=device)
    for _ in range(4):
        chi += torch.randn(shape, generator=g, device=device).square()
    w = z / torch.sqrt(chi / 4.0)
    w *= 0.02 / w.std()
    return w.to(torch.float16)


def build_blocks(n_blocks, device, seed0=0, world=1, rank=0):
    """n_blocks MLP blocks of QuantLinear (4-bit g128 uniform + outliers).
    With world > 1 each block is tensor-parallel: this rank keeps its
    column shard of gate/up and its row shard of down (whole layers are
    quantized identically on every rank, then cut)."""
    import torch
    import tensorshrink_b200 as ts
    from tensorshrink_b200.decoder import FusedProjection, ShardedProjection
    from tensorshrink_b200.tp import concat_rows
    blocks = []
    for b in range(n_blocks):
        layers = []
        for j, shape in enumerate(((INTER, HIDDEN), (INTER, HIDDEN), (HIDDEN, INTER))):
            w = student_t_cuda(shape, seed0 + 10 * b + j, device)
            dq = ts.quantize_device(w, bits=4, group_size=128, outlier_frac=0.001, double_quant=False,
                                    nf_quant=False)
            ql = ts.QuantLinear.from_device_quant(dq)
            del w, dq
            layers.append(ShardedProjection(ql, world, rank, "row" if j == 2 else "column"))
        # gate and up rows fused into one launch (the same weights, codes and
        # outliers), the down projection fed [gate | up] directly
        gate_up = FusedProjection(concat_rows([layers[0].local, layers[1].local]))
        blocks.append([gate_up, layers[2]])
    torch.cuda.synchronize(device)
    return blocks


def layer_of(p):
    """The QuantLinear a block entry runs (itself, or a shard's local layer)."""
    return getattr(p, "local", p)


_CHAINS = {}


def chain_steps(blocks, x, per_block):
    """The step as `qlinear_chain` lists: one chain of every layer (gate|up
    then the gated down projection of each block in turn), or one chain per
    block. Intermediate buffers are allocated once per (blocks, input)."""
    import torch
    from tensorshrink_b200.kernels import ChainStep
    key = (id(blocks), x.data_ptr(), tuple(x.shape), per_block)
    got = _CHAINS.get(key)
    if got is None:
        groups, cur = [[]], x
        for gate_up, down in blocks:
            gu = torch.empty(x.shape[0], layer_of(gate_up).rows, dtype=x.dtype, device=x.device)
            y = torch.empty(x.shape[0], layer_of(down).rows, dtype=x.dtype, device=x.device)
            if per_block and groups[-1]:
                groups.append([])
            groups[-1] += [ChainStep(layer_of(gate_up).qweight(), cur, gu),
                           ChainStep(layer_of(down).qweight(), gu, y, gated=True)]
            cur = y
        got = (groups, cur)
        _CHAINS[key] = got
    return got


def mlp_step(blocks, x, world=1, exchange=None, chain=None):
    """One decode step through the MLP blocks. On one GPU the layers run as
    chained persistent launches (`chain`: "step" = one launch for every
    layer, "block" = one per block, None = one launch per layer). With
    world > 1 the down projection's fp32 partial sums are summed over the
    ranks by the library's one-shot NVLink all-reduce (`exchange`), or NCCL
    without one."""
    import torch
    import torch.distributed as dist
    if world == 1 and chain:
        from tensorshrink_b200.kernels import qlinear_chain
        groups, y = chain_steps(blocks, x, chain == "block")
        for g in groups:
            qlinear_chain(g, persistent=True)
        return y
    for gate_up, down in blocks:
        gu = gate_up(x)
        if world == 1:
            x = down.gated(gu)
        else:
            y = down.gated(gu, torch.float32)   # this rank's partial sum
            if exchange is not None:
                y = exchange.all_reduce(y, out=y)
            else:
                dist.all_reduce(y)
            x = y.to(torch.bfloat16)
    return x


def step_bytes(blocks, M):
    """Algorithmic bytes of this rank's share of one step: packed weights and
    metadata, plus its activations in and outputs out."""
    b = 0
    for layers in blocks:
        for p in layers:
            ql = layer_of(p)
            b += ql.packed_nbytes() + 2 * M * (ql.in_features + ql.out_features)
    return b


def gemv_flops(blocks, M):
    return sum(2 * M * ql.in_features * ql.out_features for layers in blocks for ql in layers)


# ---------------------------------------------------------------------------
# prefill: BASELINE configs[2] layer at M = 2048 on the tensor-core kernel
# ---------------------------------------------------------------------------

def lloyd2_layer(device, rows, cols, seed=777):
    import tensorshrink_b200 as ts
    w = student_t_cuda((rows, cols), seed, device)
    d = ts.quantize_device(w, bits=2, group_size=64, outlier_frac=0.001, companded=True)
    del w
    return ts.QuantLinear.from_device_quant(d)


def prefill_measure(device, reps=20, M=2048, rows=8192, cols=8192, ql=None):
    """TFLOP/s of one [rows, cols] 2-bit Lloyd-Max g64 (+0.1% outliers) layer at
    M tokens (bf16). Each launch is timed alone between CUDA events on the
    launching stream, with L2 flushed (a 256 MB write) before it."""
    import torch
    from tensorshrink_b200 import _C, kernels

    _, tc_peak, peak_kind = peaks()
    if ql is None:
        ql = lloyd2_layer(device, rows, cols)
    qw = ql.qweight()
    x = torch.randn(M, cols, device=device).to(torch.bfloat16)
    out = torch.empty(M, rows, device=device, dtype=torch.bfloat16)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    for _ in range(3):
        kernels.qlinear(x, qw, None, torch.bfloat16, out=out)
    torch.cuda.synchronize(device)
    st = torch.cuda.current_stream(device)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    _C.launch_count(reset=True)
    for s_ev, e_ev in ev:
        flush.zero_()
        s_ev.record(st)
        kernels.qlinear(x, qw, None, torch.bfloat16, out=out)
        e_ev.record(st)
    torch.cuda.synchronize(device)
    launches = _C.launch_count(reset=True)
    ms = statistics.median(s_ev.elapsed_time(e_ev) for s_ev, e_ev in ev)
    assert torch.isfinite(out.float()).all(), "non-finite prefill output"
    tflops = 2.0 * M * rows * cols / (ms * 1e-3) / 1e12
    return {
        "metric": "QuantLinear TFLOP/s (M=2048)",
        "value": round(tflops, 1), "unit": "TFLOP/s",
        "config": {"workload": f"lloyd2_g64_outlier0.001_{rows}x{cols}_prefill", "M": M,
                   "dtype": "bf16 activations, 2-bit codes, fp32 accumulate",
                   "l2": "flushed (256 MB write) before every timed launch",
                   "timing": f"median of {reps} single launches between CUDA events"},
        "ms_per_launch": round(ms, 4),
        "gpu_launches": int(launches),
        "roofline": {"kernel": "ts::qgemm::qgemm_kernel<2,true,1,256>", "bound": "tensor",
                     "achieved": round(tflops, 1), "peak": tc_peak, "unit": "TFLOP/s",
                     "frac": round(tflops / tc_peak, 4), "peak_kind": peak_kind + " bf16 burst",
                     "flops_per_launch": 2 * M * rows * cols,
                     # dram read + write bytes of one ncu capture of this launch
                     "traffic": QGEMM_TRAFFIC_BYTES},
    }


# ---------------------------------------------------------------------------
# quantize: BASELINE configs[4] weights through the GPU quantize/pack
# ---------------------------------------------------------------------------

def quantize_measure(device, reps=3, rows=28672, cols=8192):
    """fp16-input GB/s of the public GPU quantizer (`quantize_device`: top-k
    outliers, 4-bit g128 codes, double-quant metadata, row-sorted outlier
    tables) on the largest Llama-70B projection shape, median of `reps` calls
    timed with CUDA events; plus the projected time for all 68.45 B weights."""
    import torch
    import tensorshrink_b200 as ts
    from tensorshrink_b200 import _C

    w = student_t_cuda((rows, cols), 4242, device)
    for _ in range(1):
        ts.quantize_device(w, bits=4, group_size=128, outlier_frac=0.001, double_quant=True)
    torch.cuda.synchronize(device)
    times = []
    _C.launch_count(reset=True)
    for _ in range(reps):
        s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_ev.record()
        d = ts.quantize_device(w, bits=4, group_size=128, outlier_frac=0.001, double_quant=True)
        e_ev.record()
        torch.cuda.synchronize(device)
        times.append(s_ev.elapsed_time(e_ev))
    launches = _C.launch_count(reset=True) // reps
    ms = statistics.median(times)
    nbytes = rows * cols * 2
    gbs = nbytes / (ms * 1e-3) / 1e9
    del d
    return {
        "metric": "GPU quantize+pack fp16-input GB/s",
        "value": round(gbs, 1), "unit": "GB/s",
        "config": {"workload": f"llama70b_up_{rows}x{cols}_w4g128_dq_outlier0.001", "input_dtype": "fp16",
                   "timing": f"median of {reps} calls of quantize_device between CUDA events"},
        "ms_per_call": round(ms, 3),
        "library_launches_per_call": int(launches),
        "projected_s_for_68.45B_params": round(68.45e9 * 2 / (gbs * 1e9), 2),
    }


def prefill_sweep(device, reps=10):
    """Config 3 across its token counts and shapes: TFLOP/s per (shape, M)."""
    import torch
    _, tc_peak, _ = peaks()
    out = []
    for rows, cols in ((8192, 8192), (28672, 8192), (8192, 28672)):
        ql = lloyd2_layer(device, rows, cols, seed=rows + cols)
        for M in (256, 2048, 8192):
            r = prefill_measure(device, reps=reps, M=M, rows=rows, cols=cols, ql=ql)
            out.append({"shape": [rows, cols], "M": M, "TFLOP/s": r["value"],
                        "ms_per_launch": r["ms_per_launch"], "frac": round(r["value"] / tc_peak, 4)})
        del ql
        torch.cuda.empty_cache()
    return {"workload": "lloyd2_g64_outlier0.001 prefill, bf16, L2 flushed before each launch",
            "peak": tc_peak, "unit": "TFLOP/s", "points": out}


def graph_time_ms(fn, device, reps):
    """ms per call of `fn` replayed from a CUDA graph, CUDA events around
    `reps` replays."""
    import torch
    for _ in range(2):
        fn()
    torch.cuda.synchronize(device)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize(device)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        g.replay()
    e.record()
    torch.cuda.synchronize(device)
    return s.elapsed_time(e) / reps


def decode_sweep(device, blocks, reps=50):
    """Config 2 at M in {1, 8, 32, 64} (the bench MLP blocks, bf16) and
    config 1 (32 distinct [4096, 4096] 4-bit g128 double-quant NF4 layers with
    0.1% outliers, fp16 activations, M in {1, 16}): packed-weight GB/s of the
    layers' algorithmic bytes, each a CUDA graph of one pass over weights
    larger than L2."""
    import torch
    import tensorshrink_b200 as ts
    hbm_peak, _, _ = peaks()
    res = {"unit": "GB/s", "peak": hbm_peak, "config2_mlp_bf16": [], "config1_nf4_dq_fp16": []}
    for M in (1, 8, 32, 64):
        x = torch.randn(M, HIDDEN, device=device).to(torch.bfloat16)
        ms = graph_time_ms(lambda: mlp_step(blocks, x), device, reps)
        b = step_bytes(blocks, M)
        res["config2_mlp_bf16"].append({"M": M, "GB/s": round(b / (ms * 1e-3) / 1e9, 1),
                                        "ms_per_step": round(ms, 4), "frac": round(b / (ms * 1e-3) / 1e9 / hbm_peak, 4),
                                        "tokens_per_s": round(M / (ms * 1e-3), 1)})
    layers = []
    for i in range(32):
        w = student_t_cuda((4096, 4096), 5000 + i, device)
        layers.append(ts.QuantLinear.from_device_quant(
            ts.quantize_device(w, bits=4, group_size=128, outlier_frac=0.001, double_quant=True, nf_quant=True)))
        del w
    for M in (1, 16):
        x = torch.randn(M, 4096, device=device).to(torch.float16)

        def run():
            for ql in layers:
                ql(x)
        ms = graph_time_ms(run, device, reps)
        b = sum(ql.packed_nbytes() + 2 * M * (ql.in_features + ql.out_features) for ql in layers)
        res["config1_nf4_dq_fp16"].append({"M": M, "GB/s": round(b / (ms * 1e-3) / 1e9, 1),
                                           "us_per_layer": round(ms * 1e3 / len(layers), 3),
                                           "frac": round(b / (ms * 1e-3) / 1e9 / hbm_peak, 4)})
    del layers
    torch.cuda.empty_cache()
    return res


def quantize_all_layers_measure(device, n_layers=80):
    """BASELINE config 5 (i): GPU quantize+pack of every projection of 80
    Llama-70B-shaped layers (68.45 B weights, 4-bit g128 double-quant NF4,
    0.1% outliers). Each weight is drawn on the device (untimed), then
    quantize_device runs between CUDA events; the sum over all 560 calls is
    the measured time."""
    import torch
    import tensorshrink_b200 as ts
    from tensorshrink_b200.decoder import llama_70b_config
    cfg = llama_70b_config()
    H, D, F_ = cfg.hidden, cfg.head_dim, cfg.intermediate
    shapes = [(cfg.n_heads * D, H), (cfg.n_kv_heads * D, H), (cfg.n_kv_heads * D, H), (H, cfg.n_heads * D),
              (F_, H), (F_, H), (H, F_)]
    total_ms, elems, calls = 0.0, 0, 0
    for layer in range(n_layers):
        for j, shape in enumerate(shapes):
            w = student_t_cuda(shape, 90000 + 16 * layer + j, device)
            s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_ev.record()
            d = ts.quantize_device(w, bits=4, group_size=128, outlier_frac=0.001, double_quant=True, nf_quant=True)
            e_ev.record()
            e_ev.synchronize()
            total_ms += s_ev.elapsed_time(e_ev)
            elems += w.numel()
            calls += 1
            del w, d
    return {"metric": "GPU quantize+pack of all Llama-70B-shaped weights", "layers": n_layers, "calls": calls,
            "params": elems, "seconds": round(total_ms / 1e3, 3),
            "fp16_input_GB/s": round(2 * elems / (total_ms * 1e-3) / 1e9, 1),
            "config": "4-bit g128 double-quant NF4, 0.1% outliers; weights drawn per call on the device "
                      "(not timed); CUDA events around each quantize_device call, summed"}


def decoder_measure(device, world, timed, batches=(1, 16, 64), ctx=128, steps=32, cfg=None, prefill=True,
                    exchange=None):
    """the Llama-3-8B-shaped decoder (32 layers, per-layer
    bits drawn from 2/4/8 with a fixed seed, g128 uniform + 0.1% outliers),
    tensor-parallel over the `world` ranks. Decode: B sequences with `ctx`
    tokens of context, one CUDA-graph step per token, `steps` steps timed
    with CUDA events (max over ranks). Prefill: one 2048-token sequence.
    Reports tokens/s and the aggregate packed-weight GB/s of all ranks."""
    import torch
    import torch.distributed as dist
    from tensorshrink_b200.decoder import CUDAGraphDecoder, QuantDecoder, llama3_8b_config
    cfg = cfg or llama3_8b_config(seed=0)
    model = QuantDecoder(cfg, device, exchange=exchange, max_batch=max(batches),
                         max_seq=2048 if prefill else ctx + steps + 16)
    packed = float(model.packed_nbytes())
    if world > 1:
        t = torch.tensor([packed], device=device, dtype=torch.float64)
        dist.all_reduce(t)
        packed = float(t.item())
    g = torch.Generator(device=device).manual_seed(0)
    res = {"workload": (f"llama_{cfg.n_layers}L_h{cfg.hidden}_i{cfg.intermediate}_bits_"
                        f"{'_'.join(map(str, sorted(set(model.layer_bits))))}_g{cfg.group_size}"
                        f"{'_dq' if cfg.double_quant else ''}{'_nf' if cfg.nf_quant else '_uniform'}_outlier0.001"),
           "layer_bits": model.layer_bits, "packed_bytes_all_ranks": int(packed),
           "parallelism": (f"tp x{world}, " + ("NCCL" if exchange is None else "one-shot NVLink all-reduce kernel"))
                          if world > 1 else "single GPU",
           "decode_path": ("per layer: q/k/v GEMV with the input RMSNorm staged in the kernel, the decode attention "
                           "kernel (rope + cache append + GQA), then o_proj (+residual), gate|up (post RMSNorm "
                           "staged) and the gated down projection (+residual) as one chained launch (B <= 8; larger "
                           "batches run the same ops unfused)"),
           "decode": []}
    attn_len = ctx + steps + 8
    for B in batches:
        tokens = torch.randint(0, cfg.vocab, (B, ctx), device=device, generator=g)
        first = model.prefill(tokens)
        runner = CUDAGraphDecoder(model, B, attn_len=attn_len)
        model.prefill(tokens)
        runner.start(first, ctx)
        torch.cuda.nvtx.range_push("decode")
        ms = timed(runner.step, steps) / steps
        torch.cuda.nvtx.range_pop()
        entry = {"batch": B, "context": ctx, "ms_per_step": round(ms, 4),
                 "tokens_per_s": round(B / (ms * 1e-3), 1),
                 "packed_GB/s": round(packed / (ms * 1e-3) / 1e9, 1)}
        del runner
        if B == batches[0]:
            # the same step from unfused torch ops + one qlinear launch per projection
            model.fused_decode = False
            model.prefill(tokens)
            runner = CUDAGraphDecoder(model, B, attn_len=attn_len)
            model.prefill(tokens)
            runner.start(first, ctx)
            ms_u = timed(runner.step, steps) / steps
            entry["unfused_ms_per_step"] = round(ms_u, 4)
            del runner
            model.fused_decode = True
        res["decode"].append(entry)
    if prefill:
        tokens = torch.randint(0, cfg.vocab, (1, 2048), device=device, generator=g)
        model.prefill(tokens)
        ms = timed(lambda: model.prefill(tokens), 3) / 3
        res["prefill_2048"] = {"ms": round(ms, 3), "tokens_per_s": round(2048 / (ms * 1e-3), 1)}
    del model
    torch.cuda.empty_cache()
    return res


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def run_ours(args, rank, world, device):
    import torch
    import torch.distributed as dist
    from tensorshrink_b200 import _C

    torch.manual_seed(0)
    hbm_peak, _, peak_kind = peaks()
    blocks = build_blocks(args.blocks, device, world=world, rank=rank)
    M = args.M
    exchange = None
    if world > 1 and not args.nccl:
        from tensorshrink_b200.comm import PeerExchange
        exchange = PeerExchange(max_floats=1 << 20, device=device)
    x0 = torch.randn(M, HIDDEN, device=device).to(torch.bfloat16)
    static_x = x0.clone()

    # ---- capture one step as a CUDA graph ----
    for _ in range(2):
        mlp_step(blocks, static_x, world, exchange)
    torch.cuda.synchronize(device)
    _C.launch_count(reset=True)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        static_y = mlp_step(blocks, static_x, world, exchange)
    launches_per_step = _C.launch_count(reset=True)

    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize(device)

    def timed(fn, k):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(k):
            fn()
        e.record()
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()
        ms = s.elapsed_time(e)
        if world > 1:
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    # clocks: soak for ~1 s first so the sampler sees steady state, then time
    soak_until = time.time() + args.soak
    while time.time() < soak_until:
        for _ in range(50):
            graph.replay()
        torch.cuda.synchronize(device)
    with ClockSampler(device.index) as clk:
        ms = timed(graph.replay, args.steps)
        # keep sampling across a comparable stretch when the region is short
        extra_until = time.time() + 0.5 * args.soak
        while time.time() < extra_until:
            for _ in range(50):
                graph.replay()
            torch.cuda.synchronize(device)
    ms_per_step = ms / args.steps
    bytes_step = step_bytes(blocks, M)
    if world > 1:
        # whole-job bytes: every rank's shard (the shards partition the layers)
        t = torch.tensor([float(bytes_step)], device=device, dtype=torch.float64)
        dist.all_reduce(t)
        bytes_job = float(t.item())
    else:
        bytes_job = float(bytes_step)
    value = bytes_job / (ms_per_step * 1e-3) / 1e9

    # ---- the step's launch structures, each graph-replayed ----
    # unchained: one launch per layer (the per-launch GEMV roofline);
    # per block: gate|up + gated down chained; whole step: one launch
    reps = max(args.steps, 10)
    variants = {}
    for name, mode in (("per_layer", None), ("chain_per_block", "block"), ("chain_step", "step"),
                       ("chain_step_1cta", "step")):
        if world > 1 and mode:
            continue
        if name.endswith("_1cta"):
            os.environ["TS_CHAIN_CTAS_PER_SM"] = "1"
        vx = torch.randn(M, HIDDEN, device=device).to(torch.bfloat16)
        for _ in range(2):
            mlp_step(blocks, vx, world, exchange, chain=mode)
        torch.cuda.synchronize(device)
        _C.launch_count(reset=True)
        vg = torch.cuda.CUDAGraph()
        with torch.cuda.graph(vg):
            mlp_step(blocks, vx, world, exchange, chain=mode)
        nl = _C.launch_count(reset=True)
        for _ in range(3):
            vg.replay()
        vms = timed(vg.replay, reps) / reps
        variants[name] = {"GB/s": round(bytes_job / (vms * 1e-3) / 1e9, 1), "ms_per_step": round(vms, 5),
                          "launches_per_step": int(nl)}
        os.environ.pop("TS_CHAIN_CTAS_PER_SM", None)
        del vg
    n_layers = 2 * len(blocks)
    if world == 1 and STEP_CHAIN:
        # the timed step is ONE persistent launch over every layer
        kms, kbytes = ms_per_step, bytes_step
        k_kernel = "ts::gemv_v2::gemv::qgemv_kernel<4,false,false,4,8> (chain of all layers, one launch)"
    else:
        kms = variants["per_layer"]["ms_per_step"] / n_layers
        kbytes = bytes_step / n_layers
        k_kernel = "ts::gemv_v2::gemv::qgemv_kernel<4,false,false,4,1> (gate|up and down GEMVs, one launch each)"
    k_gbs = kbytes / (kms * 1e-3) / 1e9

    # ---- e2e: public module API, pinned host input/output ----
    xh = x0.cpu().pin_memory()
    yh = torch.empty(M, HIDDEN, dtype=torch.bfloat16).pin_memory()
    xd = torch.empty_like(x0)

    def e2e_step():
        xd.copy_(xh, non_blocking=True)
        y = mlp_step(blocks, xd, world, exchange)
        yh.copy_(y, non_blocking=True)

    for _ in range(3):
        e2e_step()
    # eager: every call issued from Python (host-launch bound at M=1)
    eager_ms = timed(e2e_step, args.steps) / args.steps
    # the same public-API step captured once in a CUDA graph, as a decode
    # server runs it; every replay still copies the input from pinned host
    # memory and the result back to pinned host memory
    e2e_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(e2e_graph):
        e2e_step()
    for _ in range(3):
        e2e_graph.replay()
    e2e_ms = timed(e2e_graph.replay, args.steps) / args.steps
    e2e_val = bytes_job / (e2e_ms * 1e-3) / 1e9
    eager_val = bytes_job / (eager_ms * 1e-3) / 1e9

    # correctness guard on the timed graph output (finite, non-trivial)
    graph.replay()
    torch.cuda.synchronize(device)
    assert torch.isfinite(static_y.float()).all(), "non-finite bench output"

    # single-GPU kernel studies: at N = 1 only
    solo = world == 1
    prefill = prefill_measure(device) if solo and not args.no_prefill else None
    quant = quantize_measure(device) if solo and not args.no_prefill else None
    sweeps = None
    if solo and not args.no_sweeps:
        sweeps = {"decode": decode_sweep(device, blocks), "prefill": prefill_sweep(device)}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(blocks, M, budget_s=args.cpu_seconds)
    del blocks, graph, e2e_graph
    torch.cuda.empty_cache()
    decoder = decoder_measure(device, world, timed, exchange=exchange) if not args.no_decoder else None
    decoder70 = None
    if not args.no_decoder:
        from tensorshrink_b200.decoder import llama_70b_config
        decoder70 = decoder_measure(device, world, timed, batches=(1, 32), cfg=llama_70b_config(), prefill=False,
                                    exchange=exchange)
    quant_all = quantize_all_layers_measure(device) if solo and not args.no_prefill else None

    out = None
    if rank == 0:
        out = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 5),
            "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak",
            "vs_baseline": None,
            "dtype": "u4 codes x bf16 (fp32 accumulate)",
            "data": "synthetic (seeded Student-t(df=4) weights, N(0,1) activations)",
            "config": {
                "workload": "llama_mlp_h4096_i14336_w4g128_uniform_outlier0.001_decode",
                "M": M, "blocks": args.blocks, "matrices_per_step": 3 * args.blocks, "launches_per_step": int(launches_per_step),
                "structure": ("one persistent chained launch over every layer (fused gate|up, gated down per block)"
                              if world == 1 and STEP_CHAIN else
                              "per block: fused gate|up GEMV, gated down GEMV (+ all-reduce)"),
                "bytes_per_step": bytes_step,
                "l2": f"inputs larger than L2: {args.blocks} distinct MLP blocks "
                      f"({bytes_step / 1e6:.0f} MB packed) streamed per step",
                "parallelism": (f"tp x{world} (gate/up column-parallel, down row-parallel + "
                                f"{'NCCL all-reduce' if exchange is None else 'one-shot NVLink all-reduce kernel'}"
                                f" of fp32 partials)") if world > 1 else "single GPU",
                "timing": "CUDA graph of one step, K replays between CUDA events, max over ranks",
            },
            "tokens_per_s": round(M / (ms_per_step * 1e-3), 1),
            "e2e": {"value": round(e2e_val, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": int(xh.numel() * xh.element_size()),
                    "d2h_bytes_per_step": int(yh.numel() * yh.element_size()),
                    "ms_per_step": round(e2e_ms, 5),
                    "path": "QuantLinear modules called through the public API, captured once in a CUDA "
                            "graph together with the pinned host->device input copy and device->host "
                            "result copy; K graph replays between CUDA events",
                    "eager": {"value": round(eager_val, 2), "ms_per_step": round(eager_ms, 5),
                              "path": "the same calls issued from Python every step"}},
            "step_variants": variants,
            "roofline": {"kernel": k_kernel, "bound": "hbm",
                         "achieved": round(k_gbs, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(k_gbs / hbm_peak, 4), "peak_kind": peak_kind,
                         "bytes_per_launch": int(kbytes), "us_per_launch": round(kms * 1e3, 3),
                         # dram__bytes_read.sum + dram__bytes_write.sum of one ncu
                         # capture of this kernel (per launch)
                         "traffic": QGEMV_TRAFFIC_BYTES if not (world == 1 and STEP_CHAIN) else None},
            "gpu_launches": int(launches_per_step * args.steps),
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
            "prefill": prefill,
            "quantize": quant,
            "sweeps": sweeps,
            "decoder": decoder,
            "decoder_70b": decoder70,
            "quantize_all_70b": quant_all,
        }
    return out


def cpu_baseline(blocks, M, budget_s=10.0, impl_steps=None):
    """Time the numpy port of the reference CPU path on a bounded sample of one
    MLP block (row chunks of gate/up/down, all host threads)."""
    from oracle import goap
    threads = os.cpu_count() or 1
    qts = [layer_of(p).to_quantized_tensor() for p in blocks[0]]
    rng = np.random.default_rng(0)
    xs = {HIDDEN: rng.standard_normal((M, HIDDEN)).astype(np.float32),
          INTER: rng.standard_normal((M, INTER)).astype(np.float32)}
    frac = 1.0
    # size the sample: time 1024 rows of each matrix first
    t0 = time.perf_counter()
    for q in qts:
        goap.qlinear_threaded(xs[q.cols], q, threads, rows=1024)
    t1 = time.perf_counter() - t0
    rows_budget = int(1024 * max(1.0, (budget_s / 2) / max(t1, 1e-6)))
    done_bytes, t_total = 0, 0.0
    sample_rows = []
    for q in qts:
        r = min(q.rows, rows_budget)
        sample_rows.append(r)
    t0 = time.perf_counter()
    for q, r in zip(qts, sample_rows):
        goap.qlinear_threaded(xs[q.cols], q, threads, rows=r)
        per_row = (q.packed.nbytes + q.scale.nbytes + q.gmin.nbytes + q.outlier_idx.shape[0] * 6) / q.rows
        done_bytes += per_row * r + 4 * M * (q.cols)
    t_total = time.perf_counter() - t0
    del frac
    return {"value": round(done_bytes / t_total / 1e9, 4), "unit": "GB/s", "cores": threads,
            "kind": "port",
            "sample": f"rows {sample_rows} of gate/up/down of one MLP block at M={M} "
                      f"({t_total:.1f} s, numpy dequant + matmul in 1024-row chunks on {threads} threads)",
            "seconds": round(t_total, 2)}


# ---------------------------------------------------------------------------
# reference arm: the unmodified reference (baseline/_ref), else the oracle port
# ---------------------------------------------------------------------------

REF_DIR = ROOT / "baseline" / "_ref" / "tensorshrink"


def load_reference_modules():
    """The reference's `tensorshrink.modules`, imported from baseline/_ref
    (placed there unchanged by baseline/install_ref.py). The package
    `__init__` needs `zstandard` (absent), so the submodules are imported
    under a bare package object; None when the install is missing."""
    if not (REF_DIR / "modules.py").exists():
        return None
    import importlib
    import types
    pkg = types.ModuleType("tensorshrink")
    pkg.__path__ = [str(REF_DIR)]
    sys.modules["tensorshrink"] = pkg
    return importlib.import_module("tensorshrink.modules")


def student_t_torch(shape, seed, device):
    """The bench's weight distribution (Student-t df=4, std 0.02, fp16),
    drawn with a seeded generator on `device`."""
    if str(device).startswith("cuda"):
        return student_t_cuda(shape, seed, device)
    import torch
    g = torch.Generator().manual_seed(seed)
    z = torch.randn(shape, generator=g)
    chi = torch.zeros(shape)
    for _ in range(4):
        chi += torch.randn(shape, generator=g).square()
    w = z / torch.sqrt(chi / 4.0)
    w *= 0.02 / w.std()
    return w.to(torch.float16)


def reference_block(refmod, device, seed0=0, rows_frac=1.0):
    """One MLP block (gate, up, down) as the reference's QuantLinear, built
    by its own `QuantLinear.from_linear` with the bench's settings (4-bit
    g128 uniform, 0.1% outliers, no double quant). `rows_frac` < 1 keeps
    that leading fraction of each weight's rows (a bounded sample)."""
    import torch
    layers = []
    for j, shape in enumerate(((INTER, HIDDEN), (INTER, HIDDEN), (HIDDEN, INTER))):
        rows = max(128, int(shape[0] * rows_frac) // 128 * 128)
        w = student_t_torch(shape, seed0 + j, device)[:rows]
        lin = torch.nn.Linear(shape[1], rows, bias=False, device=device, dtype=torch.float16)
        with torch.no_grad():
            lin.weight.copy_(w)
        q, _, _ = refmod.QuantLinear.from_linear(lin, bits=4, group_size=128, outlier_frac=0.001,
                                                 double_quant=False, nf_quant=False)
        layers.append(q)
        del w, lin
    return layers


def reference_mlp(block, x):
    """gate/up/down through the reference modules, SiLU-gated like the
    library's fused path."""
    import torch.nn.functional as F
    gate, up, down = block
    return down(F.silu(gate(x)) * up(x))


def reference_step_bytes(blocks, M):
    return sum(q.packed_nbytes() + 2 * M * (q.in_features + q.out_features) for b in blocks for q in b)


def reference_gpu_anchor(refmod, args):
    """The reference's own CUDA path (QuantLinear.forward -> Triton
    `fused_quantized_linear` for M <= 64) on cuda:0: the same blocks, M and
    step as the library's device-timed `value`, timed with CUDA events."""
    import torch
    try:
        import triton
        tver = triton.__version__
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"triton not importable: {e}"}
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    blocks = [reference_block(refmod, dev, seed0=10 * b) for b in range(args.blocks)]
    x0 = torch.randn(args.M, HIDDEN, device=dev, dtype=torch.bfloat16)

    def step():
        x = x0
        for blk in blocks:
            x = reference_mlp(blk, x)
        return x

    with torch.no_grad():
        for _ in range(max(3, args.warmup)):
            step()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / args.steps
    nbytes = reference_step_bytes(blocks, args.M)
    used_triton = all(getattr(q, "_triton_eligible", False) for b in blocks for q in b)
    return {"value": round(nbytes / (ms * 1e-3) / 1e9, 2), "unit": "GB/s", "ms_per_step": round(ms, 4),
            "path": "reference QuantLinear.forward on cuda:0, eager"
                    + (" (Triton fused_quantized_linear)" if used_triton else " (no Triton path)"),
            "triton": tver, "blocks": args.blocks, "bytes_per_step": nbytes}


def run_reference_port(args, world, threads):
    """Fallback when baseline/_ref is not installed: the oracle's numpy
    restatement of the reference's CPU path on a 512-row sample."""
    from oracle import goap
    rng = np.random.default_rng(0)
    qts = []
    rows_per_step = 512
    for j, shape in enumerate(((INTER, HIDDEN), (INTER, HIDDEN), (HIDDEN, INTER))):
        w = goap.student_t_weights((rows_per_step, shape[1]), seed=j)
        qts.append(goap.quantize(w, bits=4, group_size=128, outlier_frac=0.001, mode="uniform"))
    xs = {HIDDEN: rng.standard_normal((args.M, HIDDEN)).astype(np.float32),
          INTER: rng.standard_normal((args.M, INTER)).astype(np.float32)}
    bytes_step = 0
    for q in qts:
        bytes_step += q.packed.nbytes + q.scale.nbytes + q.gmin.nbytes + q.outlier_idx.shape[0] * 10 \
            + 2 * args.M * (q.cols + q.rows)

    def step():
        for q in qts:
            goap.qlinear_threaded(xs[q.cols], q, threads, chunk_rows=128)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    sample = (f"{rows_per_step} rows of each of gate/up/down ([14336,4096] x2, [4096,14336]) at "
              f"M={args.M}: oracle numpy port, 128-row chunks on {threads} threads")
    return bytes_step / dt / 1e9, dt, "port", sample, {"sample_rows_per_matrix": rows_per_step}


def run_reference_unmodified(args, refmod, threads):
    """The reference's QuantLinear.forward on CPU tensors (its chunked
    `_dequantize_rows` + F.linear path, modules.py:924-940) over one full
    config-2 MLP block, bf16 activations, all host threads. If (K + W)
    full steps would pass ~150 s, each weight keeps a leading row sample."""
    import torch
    budget_s = 150.0
    block = reference_block(refmod, "cpu")
    x = torch.randn(args.M, HIDDEN, dtype=torch.bfloat16)
    with torch.no_grad():
        reference_mlp(block, x)
        t0 = time.perf_counter()
        reference_mlp(block, x)
        t_full = time.perf_counter() - t0
    frac = min(1.0, budget_s / max(1, args.steps + args.warmup) / max(t_full, 1e-6))
    if frac < 1.0:
        block = reference_block(refmod, "cpu", rows_frac=frac)
    with torch.no_grad():
        for _ in range(args.warmup):
            reference_mlp(block, x)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            reference_mlp(block, x)
        dt = (time.perf_counter() - t0) / args.steps
    rows = [q.out_features for q in block]
    nbytes = reference_step_bytes([block], args.M)
    sample = ("one MLP block, gate/up/down rows " + str(rows)
              + " of [14336,4096] x2 / [4096,14336]"
              + (" (full size)" if frac >= 1.0 else f" (leading {frac:.3f} of rows)")
              + f", M={args.M} bf16: unmodified reference QuantLinear.forward on CPU tensors, "
              f"{threads} threads")
    return nbytes / dt / 1e9, dt, "reference", sample, {"rows_per_matrix": rows, "same_config": frac >= 1.0}


def run_reference(args, rank, world):
    if rank != 0:
        return None
    import torch
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    refmod = load_reference_modules()
    if refmod is not None:
        value, dt, kind, sample, extra = run_reference_unmodified(args, refmod, threads)
    else:
        value, dt, kind, sample, extra = run_reference_port(args, world, threads)
    out = {
        "metric": METRIC, "value": round(value, 4), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u4 codes x bf16", "data": "synthetic",
        "config": dict({"workload": "llama_mlp_h4096_i14336_w4g128_uniform_outlier0.001_decode", "M": args.M},
                       **extra),
        "impl": "reference",
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads, "kind": kind,
                         "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if refmod is not None and torch.cuda.is_available() and not args.no_ref_gpu:
        try:
            out["gpu_anchor"] = reference_gpu_anchor(refmod, args)
        except Exception as e:  # noqa: BLE001
            out["gpu_anchor"] = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--M", type=int, default=1)
    ap.add_argument("--blocks", type=int, default=4)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-sweeps", action="store_true", help="skip the per-config M sweeps")
    ap.add_argument("--no-decoder", action="store_true", help="skip the Llama-3-8B-shaped decoder")
    ap.add_argument("--nccl", action="store_true", help="tensor-parallel exchanges through NCCL instead of the "
                                                       "library's one-shot all-reduce kernel")
    ap.add_argument("--no-ref-gpu", action="store_true",
                    help="--impl reference: skip the reference's own CUDA/Triton timing")
    ap.add_argument("--only", choices=("decoder", "quantize", "prefill"), default=None,
                    help="run one study alone (short; for launch lists and profiles): the 8B decoder at "
                         "batch 1, the [28672, 8192] quantize, or the config-3 prefill layer")
    ap.add_argument("--quant-shape", default="28672x8192", help="--only quantize: ROWSxCOLS of the weight")
    ap.add_argument("--soak", type=float, default=1.0,
                    help="seconds of untimed replays before the timed region (0 for profiling runs)")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        out = run_reference(args, rank, world)
        if out is not None:
            print(json.dumps(out), flush=True)
        return

    import torch
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=device)
    if args.only == "decoder":
        def timed_only(fn, k):
            torch.cuda.synchronize(device)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(k):
                fn()
            e.record()
            torch.cuda.synchronize(device)
            return s.elapsed_time(e)
        out = decoder_measure(device, world, timed_only, batches=(1,), steps=args.steps, prefill=False)
        if rank == 0:
            print(json.dumps(out), flush=True)
        return
    if args.only == "quantize":
        rows, cols = (int(v) for v in args.quant_shape.split("x"))
        print(json.dumps(quantize_measure(device, reps=max(1, args.steps), rows=rows, cols=cols)), flush=True)
        return
    if args.only == "prefill":
        print(json.dumps(prefill_measure(device, reps=max(1, args.steps))), flush=True)
        return
    out = run_ours(args, rank, world, device)
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
