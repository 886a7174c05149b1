"""Tensor-parallel shards on the GPU kernels.

On one GPU: the shards of a layer for 2, 4 and 8 ranks are run through the
CUDA kernels and combined as the collectives would (sum of fp32 partials for
row-parallel, concatenation for column-parallel); the result must match the
unsharded fp32 dequant-matmul within the GEMM tolerance, in the decode (GEMV)
and prefill (tensor-core) regimes. With two or more GPUs visible, the same
layers also run as two NCCL ranks.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from oracle import goap

pytestmark = pytest.mark.gpu

TOL = 1e-2


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import tensorshrink_b200._C as C
    C.load()
    yield


def _layer(rows, cols, bits, gs, mode, dq, seed, bias=True):
    import tensorshrink_b200 as ts
    w = torch.from_numpy(goap.student_t_weights((rows, cols), seed=seed)).cuda()
    d = ts.quantize_device(w, bits=bits, group_size=gs, outlier_frac=0.001, double_quant=dq,
                           nf_quant=mode == "nf", companded=mode == "lloyd")
    b = (torch.randn(rows, device="cuda") * 0.1).to(torch.bfloat16) if bias else None
    return ts.QuantLinear.from_device_quant(d, b)


def _rel(y, ref):
    return ((y.float() - ref).abs().max() / ref.abs().max()).item()


LAYERS = [
    (4096, 14336, 4, 128, "uniform", False),   # Llama down projection (row-parallel)
    (14336, 4096, 4, 128, "uniform", False),   # gate/up (column-parallel)
    (4096, 4096, 4, 128, "nf", True),          # config 1 layer, double-quant NF4
    (8192, 8192, 2, 64, "lloyd", False),       # config 3 layer
]


@pytest.mark.parametrize("shape", LAYERS)
@pytest.mark.parametrize("world", [2, 4, 8])
def test_shards_on_one_gpu(shape, world):
    from tensorshrink_b200 import kernels, tp
    rows, cols, bits, gs, mode, dq = shape
    ql = _layer(rows, cols, bits, gs, mode, dq, seed=rows + cols + world)
    W = ql.dequantize(torch.float32)
    for M in (1, 256):
        x = torch.randn(M, cols, device="cuda").to(torch.bfloat16)
        ref = x.float() @ W.T + ql.bias.float()
        # row-parallel: fp32 partials summed, bias once
        acc = torch.zeros(M, rows, device="cuda")
        for r in range(world):
            c0, c1 = tp.shard_bounds(ql.padded_cols, world, r, gs)
            sh = tp.shard_cols(ql, c0, min(c1, cols))
            acc += kernels.qlinear(x[:, c0:min(c1, cols)].contiguous(), sh.qweight(), None, torch.float32)
        err = _rel(acc + ql.bias.float(), ref)
        assert err <= TOL, ("row", M, err)
        # column-parallel: local outputs concatenated
        outs = []
        for r in range(world):
            r0, r1 = tp.shard_bounds(rows, world, r)
            outs.append(tp.shard_rows(ql, r0, r1)(x))
        err = _rel(torch.cat(outs, dim=-1), ref)
        assert err <= TOL, ("column", M, err)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        import torch.distributed as dist
        dist.init_process_group("nccl", rank=rank, world_size=world)
        from tensorshrink_b200 import tp
        torch.manual_seed(0)
        ql = _layer(4096, 14336, 4, 128, "uniform", False, seed=5)
        W = ql.dequantize(torch.float32)
        errs = []
        for M in (1, 256):
            x = torch.randn(M, 14336, device="cuda", generator=torch.Generator("cuda").manual_seed(M))
            x = x.to(torch.bfloat16)
            ref = x.float() @ W.T + ql.bias.float()
            row = tp.RowParallelQuantLinear(ql, input_is_parallel=False)
            errs.append(_rel(row(x), ref))
            col = tp.ColumnParallelQuantLinear(ql, gather_output=True)
            errs.append(_rel(col(x), ref))
        q.put((rank, errs, None))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, None, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_nccl_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, errs, err in res:
        assert err is None, (rank, err)
        assert max(errs) <= TOL, (rank, errs)


def _decoder_worker(rank, world, port, q, use_exchange=False):
    """Each rank builds the tensor-parallel decoder (whole layers quantized
    identically everywhere, then cut) and an unsharded copy in a one-rank
    group; the last-position logits after a prefill, and the tokens of a few
    decode steps, must agree."""
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        import torch.distributed as dist
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
        from tensorshrink_b200.decoder import DecoderConfig, QuantDecoder
        solo = [dist.new_group([r]) for r in range(world)][rank]
        cfg = DecoderConfig(n_layers=2, hidden=1024, n_heads=8, n_kv_heads=4, intermediate=2048, vocab=4000,
                            layer_bits=[4, 8], seed=11)
        ex = None
        if use_exchange:
            from tensorshrink_b200.comm import PeerExchange
            ex = PeerExchange(max_floats=1 << 16)
        tp_model = QuantDecoder(cfg, "cuda", exchange=ex, max_batch=2, max_seq=64)
        ref_model = QuantDecoder(cfg, "cuda", group=solo, max_batch=2, max_seq=64)
        g = torch.Generator(device="cuda").manual_seed(4)
        tokens = torch.randint(0, cfg.vocab, (2, 10), device="cuda", generator=g)
        a = tp_model.prefill(tokens, return_logits=True)
        b = ref_model.prefill(tokens, return_logits=True)
        err = ((a - b).abs().max() / b.abs().max()).item()
        cur_a = a.argmax(-1)
        cur_b = b.argmax(-1)
        agree, total = int((cur_a == cur_b).sum()), 2
        for step in range(4):
            pos = torch.tensor([10 + step], device="cuda")
            cur_a = tp_model.decode_step(cur_b, pos)
            nb = ref_model.decode_step(cur_b, pos)
            agree += int((cur_a == nb).sum())
            total += 2
            cur_b = nb
        q.put((rank, [err, 1.0 - agree / total], None))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, None, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("use_exchange", [False, True])
@pytest.mark.parametrize("world", [2, 4])
def test_tensor_parallel_decoder(world, use_exchange):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_decoder_worker, args=(r, world, port, q, use_exchange)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, vals, err in res:
        assert err is None, (rank, err)
        logit_err, disagree = vals
        assert logit_err <= 2e-2, (rank, logit_err)
        assert disagree <= 0.25, (rank, disagree)


def _exchange_worker(rank, world, port, q):
    """The one-shot NVLink all-reduce: exact against the rank-ordered sum of
    all_gather'ed partials, close to NCCL's all_reduce, correct when replayed
    from a CUDA graph, and a peer that never arrives ends a bounded wait with
    the error flag set instead of a hang."""
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        import torch.distributed as dist
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
        from tensorshrink_b200.comm import PeerExchange
        import tensorshrink_b200._C as _C
        ex = PeerExchange(max_floats=1 << 16)
        errs = []
        for n in (1, 4096, 5000, 65536):
            g = torch.Generator(device="cuda").manual_seed(100 * n + rank)
            x = torch.randn(n, device="cuda", generator=g)
            res = torch.randn(n, device="cuda", generator=torch.Generator(device="cuda").manual_seed(n))
            y = ex.all_reduce(x, residual=res)
            parts = [torch.empty_like(x) for _ in range(world)]
            dist.all_gather(parts, x)
            ref = parts[0].clone()
            for p in parts[1:]:
                ref += p
            ref = res + ref
            errs.append(float((y - ref).abs().max()))
            nc = x.clone()
            dist.all_reduce(nc)
            errs.append(float((y - res - nc).abs().max()) * 1e-3)   # different summation order
        # graph replay: epochs advance on the device
        sx = torch.zeros(4096, device="cuda")
        sy = torch.empty_like(sx)
        ex.all_reduce(sx, out=sy)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            ex.all_reduce(sx, out=sy)
        for it in range(3):
            sx.fill_(float(rank + 1 + it))
            graph.replay()
            torch.cuda.synchronize()
            want = sum(float(r + 1 + it) for r in range(world))
            errs.append(float((sy - want).abs().max()))
        ex.check()
        # a peer that never arrives: rank 0 calls alone with a 1 ms limit
        dist.barrier()
        timed_out = True
        if rank == 0:
            assert _C.load().ts_test_inject_stall(1_000_000) == 0
            ex.all_reduce(torch.ones(64, device="cuda"))
            torch.cuda.synchronize()
            try:
                ex.check()
                timed_out = False
            except RuntimeError:
                timed_out = True
        q.put((rank, errs + [0.0 if timed_out else 1.0], None))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, None, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_exchange_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, errs, err in res:
        assert err is None, (rank, err)
        assert max(errs) == 0.0 or max(errs) < 1e-6, (rank, errs)
