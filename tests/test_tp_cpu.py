"""Tensor-parallel sharding on CPU.

* Each shard's reconstructed weights equal the matching slice of the
  unsharded layer's, bit for bit (column-parallel row slices, row-parallel
  group-aligned column slices), on QuantLinear buffers built from the
  reference-generated fixtures.
* The row-parallel all-reduce and column-parallel all-gather run on two gloo
  ranks (the GPU kernels are replaced by the numpy reconstruction here; the
  kernels on sharded buffers are covered by tests/test_gpu_tp.py).
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import goap
from tests.conftest import golden_case_list, load_case
from tests.test_host_cpu import qt_from_case


def dense(ql) -> np.ndarray:
    """fp32 W of a QuantLinear from its buffers: level * scale + min, then
    base + delta at outlier positions (modules.py:912-919 order)."""
    codes = goap.unpack_codes(ql.packed.numpy(), ql.bits, ql.padded_cols)[:, : ql.cols]
    cv = ql.codebook.numpy()[codes] if ql.companded else codes.astype(np.float32)
    s, m = (t.numpy() for t in ql._scale_gmin_f32())
    g = np.arange(ql.cols) // ql.group_size
    W = (cv * s[:, g]).astype(np.float32) + m[:, g]
    r = ql.outlier_row.numpy().astype(np.int64)
    c = ql.outlier_col.numpy().astype(np.int64)
    W[r, c] = W[r, c] + ql.outlier_delta.numpy().astype(np.float32)
    return W


def full_layer(golden, name):
    from tensorshrink_b200.modules import QuantLinear
    c = load_case(golden, name)
    bias = torch.from_numpy(c["bias"]) if "bias" in c else None
    return QuantLinear(qt_from_case(c), bias)


@pytest.mark.parametrize("name", golden_case_list())
@pytest.mark.parametrize("world", [2, 4])
def test_column_shards_reconstruct_row_slices(golden, name, world):
    from tensorshrink_b200 import tp
    ql = full_layer(golden, name)
    W = dense(ql)
    for rank in range(world):
        r0, r1 = tp.shard_bounds(ql.rows, world, rank)
        try:
            sh = tp.shard_rows(ql, r0, r1)
        except ValueError as e:
            assert ql.double_quant and "super-groups" in str(e)
            return
        np.testing.assert_array_equal(dense(sh), W[r0:r1])
        if ql.bias is not None:
            assert torch.equal(sh.bias, ql.bias[r0:r1])


@pytest.mark.parametrize("name", golden_case_list())
@pytest.mark.parametrize("world", [2, 4])
def test_row_shards_reconstruct_column_slices(golden, name, world):
    from tensorshrink_b200 import tp
    ql = full_layer(golden, name)
    W = dense(ql)
    if ql.padded_cols // ql.group_size < world:
        pytest.skip("fewer groups than ranks")
    cols = ql.padded_cols if ql.padded_cols == ql.cols else None
    for rank in range(world):
        try:
            c0, c1 = tp.shard_bounds(ql.padded_cols, world, rank, ql.group_size)
        except ValueError:
            pytest.skip("groups do not split evenly")
        c1 = min(c1, ql.cols)
        sh = tp.shard_cols(ql, c0, c1)
        if ql.double_quant and not sh.double_quant:
            # super-groups straddle the cut: the shard keeps the fp16-rounded
            # scale/min (what the reference stores for a double-quantized tensor)
            np.testing.assert_allclose(dense(sh), W[:, c0:c1], rtol=0, atol=2e-3 * np.abs(W).max())
        else:
            np.testing.assert_array_equal(dense(sh), W[:, c0:c1])
        assert sh.bias is None
    del cols


def test_large_dq_layer_shards_both_ways(golden):
    """Double-quant metadata carries over when super-groups are whole rows."""
    from tensorshrink_b200 import tp
    ql = full_layer(golden, "nf4_dq_big")
    W = dense(ql)
    for world in (2, 4, 8):
        for rank in range(world):
            r0, r1 = tp.shard_bounds(ql.rows, world, rank)
            np.testing.assert_array_equal(dense(tp.shard_rows(ql, r0, r1)), W[r0:r1])
            c0, c1 = tp.shard_bounds(ql.cols, world, rank, ql.group_size)
            np.testing.assert_array_equal(dense(tp.shard_cols(ql, c0, c1)), W[:, c0:c1])


def test_shard_bounds():
    from tensorshrink_b200.tp import shard_bounds
    assert [shard_bounds(14336, 8, r, 128) for r in (0, 7)] == [(0, 1792), (12544, 14336)]
    assert shard_bounds(10, 3, 0) == (0, 4) and shard_bounds(10, 3, 2) == (7, 10)
    with pytest.raises(ValueError):
        shard_bounds(100, 2, 0, 128)


# ---------------------------------------------------------------------------
# two gloo ranks
# ---------------------------------------------------------------------------

class _DenseLocal(torch.nn.Module):
    def __init__(self, W, b):
        super().__init__()
        self.W, self.b = W, b

    def forward(self, t):
        return t @ self.W.T + self.b


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, name, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from tensorshrink_b200 import tp
        g = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))
        ql = full_layer(g, name)
        W = dense(ql)
        bias = ql.bias.float() if ql.bias is not None else torch.zeros(ql.rows)
        x = torch.from_numpy(np.random.default_rng(0).standard_normal((3, ql.cols)).astype(np.float32))
        ref = x @ torch.from_numpy(W).T + bias
        # row-parallel: fp32 partial from this rank's column slice, all-reduce, bias once
        row = tp.RowParallelQuantLinear(ql, input_is_parallel=False)
        part = x[:, row.c0:row.c1] @ torch.from_numpy(dense(row.local)).T
        y = row.reduce(part.clone(), torch.float32)
        err_row = float((y - ref).abs().max() / ref.abs().max())
        # column-parallel with gather: local outputs concatenated in rank order
        col = tp.ColumnParallelQuantLinear(ql, gather_output=True)
        Wl = torch.from_numpy(dense(col.local))
        bl = col.local.bias.float() if col.local.bias is not None else 0.0
        col.local = _DenseLocal(Wl, bl)  # the kernel's job on a GPU
        y2 = col(x)
        err_col = float((y2 - ref).abs().max() / ref.abs().max())
        q.put((rank, err_row, err_col, None))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, None, None, repr(e)))


@pytest.mark.parametrize("name", ["u4_g128_pad", "nf4_dq_big", "lloyd2_g64"])
def test_gloo_two_ranks(name):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, name, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, e_row, e_col, err in res:
        assert err is None, (rank, err)
        assert e_row < 1e-5 and e_col < 1e-5, (rank, e_row, e_col)
