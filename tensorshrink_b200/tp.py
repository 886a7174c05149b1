"""Tensor-parallel sharding of QuantLinear layers (one process per GPU).

Column-parallel: a rank keeps weight rows [r0, r1) (output features); its
output is that slice of y, with no exchange. Row-parallel: a rank keeps
weight columns [c0, c1) (input features, cut at group boundaries); it computes
an fp32 partial y from its slice of x and the partials are summed by one
all-reduce over the process group (NCCL on GPUs, gloo on CPU), after which
the bias is added once. In a Llama block q/k/v and gate/up are
column-parallel and o/down row-parallel, so each block exchanges twice.

Shards are cut from the packed buffers as they are (codes, scale/min or the
double-quant codes and metadata, codebook, outlier tables re-indexed), so
every rank reconstructs exactly the weights of its slice of the unsharded
layer; nothing is re-quantized.

Double-quant metadata is shared by super-groups of `dq_group_size`
consecutive (row, group) entries. A shard keeps the metadata as is when its
entries form whole super-groups in the same order; otherwise
(`shard_rows`/`shard_cols` raise) the layer must be sharded unquantized and
quantized per rank, which would change the values.
"""

from __future__ import annotations

from types import SimpleNamespace
from typing import Optional, Sequence

import numpy as np
import torch
import torch.distributed as dist
from torch import nn

from .modules import QuantLinear


def shard_bounds(n: int, world: int, rank: int, align: int = 1):
    """[lo, hi) of rank's share of n items, cut at multiples of `align`."""
    if n % align:
        raise ValueError(f"{n} is not a multiple of {align}")
    units = n // align
    if units < world:
        raise ValueError(f"cannot split {units} units of {align} over {world} ranks")
    base, extra = divmod(units, world)
    lo = rank * base + min(rank, extra)
    hi = lo + base + (1 if rank < extra else 0)
    return lo * align, hi * align


def _row_ptr(rows: torch.Tensor, n_rows: int) -> torch.Tensor:
    r = rows.cpu().numpy().astype(np.int64)
    ptr = np.searchsorted(r, np.arange(n_rows + 1)).astype(np.int32)
    return torch.from_numpy(ptr).to(rows.device)


def _outlier_subset(ql: QuantLinear, keep: torch.Tensor, row_shift: int, col_shift: int):
    row = ql.outlier_row[keep] - row_shift
    col = ql.outlier_col[keep] - col_shift
    delta = ql.outlier_delta[keep]
    return row.to(torch.int32).contiguous(), col.to(torch.int32).contiguous(), delta.contiguous()


def _make(ql: QuantLinear, *, rows: int, cols: int, padded_cols: int, packed, scale, gmin, dq,
          dq_group_size: int, orow, ocol, odelta, bias) -> QuantLinear:
    src = SimpleNamespace(
        orig_shape=(rows, cols), orig_dtype=ql.orig_dtype_str, bits=ql.bits, group_size=ql.group_size,
        rows=rows, cols=cols, padded_cols=padded_cols, n_groups=padded_cols // ql.group_size,
        packed=packed.contiguous(), scale=None if scale is None else scale.contiguous(),
        gmin=None if gmin is None else gmin.contiguous(),
        dq_scale_codes=dq[0] if dq else None, dq_scale_meta=dq[1] if dq else None,
        dq_gmin_codes=dq[2] if dq else None, dq_gmin_meta=dq[3] if dq else None,
        dq_group_size=dq_group_size,
        codebook_store=ql.codebook if ql.companded else None,
        outlier_row=orow, outlier_col=ocol, outlier_delta=odelta,
        outlier_row_ptr=_row_ptr(orow, rows))
    return QuantLinear(None, bias, _device_quant=src)


def shard_rows(ql: QuantLinear, r0: int, r1: int) -> QuantLinear:
    """Column-parallel piece: weight rows [r0, r1) with their bias slice."""
    if not 0 <= r0 < r1 <= ql.rows:
        raise ValueError(f"bad row range [{r0}, {r1}) of {ql.rows}")
    ng = ql.n_groups
    dq = None
    if ql.double_quant:
        gsz = ql.dq_group_size
        f0, f1 = r0 * ng, r1 * ng
        if f0 % gsz or (f1 % gsz and r1 != ql.rows):
            raise ValueError(f"rows [{r0}, {r1}) split double-quant super-groups of {gsz} entries "
                             f"({ng} groups per row)")
        s0, s1 = f0 // gsz, -(-f1 // gsz)
        # codes stay padded to whole super-groups (the last shard keeps the
        # original padding)
        e1 = min(s1 * gsz, ql.dq_scale_codes.numel())
        dq = (ql.dq_scale_codes[f0:e1].contiguous(), ql.dq_scale_meta[s0:s1].contiguous(),
              ql.dq_gmin_codes[f0:e1].contiguous(), ql.dq_gmin_meta[s0:s1].contiguous())
    keep = (ql.outlier_row >= r0) & (ql.outlier_row < r1)
    orow, ocol, odelta = _outlier_subset(ql, keep, r0, 0)
    return _make(ql, rows=r1 - r0, cols=ql.cols, padded_cols=ql.padded_cols, packed=ql.packed[r0:r1],
                 scale=None if dq else ql.scale[r0:r1], gmin=None if dq else ql.gmin[r0:r1], dq=dq,
                 dq_group_size=ql.dq_group_size, orow=orow, ocol=ocol, odelta=odelta,
                 bias=None if ql.bias is None else ql.bias[r0:r1])


def shard_cols(ql: QuantLinear, c0: int, c1: int) -> QuantLinear:
    """Row-parallel piece: weight columns [c0, c1) (group-aligned), no bias
    (the bias is added once, after the all-reduce)."""
    gs = ql.group_size
    if c0 % gs or not 0 <= c0 < c1 <= ql.cols or (c1 % gs and c1 != ql.cols):
        raise ValueError(f"column range [{c0}, {c1}) is not cut at groups of {gs}")
    g0 = c0 // gs
    g1 = -(-c1 // gs)
    ngs = g1 - g0
    per_byte = 8 // ql.bits
    b0, b1 = c0 // per_byte, g1 * gs // per_byte
    dq = None
    dq_gs = 0
    if ql.double_quant:
        # a shard row keeps groups [g0, g1) of every row; the metadata carries
        # over when each super-group is a whole number of full rows
        gsz, ng = ql.dq_group_size, ql.n_groups
        if gsz % ng:
            # super-groups span row boundaries, so a column cut splits them: the
            # shard keeps the fp16 scale/min the reference stores for a
            # double-quantized tensor (codec.py:644-652, the rounded
            # reconstruction) instead of the codes and metadata
            s32, m32 = ql._scale_gmin_f32()
            keep = (ql.outlier_col >= c0) & (ql.outlier_col < c1)
            orow, ocol, odelta = _outlier_subset(ql, keep, 0, c0)
            return _make(ql, rows=ql.rows, cols=c1 - c0, padded_cols=ngs * gs, packed=ql.packed[:, b0:b1],
                         scale=s32[:, g0:g1].to(torch.float16), gmin=m32[:, g0:g1].to(torch.float16), dq=None,
                         dq_group_size=0, orow=orow, ocol=ocol, odelta=odelta, bias=None)
        rows_per_sup = gsz // ng
        dq_gs = rows_per_sup * ngs
        n_sup = ql.dq_scale_meta.shape[0]

        def take(c):
            # this shard's groups of every row, padded to whole super-groups
            t = c[: ql.rows * ng].reshape(ql.rows, ng)[:, g0:g1].reshape(-1)
            pad = n_sup * dq_gs - t.numel()
            return torch.cat([t, t.new_zeros(pad)]) if pad > 0 else t.contiguous()
        dq = (take(ql.dq_scale_codes), ql.dq_scale_meta.contiguous(),
              take(ql.dq_gmin_codes), ql.dq_gmin_meta.contiguous())
    keep = (ql.outlier_col >= c0) & (ql.outlier_col < c1)
    orow, ocol, odelta = _outlier_subset(ql, keep, 0, c0)
    return _make(ql, rows=ql.rows, cols=c1 - c0, padded_cols=ngs * gs, packed=ql.packed[:, b0:b1],
                 scale=None if dq else ql.scale[:, g0:g1], gmin=None if dq else ql.gmin[:, g0:g1], dq=dq,
                 dq_group_size=dq_gs, orow=orow, ocol=ocol, odelta=odelta, bias=None)


def _group_info(group):
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(group), dist.get_rank(group)
    return 1, 0


class ColumnParallelQuantLinear(nn.Module):
    """This rank's output features [r0, r1) of a QuantLinear. With
    gather_output the full output is assembled by an all-gather."""

    def __init__(self, ql: QuantLinear, group=None, gather_output: bool = False, align: int = 1):
        super().__init__()
        self.group = group
        self.world, self.rank = _group_info(group)
        self.out_features, self.in_features = ql.out_features, ql.in_features
        self.align = align
        self.r0, self.r1 = shard_bounds(ql.rows, self.world, self.rank, align)
        self.local = shard_rows(ql, self.r0, self.r1)
        self.gather_output = gather_output

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = self.local(x)
        if not self.gather_output or self.world == 1:
            return y
        # shards may differ by a few rows: gather equal-size padded pieces
        bounds = [shard_bounds(self.out_features, self.world, r, self.align) for r in range(self.world)]
        width = max(hi - lo for lo, hi in bounds)
        pad = width - y.shape[-1]
        yp = torch.nn.functional.pad(y, (0, pad)) if pad else y
        parts = [torch.empty_like(yp) for _ in range(self.world)]
        dist.all_gather(parts, yp.contiguous(), group=self.group)
        return torch.cat([pt[..., : hi - lo] for pt, (lo, hi) in zip(parts, bounds)], dim=-1)


class RowParallelQuantLinear(nn.Module):
    """This rank's input features [c0, c1) of a QuantLinear; partial outputs
    (fp32) are summed by one all-reduce and the bias is added once.

    input_is_parallel: x already holds only this rank's features (the output
    of a column-parallel layer); otherwise the full x is sliced here."""

    def __init__(self, ql: QuantLinear, group=None, input_is_parallel: bool = True):
        super().__init__()
        self.group = group
        self.world, self.rank = _group_info(group)
        self.out_features, self.in_features = ql.out_features, ql.in_features
        # cut the padded width at group boundaries; the last shard ends at cols
        c0, c1 = shard_bounds(ql.padded_cols, self.world, self.rank, ql.group_size)
        self.c0, self.c1 = c0, min(c1, ql.cols)
        self.local = shard_cols(ql, self.c0, self.c1)
        self.input_is_parallel = input_is_parallel
        if ql.bias is not None:
            self.register_buffer("bias", ql.bias.detach().clone())
        else:
            self.bias = None

    def partial(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's fp32 contribution x[..., c0:c1] . W[:, c0:c1]^T."""
        from . import kernels
        if not self.input_is_parallel:
            x = x[..., self.c0:self.c1]
        x2d = x.reshape(-1, x.shape[-1]).contiguous()
        y = kernels.qlinear(x2d, self.local.qweight(), None, torch.float32)
        return y.reshape(*x.shape[:-1], self.out_features)

    def reduce(self, y: torch.Tensor, out_dtype: torch.dtype) -> torch.Tensor:
        """Sum the partials over the group, add the bias, cast."""
        if self.world > 1:
            dist.all_reduce(y, op=dist.ReduceOp.SUM, group=self.group)
        if self.bias is not None:
            y = y + self.bias.to(y.dtype)
        return y.to(out_dtype)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.reduce(self.partial(x), x.dtype)


# Llama-style projection names: column-parallel inputs, row-parallel outputs
COLUMN_NAMES: Sequence[str] = ("q_proj", "k_proj", "v_proj", "gate_proj", "up_proj")
ROW_NAMES: Sequence[str] = ("o_proj", "down_proj")


def tensor_parallelize(model: nn.Module, group=None, column_names: Sequence[str] = COLUMN_NAMES,
                       row_names: Sequence[str] = ROW_NAMES, head_dim: Optional[int] = None) -> nn.Module:
    """Replace QuantLinear children named like Llama projections by their
    tensor-parallel shards, in place. head_dim aligns q/k/v row cuts to whole
    attention heads."""
    from .modules import _set_module_by_name
    for name, mod in list(model.named_modules()):
        if not isinstance(mod, QuantLinear):
            continue
        leaf = name.rsplit(".", 1)[-1]
        if leaf in column_names:
            align = head_dim if (head_dim and leaf in ("q_proj", "k_proj", "v_proj")) else 1
            _set_module_by_name(model, name, ColumnParallelQuantLinear(mod, group, align=align))
        elif leaf in row_names:
            _set_module_by_name(model, name, RowParallelQuantLinear(mod, group))
    return model


def concat_rows(parts: Sequence[QuantLinear]) -> QuantLinear:
    """One QuantLinear whose output rows are those of `parts` in order (the
    inverse of shard_rows): e.g. q/k/v or gate/up projections fused into one
    launch. The parts must share bits, group size, columns and codebook;
    nothing is re-quantized, so every row reconstructs exactly as before.
    Double-quant parts must each hold whole super-groups."""
    p0 = parts[0]
    for p in parts[1:]:
        if (p.bits, p.group_size, p.cols, p.padded_cols, p.double_quant, p.dq_group_size, p.companded) != \
                (p0.bits, p0.group_size, p0.cols, p0.padded_cols, p0.double_quant, p0.dq_group_size, p0.companded):
            raise ValueError("concat_rows needs parts with the same layout")
        if p.companded and not torch.equal(p.codebook, p0.codebook):
            raise ValueError("concat_rows needs parts with the same codebook")
    rows = sum(p.rows for p in parts)
    offs = np.cumsum([0] + [p.rows for p in parts])
    dq = None
    if p0.double_quant:
        gsz, ng = p0.dq_group_size, p0.n_groups
        if any((p.rows * ng) % gsz for p in parts[:-1]):
            raise ValueError("double-quant super-groups straddle the parts; concat_rows cannot keep them")
        dq = tuple(torch.cat([getattr(p, n)[: (p.rows * ng + gsz - 1) // gsz * gsz if "codes" in n else None]
                              for p in parts]).contiguous()
                   for n in ("dq_scale_codes", "dq_scale_meta", "dq_gmin_codes", "dq_gmin_meta"))
    orow = torch.cat([p.outlier_row + int(o) for p, o in zip(parts, offs[:-1])]).to(torch.int32)
    ocol = torch.cat([p.outlier_col for p in parts]).to(torch.int32)
    odelta = torch.cat([p.outlier_delta for p in parts])
    bias = None
    if any(p.bias is not None for p in parts):
        bdt = next(p.bias.dtype for p in parts if p.bias is not None)
        bias = torch.cat([p.bias if p.bias is not None else torch.zeros(p.rows, dtype=bdt, device=p0.packed.device)
                          for p in parts])
    return _make(p0, rows=rows, cols=p0.cols, padded_cols=p0.padded_cols,
                 packed=torch.cat([p.packed for p in parts]),
                 scale=None if dq else torch.cat([p.scale for p in parts]),
                 gmin=None if dq else torch.cat([p.gmin for p in parts]), dq=dq,
                 dq_group_size=p0.dq_group_size, orow=orow.contiguous(), ocol=ocol.contiguous(),
                 odelta=odelta.contiguous(), bias=bias)
