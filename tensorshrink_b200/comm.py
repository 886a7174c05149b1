"""`PeerExchange`: the library's one-shot NVLink all-reduce for
tensor-parallel layers (`ts_allreduce_oneshot`, csrc/allreduce.cu).

Each rank allocates one exchange buffer, the ranks swap CUDA IPC handles
through the process group (all_gather_object: host plumbing only), and every
rank maps the others' buffers. `all_reduce(partial, residual=None, out=None)`
then sums fp32 row-parallel partials over the ranks, adding the residual,
in one kernel that pushes its slice to every peer and reduces what arrives.
The launch reads its epoch from device memory, so it can be captured in a
CUDA graph and replayed.
"""

from __future__ import annotations

import ctypes as C
from typing import Optional

import torch
import torch.distributed as dist

from . import _C


class PeerExchange:
    def __init__(self, group=None, max_floats: int = 1 << 20, device=None):
        if not (dist.is_available() and dist.is_initialized()):
            raise RuntimeError("PeerExchange needs an initialized process group")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("PeerExchange supports at most 8 ranks (one NVLink domain)")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.cap = int(max_floats)
        lib = _C.load()
        self._lib = lib
        with torch.cuda.device(self.device):
            own = C.c_void_p()
            _C.check(lib.ts_peer_alloc(self.world, self.cap, C.byref(own)), "ts_peer_alloc")
            self._own = own.value
            handle = (C.c_char * 64)()
            _C.check(lib.ts_ipc_get_handle(self._own, handle), "ts_ipc_get_handle")
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
            ptrs = []
            self._opened = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    ptrs.append(self._own)
                    continue
                p = C.c_void_p()
                hb = (C.c_char * 64).from_buffer_copy(h)
                _C.check(lib.ts_ipc_open(hb, C.byref(p)), "ts_ipc_open")
                ptrs.append(p.value)
                self._opened.append(p.value)
        self._ptrs = (C.c_void_p * self.world)(*ptrs)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        dist.barrier(group=group)

    def all_reduce(self, partial: torch.Tensor, residual: Optional[torch.Tensor] = None,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """sum over ranks of `partial` (fp32, contiguous) + `residual`; `out`
        may be `partial` or `residual` (default: a new tensor)."""
        if partial.dtype != torch.float32 or not partial.is_contiguous():
            raise ValueError("PeerExchange.all_reduce takes contiguous fp32 partial sums")
        if residual is not None and (residual.dtype != torch.float32 or not residual.is_contiguous()
                                     or residual.shape != partial.shape):
            raise ValueError("residual must be a contiguous fp32 tensor shaped like the partial sums")
        if out is None:
            out = torch.empty_like(partial)
        rc = self._lib.ts_allreduce_oneshot(
            self._ptrs, self.rank, self.world, self.cap, partial.data_ptr(),
            residual.data_ptr() if residual is not None else None, out.data_ptr(), partial.numel(),
            self.err.data_ptr(), torch.cuda.current_stream(self.device).cuda_stream)
        _C.check(rc, "ts_allreduce_oneshot")
        return out

    def check(self) -> None:
        """Raise if a bounded wait for a peer ran out since the last check."""
        v = int(self.err.item())
        if v:
            self.err.zero_()
            raise RuntimeError(f"one-shot all-reduce: a wait for a peer rank ran out (code {v})")

    def close(self) -> None:
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for p in self._opened:
            self._lib.ts_ipc_close(p)
        dist.barrier(group=self.group)      # nobody maps this rank's buffer any more
        self._lib.ts_peer_free(self._own)
        self._own = None
