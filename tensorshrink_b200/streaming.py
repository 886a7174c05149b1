"""Streaming QuantLinear weights from pinned host memory (models whose packed
weights exceed device memory).

Replaces the reference's `StreamingQuantModel` / `stream_offload_module`
(streaming.py:78-272): forward pre/post hooks on every QuantLinear keep its
buffers in pinned host memory and bring them to the device just before the
layer runs, prefetching the next `prefetch_depth` layers (in module order)
on a side stream so the host-to-device copies overlap the kernels.

Layout, chosen for the device: each layer's streamed buffers (packed codes,
scale/min or the double-quant codes and metadata, codebook, outlier
row/col/delta tables and CSR offsets) are packed once into one contiguous
pinned block, 256-byte aligned per buffer, so a layer arrives with a single
copy. The device side is a fixed ring of `prefetch_depth + 1` slots, each
the size of the largest layer, allocated once: no allocation or
caching-allocator traffic per layer. A slot is refilled only after the
compute stream has passed an event recorded when its previous layer's
forward finished. The layer's buffers are views into its slot while it is
resident. Unlike the reference, double-quantized layers stream too.
"""

from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import torch

from .modules import QuantLinear

_ALIGN = 256
_BUFFERS = ("packed", "scale", "gmin", "dq_scale_codes", "dq_scale_meta", "dq_gmin_codes", "dq_gmin_meta",
            "codebook", "outlier_row", "outlier_col", "outlier_delta", "outlier_row_ptr")


def _streamed(ql: QuantLinear) -> List[Tuple[str, torch.Tensor]]:
    out = []
    for n in _BUFFERS:
        t = getattr(ql, n, None)
        if isinstance(t, torch.Tensor):
            out.append((n, t))
    return out


class StreamingQuantModel:
    """Hooks every QuantLinear of `model` so its buffers stream in from
    pinned host memory on demand (see module doc). `enable()` installs the
    hooks, `disable()` removes them and leaves the buffers on the host."""

    def __init__(self, model: torch.nn.Module, device: str = "cuda", prefetch_depth: int = 1,
                 pin_memory: bool = True, verbose: bool = True):
        if not torch.cuda.is_available():
            raise RuntimeError("StreamingQuantModel requires a CUDA device")
        self.model = model
        self.device = torch.device(device)
        self.prefetch_depth = max(1, int(prefetch_depth))
        self._layers: List[Tuple[str, QuantLinear]] = [
            (n, m) for n, m in model.named_modules() if isinstance(m, QuantLinear)]
        if not self._layers:
            raise ValueError("model has no QuantLinear layers to stream")
        # host blocks: one contiguous (pinned) uint8 block per layer
        self._host: List[torch.Tensor] = []
        self._views: List[Dict[str, Tuple[int, torch.dtype, torch.Size]]] = []
        self._host_views: List[Dict[str, torch.Tensor]] = []
        for _, ql in self._layers:
            parts, off = {}, 0
            bufs = _streamed(ql)
            for n, t in bufs:
                parts[n] = (off, t.dtype, t.shape)
                off = -(-(off + t.numel() * t.element_size()) // _ALIGN) * _ALIGN
            block = torch.empty(max(off, _ALIGN), dtype=torch.uint8, pin_memory=pin_memory)
            hv = {}
            for n, t in bufs:
                o, dt, shp = parts[n]
                nb = t.numel() * t.element_size()
                block[o:o + nb].copy_(t.detach().contiguous().view(-1).view(torch.uint8).cpu())
                hv[n] = block[o:o + nb].view(dt).view(shp)
                setattr(ql, n, hv[n])
            if ql.bias is not None:
                ql.bias = ql.bias.detach().to(self.device)
            ql._qw = None
            self._host.append(block)
            self._views.append(parts)
            self._host_views.append(hv)
        slot_bytes = max(b.numel() for b in self._host)
        n_slots = self.prefetch_depth + 1
        self._slots = [torch.empty(slot_bytes, dtype=torch.uint8, device=self.device) for _ in range(n_slots)]
        self._slot_free = [None] * n_slots         # event: compute done with the slot's last layer
        self._slot_of: Dict[int, int] = {}         # resident layer -> slot
        self._ready: Dict[int, torch.cuda.Event] = {}
        self._next_slot = 0
        self._copy_stream = torch.cuda.Stream(device=self.device)
        self._handles: List = []
        self._enabled = False
        if verbose:
            tot = sum(b.numel() for b in self._host)
            print(f"  streaming: {len(self._layers)} QuantLinear layers in pinned host memory "
                  f"({tot / 1e6:.1f} MB), {n_slots} device slots of {slot_bytes / 1e6:.1f} MB")

    # -- per-layer copy / release ------------------------------------------------------
    def _prefetch(self, idx: int) -> None:
        if idx >= len(self._layers) or idx in self._slot_of:
            return
        s = self._next_slot
        self._next_slot = (s + 1) % len(self._slots)
        for other, slot in list(self._slot_of.items()):   # evict whatever still holds the slot
            if slot == s:
                self._release(other)
        block, dst = self._host[idx], self._slots[s]
        with torch.cuda.stream(self._copy_stream):
            if self._slot_free[s] is not None:
                self._copy_stream.wait_event(self._slot_free[s])
            dst[: block.numel()].copy_(block, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self._copy_stream)
        _, ql = self._layers[idx]
        for n, (o, dt, shp) in self._views[idx].items():
            nb = self._host_views[idx][n].numel() * self._host_views[idx][n].element_size()
            setattr(ql, n, dst[o:o + nb].view(dt).view(shp))
        ql._qw = None
        self._slot_of[idx] = s
        self._ready[idx] = ev

    def _release(self, idx: int) -> None:
        s = self._slot_of.pop(idx, None)
        if s is None:
            return
        _, ql = self._layers[idx]
        for n, t in self._host_views[idx].items():
            setattr(ql, n, t)
        ql._qw = None
        self._ready.pop(idx, None)

    def _pre_hook(self, idx: int):
        def hook(module, inputs):
            self._prefetch(idx)
            torch.cuda.current_stream(self.device).wait_event(self._ready[idx])
            for j in range(idx + 1, min(idx + 1 + self.prefetch_depth, len(self._layers))):
                self._prefetch(j)
            return None
        return hook

    def _post_hook(self, idx: int):
        def hook(module, inputs, output):
            s = self._slot_of.get(idx)
            if s is not None:
                ev = torch.cuda.Event()
                ev.record(torch.cuda.current_stream(self.device))
                self._slot_free[s] = ev
            self._release(idx)
            return None
        return hook

    # -- lifecycle ---------------------------------------------------------------------
    def enable(self) -> "StreamingQuantModel":
        if not self._enabled:
            for idx, (_, ql) in enumerate(self._layers):
                self._handles.append(ql.register_forward_pre_hook(self._pre_hook(idx)))
                self._handles.append(ql.register_forward_hook(self._post_hook(idx)))
            self._enabled = True
        return self

    def disable(self) -> None:
        for h in self._handles:
            h.remove()
        self._handles.clear()
        self._enabled = False
        for idx in list(self._slot_of):
            self._release(idx)

    def stats(self) -> dict:
        return {"n_layers": len(self._layers), "host_bytes": int(sum(b.numel() for b in self._host)),
                "layers_currently_on_gpu": len(self._slot_of),
                "gpu_resident_bytes": int(sum(s.numel() for s in self._slots))}


def stream_offload_module(model: torch.nn.Module, device: str = "cuda", prefetch_depth: int = 1,
                          pin_memory: bool = True, verbose: bool = True) -> StreamingQuantModel:
    """Enable streaming on `model` (streaming.py:240-272) and return the streamer."""
    return StreamingQuantModel(model, device, prefetch_depth, pin_memory, verbose).enable()
