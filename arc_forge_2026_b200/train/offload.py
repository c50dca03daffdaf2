"""Host offload of activation-checkpoint inputs (the reference's ``training/work/qwen38fn_lora/checkpoint_offload.py``:
a 120k-token bin's per-layer checkpoint inputs are ~118 GB, so they live in pinned host memory between the forward
and the backward).

Inside ``with CheckpointOffload(): loss = model(...)``, every tensor autograd saves that is on the GPU and at least
``min_bytes`` large (with layer-wise checkpointing: the layer inputs) is copied to pinned host memory on a side
stream (the forward does not wait for it) and its device memory is released once the copy lands. In the backward
the tensors come back in reverse order; unpacking one also starts the host-to-device copy of the next one on the
side stream, so the transfer of layer i-1's input overlaps layer i's recomputation.
"""
from __future__ import annotations

import torch


class _Offloaded:
    __slots__ = ("host", "event", "device", "index", "stride", "prefetched", "ready")

    def __init__(self, host, event, device, index, stride):
        self.host, self.event, self.device, self.index, self.stride = host, event, device, index, stride
        self.prefetched = None
        self.ready = None


class CheckpointOffload(torch.autograd.graph.saved_tensors_hooks):
    def __init__(self, min_bytes: int = 1 << 20, prefetch: bool = True):
        self.min_bytes = min_bytes
        self.prefetch = prefetch
        self.stream = torch.cuda.Stream() if torch.cuda.is_available() else None
        self.items: list[_Offloaded] = []
        self.bytes_offloaded = 0
        super().__init__(self._pack, self._unpack)

    def _pack(self, t: torch.Tensor):
        if not t.is_cuda or t.numel() * t.element_size() < self.min_bytes or self.stream is None:
            return t
        cur = torch.cuda.current_stream(t.device)
        host = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        self.stream.wait_stream(cur)  # the copy starts after t is produced
        with torch.cuda.stream(self.stream):
            host.copy_(t, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self.stream)
        t.record_stream(self.stream)  # t's memory is not reused before the copy has read it
        item = _Offloaded(host, ev, t.device, len(self.items), t.stride())
        self.items.append(item)
        self.bytes_offloaded += t.numel() * t.element_size()
        return item

    def _fetch(self, item: _Offloaded):
        with torch.cuda.stream(self.stream):
            self.stream.wait_event(item.event)
            # the saved tensor's own layout (a transposed weight stays transposed): the backward then runs the same
            # kernels on the same layout as without offload, so the gradients are bitwise identical
            dev = torch.empty_strided(item.host.size(), item.stride, dtype=item.host.dtype, device=item.device)
            dev.copy_(item.host, non_blocking=True)
            ready = torch.cuda.Event()
            ready.record(self.stream)
        item.prefetched, item.ready = dev, ready

    def _unpack(self, item):
        if not isinstance(item, _Offloaded):
            return item
        if item.prefetched is None:
            self._fetch(item)
        cur = torch.cuda.current_stream(item.device)
        cur.wait_event(item.ready)
        t = item.prefetched
        t.record_stream(cur)
        item.prefetched = None
        if self.prefetch and item.index > 0:  # backward runs the layers in reverse: fetch the previous input now
            prev = self.items[item.index - 1]
            if prev.prefetched is None:
                self._fetch(prev)
        return t  # the pinned copies live as long as this context object (a tensor may be unpacked again)
