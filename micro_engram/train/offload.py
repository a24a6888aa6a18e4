"""Activation offloading: tensors autograd saves outside checkpointed layers (with
per-layer checkpointing, each layer's input) go to pinned host memory on a side stream and
come back for the backward.

Pinned buffers are pooled by (numel, dtype) and reused every step (pinning is slow);
each copy is one cudaMemcpyAsync on the offload stream, ordered after the producer with an
event, and the device tensor is kept alive until its copy finished (record_stream).
Same mechanism as the reference (micro_engram/train/offload.py:1-66).
"""
import torch

MIN_BYTES = 1 << 20


class ActivationOffload:
    def __init__(self, device):
        self.device = device
        self.pool = {}
        self.in_use = []
        self.order = []  # packed entries of this micro-batch, in forward order
        self.stream = torch.cuda.Stream(device) if device.type == "cuda" else None

    def _buffer(self, t):
        key = (t.numel(), t.dtype)
        free = self.pool.setdefault(key, [])
        buf = free.pop() if free else torch.empty(t.numel(), dtype=t.dtype, pin_memory=True)
        self.in_use.append((key, buf))
        return buf

    def pack(self, t):
        if t.device.type != "cuda" or t.numel() * t.element_size() < MIN_BYTES or not t.is_contiguous():
            return t
        buf = self._buffer(t)
        self.stream.wait_stream(torch.cuda.current_stream(t.device))
        with torch.cuda.stream(self.stream):
            buf.copy_(t.view(-1), non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self.stream)
        t.record_stream(self.stream)
        entry = {"buf": buf, "shape": t.shape, "device": t.device, "ev": ev, "dev": None, "ready": None}
        self.order.append(entry)
        return entry

    def _fetch(self, e):
        """Start the host->device copy of entry e on the side stream (once)."""
        if e["dev"] is not None:
            return
        self.stream.wait_event(e["ev"])
        with torch.cuda.stream(self.stream):
            e["dev"] = e["buf"].to(e["device"], non_blocking=True)
            e["ready"] = torch.cuda.Event()
            e["ready"].record(self.stream)

    def unpack(self, packed):
        if isinstance(packed, torch.Tensor):
            return packed
        e = packed
        self._fetch(e)
        # the backward visits layers in reverse: start copying the previous layer's input now,
        # so it overlaps this layer's backward
        try:
            i = next(j for j in range(len(self.order) - 1, -1, -1) if self.order[j] is e)
        except StopIteration:
            i = -1
        if i > 0:
            self._fetch(self.order[i - 1])
        cur = torch.cuda.current_stream(e["device"])
        cur.wait_event(e["ready"])
        out = e["dev"]
        out.record_stream(cur)
        e["dev"] = None  # the caller owns it now
        return out.view(e["shape"])

    def context(self):
        return torch.autograd.graph.saved_tensors_hooks(self.pack, self.unpack)

    def end_step(self):
        """After the backward: every pinned buffer of this micro-batch can be reused."""
        if self.device.type == "cuda":
            torch.cuda.current_stream(self.device).synchronize()
        for key, buf in self.in_use:
            self.pool[key].append(buf)
        self.in_use = []
        self.order = []

    def pinned_bytes(self):
        return (sum(b.numel() * b.element_size() for bs in self.pool.values() for b in bs)
                + sum(b.numel() * b.element_size() for _, b in self.in_use))
