"""Activation offloading: tensors autograd saves outside checkpointed layers (with
per-layer checkpointing, each layer's input) go to pinned host memory on a side stream and
come back for the backward.

Design:
  * a pool of pinned host buffers keyed by (numel, dtype), reused every step (pinning is
    slow); a buffer returns to the pool when the micro-batch's backward is over;
  * every saved tensor becomes a _Saved record: its host buffer, the event that marks the
    end of its device->host copy, and (once fetched) its device copy and that copy's event;
  * device->host copies are ordered after the producer by a stream wait and keep the source
    alive with record_stream; host->device copies run on the same side stream;
  * the backward visits layers in reverse forward order, so fetching record i also starts
    the fetch of record i-1: its copy overlaps the backward of the current layer.

Behaviour of the reference: micro_engram/train/offload.py:1-66 (saved-tensor hooks, pinned
copies on a side stream).
"""
import torch

MIN_BYTES = 1 << 20  # smaller tensors stay on the device


class _Saved:
    __slots__ = ("host", "shape", "device", "copied", "index", "on_device", "arrived")

    def __init__(self, host, shape, device, copied, index):
        self.host, self.shape, self.device, self.copied, self.index = host, shape, device, copied, index
        self.on_device = None  # device tensor once fetched (until handed to autograd)
        self.arrived = None    # event: its host->device copy finished


class _PinnedPool:
    def __init__(self):
        self.free = {}
        self.lent = []

    def take(self, numel, dtype):
        key = (numel, dtype)
        stack = self.free.setdefault(key, [])
        buf = stack.pop() if stack else torch.empty(numel, dtype=dtype, pin_memory=True)
        self.lent.append((key, buf))
        return buf

    def give_back_all(self):
        for key, buf in self.lent:
            self.free[key].append(buf)
        self.lent = []

    def nbytes(self):
        held = [b for bufs in self.free.values() for b in bufs] + [b for _, b in self.lent]
        return sum(b.numel() * b.element_size() for b in held)


class ActivationOffload:
    def __init__(self, device):
        self.device = device
        self.stream = torch.cuda.Stream(device) if device.type == "cuda" else None
        self._pool = _PinnedPool()
        self.order = []  # _Saved records of this micro-batch, in forward order

    @staticmethod
    def _worth_moving(t):
        return t.device.type == "cuda" and t.is_contiguous() and t.numel() * t.element_size() >= MIN_BYTES

    def pack(self, t):
        if not self._worth_moving(t):
            return t
        host = self._pool.take(t.numel(), t.dtype)
        side = self.stream
        side.wait_stream(torch.cuda.current_stream(t.device))
        copied = torch.cuda.Event()
        with torch.cuda.stream(side):
            host.copy_(t.view(-1), non_blocking=True)
            copied.record(side)
        t.record_stream(side)  # the device tensor stays allocated until the copy is done
        rec = _Saved(host, t.shape, t.device, copied, len(self.order))
        self.order.append(rec)
        return rec

    def _fetch(self, rec):
        """Start the host->device copy of `rec` on the side stream (at most once)."""
        if rec.on_device is not None:
            return
        side = self.stream
        side.wait_event(rec.copied)
        rec.arrived = torch.cuda.Event()
        with torch.cuda.stream(side):
            rec.on_device = rec.host.to(rec.device, non_blocking=True)
            rec.arrived.record(side)

    def unpack(self, packed):
        if not isinstance(packed, _Saved):
            return packed
        self._fetch(packed)
        if packed.index > 0:  # prefetch the input of the layer the backward visits next
            self._fetch(self.order[packed.index - 1])
        consumer = torch.cuda.current_stream(packed.device)
        consumer.wait_event(packed.arrived)
        out, packed.on_device = packed.on_device, None  # autograd owns the device copy now
        out.record_stream(consumer)
        return out.view(packed.shape)

    def context(self):
        return torch.autograd.graph.saved_tensors_hooks(self.pack, self.unpack)

    def end_step(self):
        """After the backward: every pinned buffer of this micro-batch can be reused."""
        if self.device.type == "cuda":
            torch.cuda.current_stream(self.device).synchronize()
        self._pool.give_back_all()
        self.order = []

    def pinned_bytes(self):
        return self._pool.nbytes()
