"""Per-phase device timers and NVTX ranges for the training step.

`PhaseTimers` brackets named phases of a step with CUDA events on the current stream (no
synchronisation while the step runs); `report()` synchronises once and returns the summed
milliseconds per phase. Each phase is also an NVTX range (visible in Nsight Systems / ncu's
NVTX filters). On CPU, or when disabled, every call is a no-op.

    timers = PhaseTimers(enabled=True)
    with timers.phase("forward"):
        ...
    timers.report()   # {"forward": 812.4, ...}
"""
import contextlib

import torch


class PhaseTimers:
    def __init__(self, enabled=False, device=None):
        self.enabled = bool(enabled) and torch.cuda.is_available() and (device is None or device.type == "cuda")
        self.pending = []   # (name, start event, end event)
        self.totals = {}

    @contextlib.contextmanager
    def phase(self, name):
        if not self.enabled:
            yield
            return
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push(name)
        start.record()
        try:
            yield
        finally:
            end.record()
            torch.cuda.nvtx.range_pop()
            self.pending.append((name, start, end))

    def report(self, reset=True):
        """{phase: milliseconds} summed over every interval recorded since the last reset."""
        if not self.enabled:
            return {}
        if self.pending:
            self.pending[-1][2].synchronize()
        for name, start, end in self.pending:
            self.totals[name] = self.totals.get(name, 0.0) + start.elapsed_time(end)
        self.pending = []
        out = {k: round(v, 3) for k, v in self.totals.items()}
        if reset:
            self.totals = {}
        return out


def nvtx_range(name):
    """An NVTX range as a context manager (no-op without CUDA)."""
    if torch.cuda.is_available():
        return torch.cuda.nvtx.range(name)
    return contextlib.nullcontext()
