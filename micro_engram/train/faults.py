"""Host-side fault injection and failure detection for the trainer.

Fault injection (tests and drills only): MICRO_ENGRAM_FAULT="<rank>:<step>[:<kind>]" makes that
rank fail when it is about to run optimizer step <step> (1-based), between steps, with none of
its kernels or collectives in flight:
    raise   (default) raise FaultInjected; main()'s fail-fast handler exits the process (1)
    exit    leave at once with os._exit(3), as a crashed process would
    hang    stop calling collectives (sleep); the others' next collective times out
No fault is ever injected on a GPU: the failure is made on the host, the surviving ranks learn
of it through their process group (a closed connection, or the group's timeout, set by
MICRO_ENGRAM_PG_TIMEOUT_S) and fail fast themselves.

Failure detection on the device side is the status word every bounded wait of the sm_100a
kernels writes into (row store, P2P all-reduce, tcgen05 GEMM and attention); `check_device`
raises when any of them recorded an error.
"""
import os
import time


class FaultInjected(RuntimeError):
    pass


def parse_fault(spec):
    """(rank, step, kind) from "r:s[:kind]", or None."""
    if not spec:
        return None
    parts = spec.split(":")
    if len(parts) not in (2, 3):
        raise ValueError(f"MICRO_ENGRAM_FAULT must be rank:step[:raise|exit|hang], got {spec!r}")
    kind = parts[2] if len(parts) == 3 else "raise"
    if kind not in ("raise", "exit", "hang"):
        raise ValueError(f"MICRO_ENGRAM_FAULT kind must be raise, exit or hang, got {kind!r}")
    return int(parts[0]), int(parts[1]), kind


class FaultHook:
    """Checked by the training loop before each optimizer step."""

    def __init__(self, rank, spec=None):
        self.rank = rank
        self.fault = parse_fault(spec if spec is not None else os.environ.get("MICRO_ENGRAM_FAULT"))

    def before_step(self, step):
        if self.fault is None:
            return
        rank, at, kind = self.fault
        if rank != self.rank or step != at:
            return
        if kind == "exit":
            os._exit(3)
        if kind == "hang":
            while True:  # host-side only: this process stops taking part; nothing waits on the GPU
                time.sleep(3600)
        raise FaultInjected(f"injected fault on rank {rank} before step {at}")


def check_device(trainer):
    """Raise when a kernel's bounded wait or bounds check recorded an error (reads the status
    words: a host synchronisation, so the loop calls it at logging steps only)."""
    for slot in trainer.slots:
        store = slot.engram.__dict__.get("row_store")
        if store is not None:
            store.check_status()
    ar = getattr(trainer, "_p2p_ar", None)
    if ar is not None:
        ar.check_status()
    vocab = getattr(trainer, "vocab", None)
    if vocab is not None:
        vocab.check_status()
    if trainer.device.type == "cuda":
        from micro_engram_fork_b200 import native

        C = native()
        dev = trainer.device.index or 0
        for name, st in (("tcgen05 GEMM", C.gemm_status(dev)), ("tcgen05 attention", C.attn_tc_status(dev))):
            code = st.tolist()
            if code[0] != 0:
                raise RuntimeError(f"[micro_engram] {name} kernel error {code[0]} (where {code[1]})")
