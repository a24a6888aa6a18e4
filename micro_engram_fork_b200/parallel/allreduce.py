"""Mean all-reduce of the replicated dense engram gradients over symmetric peer memory.

One flat fp32 vector per rank is packed into this rank's staging half of a SymmBuffer (two
halves, alternating by call) and ONE kernel (csrc/p2p.cu) signals every peer, waits for all
of them (bounded: a timeout leaves an error in `status` instead of hanging) and sums all
ranks' staged vectors straight out of their memory over NVLink, times 1/world. Same result as
the reference's flat fp32 NCCL all_reduce followed by / world (micro_engram/train/loop.py:316-327).
Collective: every rank calls it the same number of times, in the same order.
"""
import torch
import torch.distributed as dist

from .. import native
from .symm import SymmBuffer

_FLAG_BYTES = 256  # flags [world <= 16] u32, padded


def zero_on_error(out, status):
    """A call whose bounded wait ran out leaves `out` unwritten, or partly written (stale or
    uninitialised values). Replace it by zeros, decided on the device, so no step trains on
    garbage before the host reads the status word at its next logging step and stops the run."""
    return out.masked_fill_(status[:1] != 0, 0.0)


class P2PAllReduce:
    def __init__(self, n, device, group=None, timeout_s=10.0):
        self.n = int(n)
        self.device = torch.device(device)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.timeout_s = float(timeout_s)
        self.stage_off = _FLAG_BYTES
        self.half = (self.n + 3) // 4 * 4  # staging half stride (elements): both halves 16-byte aligned
        self.buf = SymmBuffer(_FLAG_BYTES + 2 * self.half * 4, self.device, group)
        self.buf.view(0, (_FLAG_BYTES // 4,), torch.int32).zero_()
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=group)  # every rank's flags are zero before anyone signals
        self.bases = torch.tensor(self.buf.ptrs, dtype=torch.int64, device=self.device)
        self.status = torch.zeros(2, dtype=torch.int32, device=self.device)
        self.out = torch.empty(self.n, dtype=torch.float32, device=self.device)
        self.calls = 0

    @torch.no_grad()
    def __call__(self, tensors):
        """Mean over ranks of the concatenation of `tensors` (flattened, any float dtype,
        total numel n); returns the fp32 [n] result (a buffer reused by the next call)."""
        self.calls += 1
        stage = self.buf.view(self.stage_off + (self.calls & 1) * self.half * 4, (self.n,), torch.float32)
        k = 0
        for t in tensors:
            m = t.numel()
            stage[k:k + m].copy_(t.reshape(-1))
            k += m
        if k != self.n:
            raise ValueError(f"P2PAllReduce: got {k} values, built for {self.n}")
        native().p2p_allreduce_mean(self.bases, self.rank, self.stage_off, self.n, self.calls, 1.0 / self.world,
                                    self.timeout_s, self.out, self.status)
        return zero_on_error(self.out, self.status)

    def check_status(self):
        st = self.status.tolist()
        if st[0] != 0:
            raise RuntimeError(f"[micro_engram] P2P all-reduce error code {st[0]} (waiting on rank {st[1]})")

    def close(self):
        if self.buf is not None:
            self.buf.close()
            self.buf = None
