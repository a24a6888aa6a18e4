"""Peer-memory collectives of the vocab-parallel loss (the CUDA path runs no NCCL call).

Per chunk of tokens the loss needs every rank's hidden states and labels (an all-gather), the
merge of every rank's per-token (max, sum-exp, target) partials (an all-gather of 3 floats per
token and rank, merged locally in rank order), and each token's dH summed over the ranks' vocab
slices, back on the token's rank (a reduce-scatter). Here:

  gather       each rank copies its rows into its half of a symmetric staging buffer; ONE kernel
               signals every peer, waits (bounded) for all of them and copies every rank's stage
               out of its memory over NVLink (p2p_gather)
  scatter-sum  the dH GEMM's epilogue stores each output tile straight into this rank's receive
               slot on the GPU that owns those tokens (gemm_f32_scatter); then one kernel per rank
               signals, waits for every peer's stores to be done and sums its slots in a fixed
               order (p2p_sum_slots), so the result is the same on every run

Each region is double-buffered by call parity: a rank writes the stage of call k only after its
kernel of call k-1 saw every peer's signal k-1, and a peer signals k-1 only after its kernel of
call k-2 (the last reader of that parity) finished. Every wait is bounded (timeout_s): a peer
that never arrives leaves an error code in `status` instead of a hang. Plain P2P loads and
stores, no multicast. Collective: every rank makes the same calls in the same order.

Reference semantics: micro_engram/train/head.py:76-165 (NCCL all_gather of hidden and labels,
all_reduce of the partials, reduce_scatter of dH).
"""
import torch
import torch.distributed as dist

from .. import native
from .symm import SymmBuffer

_FLAGS = 256  # bytes of flag words at the start of each region


def _round16(n):
    return (n + 15) // 16 * 16


class VocabComm:
    def __init__(self, n_max, d, device, group=None, timeout_s=10.0):
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.n_max, self.d, self.device = int(n_max), int(d), torch.device(device)
        self.timeout_s = float(timeout_s)
        # gather region: [flags][2 halves of (hidden bf16 [n, d] | labels int64 [n] | partials fp32 [3, world*n])]
        self.h_bytes = _round16(self.n_max * self.d * 2)
        self.l_bytes = _round16(self.n_max * 8)
        self.p_bytes = _round16(3 * self.world * self.n_max * 4)
        self.half = self.h_bytes + self.l_bytes + self.p_bytes
        self.gbuf = SymmBuffer(_FLAGS + 2 * self.half, self.device, group)
        # receive region: [flags][2 parities][world slots][n, d] fp32
        self.slot_elems = self.n_max * self.d
        self.rbuf = SymmBuffer(_FLAGS + 2 * self.world * self.slot_elems * 4, self.device, group)
        for b in (self.gbuf, self.rbuf):
            b.view(0, (_FLAGS // 4,), torch.int32).zero_()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)  # every rank's flags are zero before anyone signals
        self.gbases = torch.tensor(self.gbuf.ptrs, dtype=torch.int64, device=self.device)
        self.rbases = torch.tensor(self.rbuf.ptrs, dtype=torch.int64, device=self.device)
        # per parity: every rank's receive area (slot 0) for the scattering GEMM's epilogue
        self.recv = [torch.tensor([p + _FLAGS + par * self.world * self.slot_elems * 4 for p in self.rbuf.ptrs],
                                  dtype=torch.int64, device=self.device) for par in (0, 1)]
        self.status = torch.zeros(2, dtype=torch.int32, device=self.device)
        self.gather_calls = self.scatter_calls = 0

    def _stage(self, rel):
        return _FLAGS + (self.gather_calls & 1) * self.half + rel

    def _exchange(self, rel, nbytes, out):
        C = native()
        C.p2p_gather(self.gbases, self.rank, self.gather_calls, _FLAGS + rel, self.half, _round16(nbytes) // 16, out,
                     self.timeout_s, self.status)

    def gather(self, h, labels):
        """(hidden [world * n, d], labels [world * n]) of every rank's n rows, rank-major."""
        n = h.shape[0]
        if n > self.n_max:
            raise ValueError(f"VocabComm: chunk of {n} tokens, built for {self.n_max}")
        self.gather_calls += 1
        self.gbuf.view(self._stage(0), (n, self.d), torch.bfloat16).copy_(h)
        self.gbuf.view(self._stage(self.h_bytes), (n,), torch.int64).copy_(labels)
        H = torch.empty(self.world * n, self.d, dtype=torch.bfloat16, device=self.device)
        self._exchange(0, n * self.d * 2, H)  # this signal also publishes the labels below
        L = torch.empty(self.world, _round16(n * 8) // 8, dtype=torch.int64, device=self.device)
        self._exchange(self.h_bytes, n * 8, L)
        return H, L[:, :n].reshape(-1)

    def merge(self, m, s, tgt):
        """(log-sum-exp, target logit) per gathered token from every rank's partials: each rank's
        (m, s, tgt) [world * n] fp32 over its own vocab rows, s = sum of exp(z - m)."""
        k = m.numel()
        if k > self.world * self.n_max:
            raise ValueError("VocabComm: partials larger than built for")
        self.gather_calls += 1
        torch.stack([m, s, tgt], out=self.gbuf.view(self._stage(self.h_bytes + self.l_bytes), (3, k), torch.float32))
        every = torch.empty(self.world, _round16(3 * k * 4) // 4, dtype=torch.float32, device=self.device)
        self._exchange(self.h_bytes + self.l_bytes, 3 * k * 4, every)
        every = every[:, :3 * k].view(self.world, 3, k)
        top = every[:, 0].amax(dim=0)
        total = (every[:, 1] * torch.exp(every[:, 0] - top)).sum(dim=0)
        return top + torch.log(total), every[:, 2].sum(dim=0)

    def scatter_sum(self, z, w, out):
        """out [n, d] fp32 = this rank's rows of sum over ranks of (z . w), z [world * n, K]:
        the GEMM stores each rank's n rows into that rank's receive slot, then the slots are
        summed locally."""
        n = out.shape[0]
        if n > self.n_max or z.shape[0] != self.world * n:
            raise ValueError("VocabComm: scatter of a chunk larger than built for")
        self.scatter_calls += 1
        C = native()
        C.gemm_f32_scatter(z, w, self.recv[self.scatter_calls & 1], n, self.rank, self.slot_elems)
        C.p2p_sum_slots(self.rbases, self.rank, self.scatter_calls, _FLAGS, self.slot_elems, out, self.timeout_s,
                        self.status)
        return out

    def check_status(self):
        code = self.status.tolist()
        if code[0] != 0:
            raise RuntimeError(f"[micro_engram] vocab-loss peer exchange error {code[0]} (waiting on rank {code[1]})")

    def close(self):
        for b in (self.gbuf, self.rbuf):
            b.close()
