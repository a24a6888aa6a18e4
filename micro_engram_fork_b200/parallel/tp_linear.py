"""Row-parallel linear with its all-reduce fused into the GEMM (tensor-parallel serving).

y = sum over the TP ranks r of x_r . W_r^T, replicated on every rank: x_r [M, K/tp] is this
rank's slice of the input features and W_r [N, K/tp] its slice of the weight (the layout of
vLLM's RowParallelLinear, used for o_proj and down_proj). vLLM runs a library GEMM and then an
all-reduce of the bf16 partials (vllm/model_executor/layers/linear.py, RowParallelLinear.
forward). Here the reduction is an NVLink reduce-scatter + all-gather over peer memory:

  1. the tcgen05 GEMM keeps its fp32 accumulators and its epilogue stores each row block of
     the partial straight into the receive slot of the rank that owns those rows (M rows cut
     into `world` equal blocks), so the reduce-scatter's transfer overlaps the GEMM tile by
     tile (gemm_f32_scatter with a K-major weight; one partial wave of tiles, as in decode, is
     split along K so every SM streams the weight)
  2. one kernel per rank waits (bounded) until every peer's stores are done, sums its slots in
     rank order in fp32 and rounds once to bf16 into its stage (p2p_sum_slots)
  3. one kernel per rank waits for every peer's stage and copies all of them over NVLink (the
     all-gather, p2p_gather)

The partials stay fp32 until the one final rounding (an all-reduce of bf16 partials rounds at
every add), and the fixed summation order gives the same bits on every rank and every run.
Both regions are double-buffered by call parity as in the vocab-parallel loss
(parallel/vocab_comm.py): a rank writes parity k & 1 only after its own kernels of call k - 1
saw every peer arrive at call k - 1, which every peer does only after its readers of call k - 2
finished. Collective: every rank makes the same calls in the same order, which a TP forward
does. Plain P2P loads and stores, no multicast. A wait that runs out leaves an error code in
`status` (check_status) instead of hanging the GPU, and the call's output is all NaN rather
than another call's values, so no host sync is needed to keep stale data out.
"""
import torch
import torch.distributed as dist

from .. import native
from .symm import SymmBuffer

_FLAGS = 256  # bytes of flag words at the start of each region


def _round16(n):
    return (n + 15) // 16 * 16


class TPRowLinear:
    """Fused row-parallel linear for up to `n_max` rows of `n_out` output features."""

    def __init__(self, n_max, n_out, device, group=None, timeout_s=10.0):
        if n_out % 8:
            raise ValueError(f"TPRowLinear: output features {n_out} not a multiple of 8")
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.n_out, self.device, self.timeout_s = int(n_out), torch.device(device), float(timeout_s)
        self.rows = -(-int(n_max) // self.world)  # rows each rank owns at most
        self.n_max = self.rows * self.world
        self.slot_elems = self.rows * self.n_out  # fp32 partial of one peer's row block
        self.rbuf = SymmBuffer(_FLAGS + 2 * self.world * self.slot_elems * 4, self.device, group)
        self.half = _round16(self.rows * self.n_out * 2)  # bf16 stage of one parity
        self.gbuf = SymmBuffer(_FLAGS + 2 * self.half, self.device, group)
        for b in (self.rbuf, self.gbuf):
            b.view(0, (_FLAGS // 4,), torch.int32).zero_()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)  # every rank's flags are zero before anyone signals
        self.rbases = torch.tensor(self.rbuf.ptrs, dtype=torch.int64, device=self.device)
        self.gbases = torch.tensor(self.gbuf.ptrs, dtype=torch.int64, device=self.device)
        self.recv = [torch.tensor([p + _FLAGS + par * self.world * self.slot_elems * 4 for p in self.rbuf.ptrs],
                                  dtype=torch.int64, device=self.device) for par in (0, 1)]
        self.status = torch.zeros(2, dtype=torch.int32, device=self.device)
        self.calls = 0

    def __call__(self, x, weight):
        """x [M, K_local] bf16, weight [n_out, K_local] bf16 -> [M, n_out] bf16, summed over ranks."""
        M = x.shape[0]
        if M > self.n_max or weight.shape[0] != self.n_out:
            raise ValueError(f"TPRowLinear: {M} rows x {weight.shape[0]} features, built for "
                             f"{self.n_max} x {self.n_out}")
        n = max(1, -(-M // self.world))
        self.calls += 1
        par = self.calls & 1
        C = native()
        C.gemm_f32_scatter(x, weight, self.recv[par], n, self.rank, self.slot_elems, True)
        stage = self.gbuf.view(_FLAGS + par * self.half, (n, self.n_out), torch.bfloat16)
        C.p2p_sum_slots(self.rbases, self.rank, self.calls, _FLAGS, self.slot_elems, stage, self.timeout_s,
                        self.status)
        y = torch.empty(self.world * n, self.n_out, dtype=torch.bfloat16, device=self.device)
        C.p2p_gather(self.gbases, self.rank, self.calls, _FLAGS, self.half, n * self.n_out * 2 // 16, y,
                     self.timeout_s, self.status, True)  # NaN rows, not stale ones, if a wait ran out
        return y[:M]

    def check_status(self):
        code = self.status.tolist()
        if code[0] != 0:
            raise RuntimeError(f"[micro_engram] TP row-linear peer exchange error {code[0]} (waiting on rank "
                               f"{code[1]})")

    def close(self):
        for b in (self.rbuf, self.gbuf):
            b.close()
