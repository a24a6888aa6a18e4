"""The fused row-parallel linear (GEMM -> reduce-scatter -> all-gather over peer memory) against
fp32 PyTorch: y = sum over ranks of x_r . W_r^T.

One GPU: `world` ranks emulated with one plain buffer each. The flag words every barrier waits
for are published by the test before the launches, and the launch order (every rank's GEMM,
then every rank's sum, then every rank's gather) means every wait is satisfied by data an
earlier, finished launch wrote: no kernel depends on another running at the same time. A call
whose flags nobody publishes must end with a timeout status.

Two GPUs (skipped with fewer): TPRowLinear itself over NCCL-initialised ranks, several calls of
different row counts (both parities, a ragged M, a decode-sized M)."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
_FLAGS = 256


def _round16(n):
    return (n + 15) // 16 * 16


def _close(got, want):
    """bf16 rounding of an fp32 sum: half an ulp of bf16 plus fp32 accumulation noise."""
    err = (got.double() - want.double()).abs()
    lim = want.double().abs() * 2.0 ** -8 + 1e-4 * want.double().abs().max() + 1e-6
    return bool((err <= lim).all()), err.max().item()


def _emulated(world, M, N, K, publish=True):
    from micro_engram_fork_b200 import native

    C = native()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(M + N + world)
    xs = [torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16) for _ in range(world)]
    ws = [(torch.randn(N, K, device=dev, generator=g) * K ** -0.5).to(torch.bfloat16) for _ in range(world)]
    rows = -(-M // world)
    slot = rows * N
    half = _round16(rows * N * 2)
    rb = [torch.zeros(_FLAGS + 2 * world * slot * 4, dtype=torch.uint8, device=dev) for _ in range(world)]
    gb = [torch.zeros(_FLAGS + 2 * half, dtype=torch.uint8, device=dev) for _ in range(world)]
    rbases = torch.tensor([b.data_ptr() for b in rb], dtype=torch.int64, device=dev)
    gbases = torch.tensor([b.data_ptr() for b in gb], dtype=torch.int64, device=dev)
    status = [torch.zeros(2, dtype=torch.int32, device=dev) for _ in range(world)]
    call, par = 1, 1
    recv = torch.tensor([b.data_ptr() + _FLAGS + par * world * slot * 4 for b in rb], dtype=torch.int64, device=dev)
    if publish:
        for b in rb + gb:
            b[:_FLAGS].view(torch.int32)[:world] = call
    outs = []
    for r in range(world):
        C.gemm_f32_scatter(xs[r], ws[r], recv, rows, r, slot, True)
    stages = [b[_FLAGS + par * half:_FLAGS + par * half + rows * N * 2].view(torch.bfloat16).view(rows, N) for b in gb]
    for r in range(world):
        C.p2p_sum_slots(rbases, r, call, _FLAGS, slot, stages[r], 0.2 if not publish else 5.0, status[r])
    for r in range(world):
        y = torch.empty(world * rows, N, dtype=torch.bfloat16, device=dev)
        C.p2p_gather(gbases, r, call, _FLAGS, half, rows * N * 2 // 16, y, 0.2 if not publish else 5.0, status[r],
                     True)
        outs.append(y[:M])
    torch.cuda.synchronize()
    want = sum(x.float() @ w.float().t() for x, w in zip(xs, ws))
    return outs, want, [s.tolist() for s in status]


@cuda
@pytest.mark.parametrize("world,M,N,K", [(2, 64, 1536, 2048), (2, 301, 1024, 512), (3, 2048, 5376, 1024),
                                         (2, 8192, 2688, 768), (4, 40, 256, 4096)])
def test_row_linear_emulated_ranks(world, M, N, K):
    outs, want, status = _emulated(world, M, N, K)
    for r in range(world):
        assert status[r] == [0, 0], status
        ok, err = _close(outs[r], want)
        assert ok, f"rank {r}: max err {err}"
        assert torch.equal(outs[r], outs[0]), "ranks disagree"


@cuda
def test_row_linear_wait_times_out():
    """Nobody publishes the flags: rank 0's kernels run first, so their waits for rank 1 run out;
    rank 0 reports the timeout (on rank 1) and its output is poisoned, not stale. (Rank 1's
    kernels run after rank 0's signalled, so in this sequential emulation their waits pass.)"""
    outs, _want, status = _emulated(2, 64, 256, 256, publish=False)
    assert status[0] == [1, 1]  # ME_ERR_TIMEOUT, waiting on rank 1
    assert torch.isnan(outs[0].float()).all()


def _worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    try:
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        from micro_engram_fork_b200.parallel.tp_linear import TPRowLinear

        N, K = 5376, 1024
        lin = TPRowLinear(4096, N, dev)
        errs = []
        for i, M in enumerate((4096, 64, 301, 1, 2048)):
            g = torch.Generator(device=dev).manual_seed(100 * i + rank)
            x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
            w = (torch.randn(N, K, device=dev, generator=g) * K ** -0.5).to(torch.bfloat16)
            y = lin(x, w)
            xs = [torch.empty_like(x) for _ in range(world)]
            wl = [torch.empty_like(w) for _ in range(world)]
            dist.all_gather(xs, x)
            dist.all_gather(wl, w)
            want = sum(a.float() @ b.float().t() for a, b in zip(xs, wl))
            ok, err = _close(y, want)
            every = [torch.empty_like(y) for _ in range(world)]
            dist.all_gather(every, y.contiguous())
            errs.append((M, ok, err, all(torch.equal(e, every[0]) for e in every)))
        torch.cuda.synchronize()
        lin.check_status()
        dist.barrier()
        lin.close()
        dist.destroy_process_group()
        q.put((rank, errs))
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        q.put((rank, repr(exc)))


@cuda
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp_row_linear_two_gpus():
    import multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r, res in got.items():
        assert not isinstance(res, str), f"rank {r}: {res}"
        for M, ok, err, same in res:
            assert ok, f"rank {r}, M={M}: max err {err}"
            assert same, f"M={M}: ranks disagree"
