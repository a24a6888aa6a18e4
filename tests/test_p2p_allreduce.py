"""The fused peer-memory all-reduce of the dense engram gradients (csrc/p2p.cu,
micro_engram_fork_b200/parallel/allreduce.py).

One GPU: two "ranks" emulated in one process with two local buffers. With the second rank's
flag set by hand before the launch, the kernel sums both staged vectors (mean); with the flag
never set, its bounded wait runs out and it reports ME_ERR_TIMEOUT without writing (no
kernel waits on another launch). Two GPUs: real ranks over CUDA IPC peer memory, three
calls in a row (both staging halves, reused), against NCCL all_reduce / world."""
import os
import traceback

import pytest
import torch

pytestmark = pytest.mark.gpu

FLAG_BYTES = 256


def _emulated(n, flag_other):
    from micro_engram_fork_b200 import native

    dev = torch.device("cuda", 0)
    half = (n + 3) // 4 * 4  # staging halves start 16-byte aligned
    bufs = [torch.zeros(FLAG_BYTES // 4 + 2 * half, dtype=torch.float32, device=dev) for _ in range(2)]
    vals = [torch.randn(n, device=dev) for _ in range(2)]
    call = 3  # odd call: staging half 1
    for b, v in zip(bufs, vals):
        b[FLAG_BYTES // 4 + half:FLAG_BYTES // 4 + half + n].copy_(v)
    if flag_other:  # rank 1 "has staged" call 3
        bufs[0][:FLAG_BYTES // 4].view(torch.int32)[1] = call
    bases = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=dev)
    out = torch.full((n,), float("nan"), device=dev)
    status = torch.zeros(2, dtype=torch.int32, device=dev)
    native().p2p_allreduce_mean(bases, 0, FLAG_BYTES, n, call, 0.5, 0.3, out, status)
    torch.cuda.synchronize()
    # rank 0 signalled itself and its peer
    assert int(bufs[0][:FLAG_BYTES // 4].view(torch.int32)[0]) == call
    assert int(bufs[1][:FLAG_BYTES // 4].view(torch.int32)[0]) == call
    return out, status, (vals[0] + vals[1]) * 0.5


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
@pytest.mark.parametrize("n", [4096, 1001])
def test_emulated_two_ranks_sum(n):
    out, status, want = _emulated(n, True)
    assert status.tolist() == [0, 0]
    torch.testing.assert_close(out, want, rtol=1e-6, atol=1e-6)


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_missing_peer_times_out():
    from micro_engram_fork_b200.parallel.allreduce import zero_on_error

    out, status, _ = _emulated(1024, False)
    assert status.tolist() == [1, 1]  # ME_ERR_TIMEOUT, waiting on rank 1
    assert bool(torch.isnan(out).all())  # nothing written
    # what the trainer copies into the gradients after such a call: zeros, never the unwritten
    # (here NaN) buffer or a previous call's result
    guarded = zero_on_error(out, status)
    assert bool((guarded == 0).all())


def _worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    try:
        from micro_engram_fork_b200.parallel.allreduce import P2PAllReduce

        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=120))
        shapes = [(1536, 517), (5376,), (3, 7)]
        ar = P2PAllReduce(sum(torch.Size(s).numel() for s in shapes), dev, timeout_s=10.0)
        for call in range(3):
            g = torch.Generator(device=dev).manual_seed(100 * call + rank)
            ts = [torch.randn(s, generator=g, device=dev).to(torch.bfloat16 if i == 0 else torch.float32)
                  for i, s in enumerate(shapes)]
            got = ar(ts).clone()
            want = torch.cat([t.reshape(-1).float() for t in ts])
            dist.all_reduce(want)
            want /= world
            torch.cuda.synchronize()
            ar.check_status()
            torch.testing.assert_close(got, want, rtol=1e-6, atol=1e-6)
        dist.barrier()
        ar.close()
        q.put((rank, "ok", None))
    except Exception:  # noqa: BLE001
        q.put((rank, "err", traceback.format_exc()))
    finally:
        import torch.distributed as dist

        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_p2p_allreduce_two_gpus():
    import torch.multiprocessing as mp

    from conftest import free_port

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    errs = []
    for _ in range(world):
        rank, status, msg = q.get(timeout=600)
        if status != "ok":
            errs.append(f"rank {rank}:\n{msg}")
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    assert not errs, "\n".join(errs)
