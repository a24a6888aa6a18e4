"""The vocab-parallel fused loss on two GPUs, exchanging over peer memory only.

Each rank holds half of a V = 4999 tied head (odd row counts: padded shards) and its own 700
tokens (three loss chunks, the last partial, every 7th token untrained). The loss sum and dH of
each rank are compared with the full-logit loss computed in fp64 on that rank's tokens, with
every rank's loss scaled by a different weight (each rank's dH rows must carry its own weight).
During the loss every NCCL collective of torch.distributed is replaced by a function that fails,
so the test also shows that the CUDA path makes no NCCL call. A second run of the same inputs
must give bitwise the same loss and gradient (the partials and dH are summed in rank order)."""
import os
import traceback

import pytest
import torch

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, softcap, q):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    try:
        from micro_engram.train.head import VocabShard, reference_loss_sum

        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=120))
        torch.manual_seed(0)
        V, d, N = 4999, 256, 700
        W = (torch.randn(V, d) * 0.05).to(torch.bfloat16)
        shard = VocabShard(W, rank, world, softcap=softcap, chunk_tokens=256, device=dev)
        shard.comm()  # built (collectively) before NCCL is switched off below
        g = torch.Generator().manual_seed(100 + rank)
        h0 = torch.randn(N, d, generator=g).to(torch.bfloat16).to(dev)
        labels = torch.randint(0, V, (N,), generator=g).to(dev)
        labels[::7] = -100
        weight = 0.37 * (rank + 1)

        def forbidden(*a, **k):
            raise AssertionError("the CUDA loss path called an NCCL collective")

        names = ("all_gather_into_tensor", "all_reduce", "reduce_scatter_tensor", "all_gather", "all_to_all_single",
                 "broadcast", "barrier")
        saved = {n: getattr(dist, n) for n in names}
        runs = []
        for _ in range(2):
            h = h0.clone().requires_grad_()
            for n in names:
                setattr(dist, n, forbidden)
            try:
                total, count = shard.loss_sum(h, labels)
                (total * weight).backward()
            finally:
                for n, f in saved.items():
                    setattr(dist, n, f)
            torch.cuda.synchronize()
            runs.append((total.detach().clone(), h.grad.clone()))
        shard.check_status()
        assert torch.equal(runs[0][0], runs[1][0]) and torch.equal(runs[0][1], runs[1][1]), "not repeatable"
        total, grad = runs[0]
        h64 = h0.double().requires_grad_()
        ref = reference_loss_sum(h64, labels, W.double().to(dev), softcap)
        (ref * weight).backward()
        assert abs(total.item() - ref.item()) <= 2e-3 * abs(ref.item()) + 1e-2, (total.item(), ref.item())
        err = (grad.double() - h64.grad).abs().max().item()
        assert err <= 3e-2 * h64.grad.abs().max().item() + 1e-4, err
        dist.barrier()
        shard._comm.close()
        q.put((rank, "ok", None))
    except Exception:  # noqa: BLE001
        q.put((rank, "err", traceback.format_exc()))
    finally:
        import torch.distributed as dist

        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("softcap", [30.0, None])
def test_vocab_parallel_loss_two_gpus(softcap):
    import torch.multiprocessing as mp

    from conftest import free_port

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, softcap, q)) for r in range(world)]
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
