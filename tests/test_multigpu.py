"""Row-sharded engram on 2+ GPUs (NCCL + peer-mapped row stores): the fused gather reads
rows straight from their owners over NVLink, the backward pushes row gradients into the
owners' compact accumulators (peer atomics claim the slots), and the touched-row Adam
updates them. The oracle is the full-table
engram with FSDP-style averaged gradients, run on the same GPUs. Skipped with fewer than 2
GPUs; every rank runs the same collectives in the same order."""
import copy
import os
import traceback

import pytest
import torch

pytestmark = pytest.mark.gpu

N_ROWS, D, E = 4099, 256, 64


def _worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    try:
        import datetime

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=120))
        from micro_engram.module import MicroEngram
        from micro_engram.rows import RowTables, row_range

        torch.manual_seed(0)
        full = MicroEngram(model_dim=D, table_size=N_ROWS, engram_dim=E, num_heads=2, vocab_size=500,
                           gate="scalar_sqrt", table_sizes={3: 2053})
        with torch.no_grad():
            full.value.weight.normal_(std=0.05)
        full = full.to(dev).to(torch.bfloat16)
        sh = copy.deepcopy(full)
        # 600 lookups per table per rank and step: the compact accumulators hold 600 x world slots
        sh.shard_rows(rank, world, device=dev, dtype=torch.bfloat16, row_capacity=600 * world)
        assert sh.row_store is not None and sh.row_store.world == world
        g = torch.Generator().manual_seed(10 + rank)
        ids = torch.randint(3, 500, (2, 300), generator=g).to(dev)
        ids[0, :20] = 7
        pos = torch.cat([torch.arange(120), torch.arange(180)]).expand(2, 300).to(dev)
        h = (torch.randn(2, 300, D, generator=g) * 4).to(dev).to(torch.bfloat16)
        out_f = full(h, ids, pos)
        out_s = sh(h, ids, pos)
        err = (out_f.float() - out_s.float()).abs().max().item()
        assert err <= 2e-2 * out_f.float().abs().max().item(), f"forward differs: {err}"
        out_f.float().pow(2).sum().backward()
        out_s.float().pow(2).sum().backward()
        torch.cuda.synchronize()
        dist.barrier()  # every peer's pushes have landed
        sh.row_store.check_status()
        for k, t in enumerate(full.tables):
            gw = t.weight.grad.clone()
            dist.all_reduce(gw)
            gw /= world
            start, count = row_range(sh.table_rows[k], rank, world)
            rows, acc = sh.row_store.touched(k)
            dense = torch.zeros(count, E, device=dev)
            dense[rows] = acc
            ref = gw[start:start + count]
            e2 = (dense - ref).abs().max().item()
            assert e2 <= 3e-2 * ref.abs().max().item() + 1e-6, f"table {k} grads differ: {e2}"
        # one optimizer step through RowTables (touched-row rowwise Adam)
        rt = RowTables([("model.layers.0.micro_engram.", sh)], lr=1e-2, lazy=True, rowwise=True, sparse_grads=True)
        before = [p.detach().clone() for p in sh.row_shards]
        norm = rt.clip(1.0)
        rt.step(1e-2)
        torch.cuda.synchronize()
        moved = sum(int((p.detach() != b).any(dim=1).sum()) for p, b in zip(sh.row_shards, before))
        touched_total = torch.tensor([moved], device=dev)
        dist.all_reduce(touched_total)
        assert norm > 0 and int(touched_total) > 0
        q.put((rank, "ok", None))
    except Exception:  # noqa: BLE001
        q.put((rank, "err", traceback.format_exc()))
    finally:
        import torch.distributed as dist

        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_row_sharded_engram_two_gpus():
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
