"""Checkpoint round trip of the engram tables' optimizer state when the table-sized moments
live in pinned host memory (table_moments_on_host), under an NCCL process group as in
training: RowTables.save writes them as Shard(0) DTensors over host tensors, RowTables.load
reads them back in place into host memory (bit-identical), and one more step from the loaded
state matches one more step from the original (up to the order of the fp32 gradient atomics). Runs as one NCCL rank in a child process."""
import os
import tempfile
import traceback

import pytest
import torch

pytestmark = pytest.mark.gpu


def _engram(dev):
    from micro_engram.module import MicroEngram

    torch.manual_seed(0)
    e = MicroEngram(model_dim=128, table_size=3001, engram_dim=32, num_heads=2, vocab_size=500, gate="scalar_sqrt")
    with torch.no_grad():
        e.value.weight.normal_(std=0.05)
    e = e.to(dev).to(torch.bfloat16)
    e.shard_rows(0, 1, device=dev, dtype=torch.bfloat16, row_capacity=2 * 200)
    return e


def _step(e, rt, dev, seed):
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(3, 500, (2, 200), generator=g).to(dev)
    pos = torch.arange(200).expand(2, 200).to(dev)
    h = (torch.randn(2, 200, 128, generator=g) * 4).to(dev).to(torch.bfloat16)
    e(h, ids, pos).float().pow(2).sum().backward()
    rt.clip(1.0)
    rt.step(1e-2)


def _worker(port, folder, q):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK="0", WORLD_SIZE="1", LOCAL_RANK="0",
                      NCCL_NVLS_ENABLE="0")
    try:
        from micro_engram.rows import RowTables

        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=0, world_size=1, device_id=dev, timeout=datetime.timedelta(seconds=120))

        def make():
            e = _engram(dev)
            rt = RowTables([("model.layers.0.micro_engram.", e)], lr=1e-2, lazy=True, rowwise=True,
                           sparse_grads=True)
            rt.optimizer.move_row_moments_to_host()
            rt.optimizer.materialize_state()
            return e, rt

        e, rt = make()
        assert all(not rt.optimizer.state[p]["exp_avg"].is_cuda for p in rt.params())
        _step(e, rt, dev, 1)
        rt.save(os.path.join(folder, "tables"), os.path.join(folder, "optim"))
        e2, rt2 = make()
        n, loaded = rt2.load(os.path.join(folder, "tables"), os.path.join(folder, "optim"))
        assert n == len(e.row_shards) and loaded
        for p, p2 in zip(rt.params(), rt2.params()):
            s, s2 = rt.optimizer.state[p], rt2.optimizer.state[p2]
            assert not s2["exp_avg"].is_cuda and torch.equal(s["exp_avg"], s2["exp_avg"])
            assert torch.equal(p.detach(), p2.detach())
        for x, r in ((e, rt), (e2, rt2)):
            _step(x, r, dev, 2)
        torch.cuda.synchronize()
        for p, p2 in zip(rt.params(), rt2.params()):  # equal up to the gradient atomics' order
            torch.testing.assert_close(p.detach().float(), p2.detach().float(), rtol=0.05, atol=2e-3)
            torch.testing.assert_close(rt.optimizer.state[p]["exp_avg"].float(),
                                       rt2.optimizer.state[p2]["exp_avg"].float(), rtol=0.05, atol=2e-3)
        e.row_store.check_status()
        q.put(("ok", None))
    except Exception:  # noqa: BLE001
        q.put(("err", traceback.format_exc()))
    finally:
        import torch.distributed as dist

        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_host_moments_checkpoint_round_trip():
    import torch.multiprocessing as mp

    from conftest import free_port

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    folder = tempfile.mkdtemp()
    p = ctx.Process(target=_worker, args=(free_port(), folder, q))
    p.start()
    status, msg = q.get(timeout=600)
    p.join(timeout=120)
    if p.is_alive():
        p.kill()
    assert status == "ok", msg
