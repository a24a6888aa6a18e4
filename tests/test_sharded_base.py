"""The row-sharded frozen base (base_placement: sharded) and the all-gather its GEMMs carry.

One GPU: the tcgen05 GEMM's side-copy warp copies a segment table (two "peer" buffers into one
destination) while it computes, alone or split with the standalone gather kernel, and the GEMM
result is unchanged by it. Two GPUs: a decoder whose layers are row-sharded over two ranks
(gathered over NVLink by the GEMMs) gives bitwise the same forward output and input gradient
as the same decoder replicated, over two micro-batches (forward 0..L-1, backward L-1..0 and
again: every gather slot is reused)."""
import os
import traceback

import pytest
import torch

pytestmark = pytest.mark.gpu


def _dev():
    return torch.device("cuda", 0)


def _segments(parts, dst):
    rows, start, off = [], 0, 0
    for p in parts:
        n16 = p.numel() * p.element_size() // 16
        rows.append((p.data_ptr(), dst.data_ptr() + off, start, n16))
        start += n16
        off += p.numel() * p.element_size()
    return torch.tensor(rows, dtype=torch.int64, device=dst.device), start


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
@pytest.mark.parametrize("split", [None, 0.37])
def test_gemm_carries_copy(split):
    from micro_engram_fork_b200 import native

    C = native()
    torch.manual_seed(0)
    parts = [torch.randn(1000, 520, device=_dev()).to(torch.bfloat16), torch.randn(777, 520, device=_dev()).to(
        torch.bfloat16)]
    dst = torch.zeros(1777, 520, device=_dev(), dtype=torch.bfloat16)
    segs, total = _segments(parts, dst)
    A = torch.randn(2048, 1536, device=_dev()).to(torch.bfloat16)
    W = (torch.randn(5376, 1536, device=_dev()) / 40).to(torch.bfloat16)
    plain = C.gemm(A, W, True, None)
    stop = total if split is None else int(total * split)
    C.gemm_carry_copy(0, segs.data_ptr(), segs.shape[0], 0, stop)
    carried = C.gemm(A, W, True, None)
    if stop < total:
        C.layer_gather(segs, stop, total)
    torch.cuda.synchronize()
    assert int(C.gemm_status(0)[0]) == 0
    assert torch.equal(carried, plain), "the side copy changed the GEMM result"
    assert torch.equal(dst, torch.cat(parts)), "side copy + standalone gather did not copy the segments"
    # a GEMM launched later carries nothing (the job is consumed by one launch)
    dst.zero_()
    C.gemm(A, W, True, None)
    torch.cuda.synchronize()
    assert int(dst.abs().sum()) == 0


def _worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    try:
        from micro_engram_fork_b200.models import gemma as G
        from micro_engram_fork_b200.parallel import sharded_base as SB

        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=120))
        cfg = G.tiny_config(num_hidden_layers=5, layer_types=["sliding_attention"] * 4 + ["full_attention"])

        def build():
            m = G.GemmaTextModel(cfg).to(dev)
            for layer in m.layers:
                layer._relink()
            G.init_random_(m, seed=3)
            G.cast_projections_(m, torch.bfloat16)
            for layer in m.layers:
                layer.gradient_checkpointing = "none"
            return m

        ref, sharded = build(), build()
        sb = SB.ShardedBase(sharded.layers, rank, world, dev)
        SB.activate(sb)
        lens = [100, 300, 37, 75]
        pos = torch.cat([torch.arange(n) for n in lens]).to(dev)
        outs = []
        for model in (ref, sharded):
            if model is ref:
                SB.activate(None)
            else:
                SB.activate(sb)
            torch.manual_seed(7)
            res = []
            for _ in range(2):  # two micro-batches: every slot is reused in both directions
                x = torch.randn(pos.numel(), cfg.hidden_size, device=dev).to(torch.bfloat16).requires_grad_()
                y = model(x, pos)
                y.float().square().sum().backward()
                res += [y.detach().clone(), x.grad.clone()]
            outs.append(res)
        torch.cuda.synchronize()
        from micro_engram_fork_b200 import native

        assert int(native().gemm_status(rank)[0]) == 0
        for a, b in zip(*outs):
            assert torch.equal(a, b), f"sharded differs from replicated: {(a.float() - b.float()).abs().max()}"
        dist.barrier()
        SB.activate(None)
        sb.close()
        q.put((rank, "ok", None))
    except Exception:  # noqa: BLE001
        q.put((rank, "err", traceback.format_exc()))
    finally:
        import torch.distributed as dist

        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_matches_replicated_two_gpus():
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
