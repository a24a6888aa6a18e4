"""Shared test helpers: multi-process gloo runs and the bf16 noise-floor tolerance."""
import os
import traceback

import torch
import torch.multiprocessing as mp


def _worker(rank, world, port, fn, args, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), MICRO_ENGRAM_CPU="1")
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        out = fn(rank, world, *args)
        q.put((rank, "ok", out))
    except Exception:  # noqa: BLE001
        q.put((rank, "err", traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def run_dist(fn, world, *args, timeout=300):
    """Run fn(rank, world, *args) on `world` gloo CPU processes; returns {rank: result}."""
    from conftest import free_port

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fn, args, q)) for r in range(world)]
    for p in procs:
        p.start()
    results, errors = {}, []
    for _ in range(world):
        rank, status, out = q.get(timeout=timeout)
        if status == "ok":
            results[rank] = out
        else:
            errors.append(f"rank {rank}:\n{out}")
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    if errors:
        raise AssertionError("\n".join(errors))
    return results


def noise_floor_check(out, ref32, plain_bf16, rel=1.5, eps=1e-3, name=""):
    """A bf16 kernel passes when its error against the fp32 reference is at most `rel` x the
    error of the plain bf16 PyTorch computation of the same op (plus eps)."""
    err = (out.float() - ref32.float()).abs().max().item()
    base = (plain_bf16.float() - ref32.float()).abs().max().item()
    assert err <= rel * base + eps, f"{name}: kernel error {err:.3e} vs bf16 noise floor {base:.3e}"
    return err, base
