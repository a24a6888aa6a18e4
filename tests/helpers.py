"""Shared test helpers: multi-process gloo runs and the bf16 noise-floor tolerance."""
import os
import traceback

import torch
import torch.multiprocessing as mp


def _pack(x):
    """Tensors travel between processes by value (numpy), not through shared-memory handles that
    die with the worker."""
    if isinstance(x, torch.Tensor):
        return ("__tensor__", x.detach().cpu().float().numpy() if x.dtype == torch.bfloat16 else x.detach().cpu().numpy(),
                str(x.dtype))
    if isinstance(x, (list, tuple)):
        return type(x)(_pack(v) for v in x)
    if isinstance(x, dict):
        return {k: _pack(v) for k, v in x.items()}
    return x


def _unpack(x):
    if isinstance(x, tuple) and len(x) == 3 and x[0] == "__tensor__":
        t = torch.from_numpy(x[1])
        return t.to(getattr(torch, x[2].split(".")[-1]))
    if isinstance(x, (list, tuple)):
        return type(x)(_unpack(v) for v in x)
    if isinstance(x, dict):
        return {k: _unpack(v) for k, v in x.items()}
    return x


def _worker(rank, world, port, fn, args, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), MICRO_ENGRAM_CPU="1")
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        out = fn(rank, world, *args)
        q.put((rank, "ok", _pack(out)))
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
            results[rank] = _unpack(out)
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
