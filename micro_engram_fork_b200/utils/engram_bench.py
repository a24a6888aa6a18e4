"""The isolated engram module benchmark on 1..8 GPUs of one node.

    python -m micro_engram_fork_b200.utils.engram_bench [--steps 5 --warmup 3]
    torchrun --nproc-per-node N -m micro_engram_fork_b200.utils.engram_bench [--impl reference]

Per GPU: hidden states of 8 rows x 8192 tokens x d 5376 (bf16, N(0, 1)) and token ids
Zipf(1.1) over a 262,144 vocabulary in documents of 256-4096 tokens; one engram with 2/3/4-gram
tables {1572864, 4194304, 4194304} rows x 8 heads x dim 64, scalar_sqrt gate, bf16 tables,
row-sharded over the GPUs, rowwise Adam with stochastic rounding. A step is the forward (hash,
fetch of every looked-up row from its owner, gated add into the hidden states), the backward
(every looked-up row's gradient returned to its owner, dense gradients) and the optimizer
(touched-row Adam on the tables, AdamW on the dense weights; dense gradients averaged over
ranks).

ours       the row store in peer memory: gather kernel reading owners' rows over NVLink,
           tcgen05 key/value GEMMs, fused gate, row-gradient push into the owners' compact
           accumulators, touched-row Adam, P2P dense all-reduce
reference  the reference's MicroEngram with micro_engram_sharding: rows (unique ids and rows
           exchanged with all_to_all over NCCL) and its RowTables optimizer, from baseline/_ref

Timing: CUDA events around K steps after W warm-up steps, barrier + synchronize on both sides,
max over ranks. The roofline is the slower of the tensor-core time of the six projection GEMMs
(key and value: forward, input gradient, weight gradient) at the measured bf16 peak and the
NVLink time of the bytes that must cross it per GPU (each remote lookup's 128-byte bf16 row in,
its bf16 gradient back with an 8-byte header; (world-1)/world of the lookups are remote) at the
measured 770 GB/s per direction; frac_of_roofline = roofline / measured step.
"""
import argparse
import json
import os
import sys

TABLES = {2: 1572864, 3: 4194304, 4: 4194304}
HEADS, EDIM, DMODEL, VOCAB = 8, 64, 5376, 262144
ROWS_PER_GPU, SEQ = 8, 8192
NVLINK_GBS = 770.0


def _setup_dist():
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if "MASTER_ADDR" not in os.environ:
        import socket

        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            os.environ["MASTER_PORT"] = str(s.getsockname()[1])
        os.environ["MASTER_ADDR"] = "127.0.0.1"
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if not dist.is_initialized():
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    return rank, world, dev


def _inputs(rank, dev, seed=0):
    """ids [8, 8192] Zipf(1.1) with position_ids restarting per document, hidden [8, 8192, d]."""
    import numpy as np
    import torch

    rng = np.random.default_rng(seed + 1000 * rank)
    p = np.arange(1, VOCAB + 1, dtype=np.float64) ** -1.1
    cdf = np.cumsum(p / p.sum())
    ids = np.searchsorted(cdf, rng.random((ROWS_PER_GPU, SEQ))).astype(np.int64)
    pos = np.zeros((ROWS_PER_GPU, SEQ), dtype=np.int64)
    for r in range(ROWS_PER_GPU):
        t = 0
        while t < SEQ:
            n = int(rng.integers(256, 4097))
            pos[r, t:t + n] = np.arange(min(n, SEQ - t))
            t += n
    g = torch.Generator(device=dev).manual_seed(seed + rank)
    hidden = torch.randn(ROWS_PER_GPU, SEQ, DMODEL, device=dev, generator=g).to(torch.bfloat16)
    return torch.from_numpy(ids).to(dev), torch.from_numpy(pos).to(dev), hidden


def _time(step, steps, warmup, world):
    import torch
    import torch.distributed as dist

    for _ in range(warmup):
        step()
    dist.barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        step()
    t1.record()
    dist.barrier()
    torch.cuda.synchronize()
    ms = torch.tensor([t0.elapsed_time(t1) / steps], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms)


def _engram_ours(dev, rank, world):
    import torch

    from micro_engram.module import MicroEngram
    from micro_engram.rows import RowTables, _group

    e = MicroEngram(model_dim=DMODEL, engram_dim=EDIM, num_heads=HEADS, orders=(2, 3, 4), table_sizes=TABLES,
                    vocab_size=VOCAB, gate="scalar_sqrt", build_tables=False, seed=0)
    e.to(dev)
    with torch.no_grad():
        e.value.weight.normal_(0, 0.02)  # a trained-looking output projection: real row gradients
    e.to(torch.bfloat16)
    e.shard_rows(rank, world, device=dev, dtype=torch.bfloat16, group=_group(world),
                 row_capacity=ROWS_PER_GPU * SEQ * world)
    rows = RowTables([("layers.0.micro_engram.", e)], lr=5e-3, lazy=True, rowwise=True, sparse_grads=True)
    return e, rows


def run_ours(args):
    import torch

    from micro_engram.optim import LazyAdamW

    rank, world, dev = _setup_dist()
    e, rows = _engram_ours(dev, rank, world)
    dense = [p for p in e.parameters() if p.requires_grad]
    opt = LazyAdamW([{"params": dense, "lazy": False}], lr=1e-3, stochastic_rounding=True)
    ids, pos, hidden = _inputs(rank, dev)
    h = hidden.reshape(-1, DMODEL)
    ar = None
    if world > 1:
        from micro_engram_fork_b200.parallel.allreduce import P2PAllReduce

        ar = P2PAllReduce(sum(p.numel() for p in dense), dev)

    def step():
        x = h.detach().requires_grad_()
        out = e(x.view(ROWS_PER_GPU, SEQ, DMODEL), ids, pos)
        out.backward(torch.ones_like(out))
        if ar is not None:
            mean = ar([p.grad for p in dense])
            off = 0
            for p in dense:
                p.grad.copy_(mean[off:off + p.numel()].view_as(p))
                off += p.numel()
        rows.clip(2.0)
        opt.step()
        rows.step(5e-3)
        opt.zero_grad(set_to_none=True)

    ms = _time(step, args.steps, args.warmup, world)
    store = e.__dict__.get("row_store")
    if store is not None:
        store.check_status()
    if args.kernel_table:
        _kernel_table(step, args.kernel_table, rank)
    return ms, rank, world


def _kernel_table(step, path, rank):
    """Device time per kernel of one extra (untimed) step, rank 0's view, for finding the limiter."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step()
        torch.cuda.synchronize()
    if rank == 0:
        with open(path, "w") as f:
            f.write(prof.key_averages().table(sort_by="device_time_total", row_limit=40, max_name_column_width=90))


def run_reference(args):
    import torch

    here = os.path.dirname(os.path.abspath(__file__))
    ref_root = os.path.join(here, "..", "..", "baseline", "_ref")
    if not os.path.isfile(os.path.join(ref_root, "micro_engram", "rows.py")):
        print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref is not installed"}))
        return None
    for k in [k for k in sys.modules if k == "micro_engram" or k.startswith("micro_engram.")]:
        del sys.modules[k]
    sys.path.insert(0, os.path.abspath(ref_root))
    from micro_engram.module import MicroEngram
    from micro_engram.rows import RowTables

    sys.path.pop(0)
    rank, world, dev = _setup_dist()
    e = MicroEngram(model_dim=DMODEL, engram_dim=EDIM, num_heads=HEADS, orders=(2, 3, 4), table_sizes=TABLES,
                    vocab_size=VOCAB, gate="scalar_sqrt", build_tables=False, seed=0).to(dev)
    with torch.no_grad():
        e.value.weight.normal_(0, 0.02)
    e.to(torch.bfloat16)
    e.shard_rows(rank, world, device=dev, dtype=torch.bfloat16)
    rows = RowTables([("layers.0.micro_engram.", e)], lr=5e-3, lazy=True, rowwise=True, sparse_grads=True)
    dense = [p for p in e.parameters() if p.requires_grad]
    opt = torch.optim.AdamW(dense, lr=1e-3)
    ids, pos, hidden = _inputs(rank, dev)
    h = hidden.reshape(-1, DMODEL)
    import torch.distributed as dist

    def step():
        x = h.detach().requires_grad_()
        out = e(x.view(ROWS_PER_GPU, SEQ, DMODEL), ids, pos)
        out.backward(torch.ones_like(out))
        if world > 1:
            flat = torch.cat([p.grad.reshape(-1).float() for p in dense])
            dist.all_reduce(flat)
            flat /= world
            off = 0
            for p in dense:
                p.grad.copy_(flat[off:off + p.numel()].view_as(p))
                off += p.numel()
        rows.clip(2.0)
        opt.step()
        rows.step(5e-3)
        opt.zero_grad(set_to_none=True)

    ms = _time(step, args.steps, args.warmup, world)
    return ms, rank, world


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--kernel-table", default="", help="write one profiled step's per-kernel device times here")
    args = ap.parse_args()
    got = run_reference(args) if args.impl == "reference" else run_ours(args)
    if got is None:
        return
    ms, rank, world = got
    lookups = ROWS_PER_GPU * SEQ * len(TABLES) * HEADS
    remote = (world - 1) / world
    # bytes that must cross NVLink per GPU: every remote lookup's bf16 row in (written by its owner)
    # and its bf16 gradient back (plus an 8-byte header per entry)
    nvlink_bytes = lookups * remote * (EDIM * 2 + EDIM * 2 + 8)
    # tensor-core work: key and value projections forward, their input gradient and weight gradient
    tokens, mem = ROWS_PER_GPU * SEQ, len(TABLES) * HEADS * EDIM
    flops = 3 * 2 * (2 * tokens * mem * DMODEL)
    from micro_engram_fork_b200.utils.kernel_bench import peaks

    peak = peaks()
    link_ms = nvlink_bytes / (NVLINK_GBS * 1e9) * 1e3
    tc_ms = flops / (peak["bf16_tflops"] * 1e12) * 1e3
    roof_ms = max(link_ms, tc_ms)
    if rank == 0:
        print(json.dumps({
            "impl": args.impl, "metric": "engram module fwd+bwd+update step (config 2)", "ms_per_step": round(ms, 3),
            "tokens_per_s": round(ROWS_PER_GPU * SEQ * world / (ms / 1e3), 1), "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "lookups_per_gpu": lookups,
            "nvlink_bytes_per_gpu": int(nvlink_bytes), "nvlink_roofline_ms": round(link_ms, 3),
            "gemm_flops_per_gpu": flops, "tensor_roofline_ms": round(tc_ms, 3),
            "frac_of_roofline": round(roof_ms / ms, 4),
            "roofline": f"max(GEMM FLOPs at {peak['bf16_tflops']} TFLOP/s ({peak['source']}), NVLink bytes at "
                        f"{NVLINK_GBS} GB/s per direction)",
            "config": {"tables": TABLES, "heads": HEADS, "dim": EDIM, "tokens_per_gpu": ROWS_PER_GPU * SEQ,
                       "d_model": DMODEL, "data": "synthetic Zipf(1.1) ids, docs 256-4096, hidden N(0,1) bf16"}}),
              flush=True)
    import torch.distributed as dist

    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", ".."))
    main()
