"""Row-parallel linear + all-reduce on N GPUs (tensor-parallel serving's o_proj and down_proj of
the 31B-class decoder): the fused peer-memory op (parallel/tp_linear.py: the tcgen05 GEMM's
epilogue reduce-scatters its fp32 partial over NVLink, then a slot sum and an all-gather)
against what vLLM runs, a library GEMM (F.linear) and then an all-reduce (NCCL here), and
against the library GEMM alone (no communication at all, the floor).

  torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m micro_engram_fork_b200.utils.tp_bench [--iters 50]

Shapes: N = 5376 output features; K = 16384 (o_proj of a global-attention layer: 32 heads x
512) and 21504 (down_proj), each split over the ranks; M = 64 (a decode step of 64 requests),
512 and 8192 (prefill chunks). Inputs larger than L2: four copies of each weight are cycled.
Device time with CUDA events after warm-up, max over ranks. Roofline of the fused op: the
slowest of the GEMM at the measured bf16 peak, this rank's weight slice read at the measured
HBM bandwidth, and the bytes each rank receives over NVLink ((world - 1) / world x M x N x
(4 bytes of fp32 partial + 2 bytes of bf16 result)) at the measured 770 GB/s per direction.
"""
import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist
import torch.nn.functional as F

LINK_GBS = 770.0


def _peaks():
    path = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, 6650.0, "fallback"


def _time(fn, iters, dev):
    for _ in range(3):
        fn(0)
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(iters):
        fn(i)
    e1.record()
    torch.cuda.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1) / iters], device=dev, dtype=torch.float64)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--m", type=int, nargs="+", default=[64, 512, 8192])
    args = ap.parse_args(argv)
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    from ..parallel.tp_linear import TPRowLinear

    peak_tf, hbm_gbs, src = _peaks()
    N = 5376
    lin = TPRowLinear(max(args.m), N, dev)
    rows = []
    g = torch.Generator(device=dev).manual_seed(rank)
    for name, K in (("o_proj", 16384), ("down_proj", 21504)):
        k = K // world
        ws = [(torch.randn(N, k, device=dev, generator=g) * k ** -0.5).to(torch.bfloat16) for _ in range(4)]
        for M in args.m:
            x = torch.randn(M, k, device=dev, generator=g).to(torch.bfloat16)

            def fused(i):
                return lin(x, ws[i % 4])

            def library(i):
                y = F.linear(x, ws[i % 4])
                dist.all_reduce(y)
                return y

            def gemm_only(i):
                return F.linear(x, ws[i % 4])

            res = {n: _time(f, args.iters, dev) for n, f in (("fused", fused), ("gemm+nccl", library),
                                                              ("gemm only", gemm_only))}
            flops = 2.0 * M * N * k
            roof = max(flops / (peak_tf * 1e12), N * k * 2 / (hbm_gbs * 1e9),
                       (world - 1) / world * M * N * 6 / (LINK_GBS * 1e9)) * 1e3
            rows.append({"linear": name, "M": M, "K_per_rank": k,
                         **{f"{n}_ms": round(v, 4) for n, v in res.items()},
                         "fused_speedup_vs_gemm+nccl": round(res["gemm+nccl"] / res["fused"], 3),
                         "roofline_ms": round(roof, 4), "fused_frac_of_roofline": round(roof / res["fused"], 3)})
    torch.cuda.synchronize()
    lin.check_status()
    dist.barrier()
    lin.close()
    if rank == 0:
        print(json.dumps({"bench": "tp row-parallel linear + all-reduce", "world": world, "N": N,
                          "peaks": {"bf16_tflops": peak_tf, "hbm_gbs": hbm_gbs, "link_gbs": LINK_GBS,
                                    "source": src}, "rows": rows}), flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
