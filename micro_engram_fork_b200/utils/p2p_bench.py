"""Dense-gradient all-reduce on N GPUs: the fused peer-memory kernel (P2PAllReduce) against
NCCL all_reduce + divide, on the reference's size (2 x 1536 x 5376 + 2 x 5376 fp32 = 66 MB
per engram). Device time with CUDA events after warm-up, max over ranks; roofline = bytes this
rank reads from its peers over NVLink ((world - 1) x 66 MB) at the measured 770 GB/s per
direction.

  torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m micro_engram_fork_b200.utils.p2p_bench [--iters 20]
"""
import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

LINK_GBS = 770.0


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--n", type=int, default=2 * 1536 * 5376 + 2 * 5376)
    args = ap.parse_args(argv)
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    from ..parallel.allreduce import P2PAllReduce

    ar = P2PAllReduce(args.n, dev)
    x = torch.randn(args.n, device=dev)

    def nccl():
        y = x.clone()
        dist.all_reduce(y)
        y /= world

    def p2p():
        ar([x])

    res = {}
    for name, fn in (("p2p kernel", p2p), ("nccl all_reduce", nccl)):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ms = torch.tensor([e0.elapsed_time(e1) / args.iters], device=dev, dtype=torch.float64)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        ms = float(ms)
        nvlink_bytes = (world - 1) * args.n * 4
        roof_ms = nvlink_bytes / (LINK_GBS * 1e9) * 1e3
        res[name] = {"ms": round(ms, 4), "roofline_ms": round(roof_ms, 4), "frac_of_roofline": round(roof_ms / ms, 3)}
    ar.check_status()
    got = ar([x]).clone()
    ok = torch.allclose(got, sum_over_ranks(x, world), rtol=1e-5, atol=1e-5)
    if rank == 0:
        print(json.dumps({"world": world, "n": args.n, "mbytes": round(args.n * 4 / 1e6, 1), "results": res,
                          "matches_nccl": bool(ok)}))
    ar.close()
    dist.destroy_process_group()


def sum_over_ranks(x, world):
    y = x.clone()
    dist.all_reduce(y)
    return y / world


if __name__ == "__main__":
    main()
