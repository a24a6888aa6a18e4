"""Kernel microbenchmarks of the sm_100a kernels on the 31B-class shapes, timed with CUDA
events (warm-up, synchronize on both sides) and reported against the measured roofline
(MEASURED_PEAKS.json: cuBLAS bf16 burst TFLOP/s and copy bandwidth; the recipe's fallback
figures otherwise). Also the workload that the committed ncu summaries in profiles/ capture.

  python -m micro_engram_fork_b200.utils.kernel_bench [--case all|gemm|attn_fwd|attn_bwd|gate|ce|qkv|geglu] [--iters N]
"""
import argparse
import json
import os

import torch

_FALLBACK = {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0}


def peaks():
    here = os.path.dirname(os.path.abspath(__file__))
    path = os.path.join(here, "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {"bf16_tflops": float(d["bf16_tflops"]), "hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {**_FALLBACK, "source": "fallback"}


def _time(fn, iters):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def _docs(T, dev, lens=(2000, 3000, 1192, 2000)):
    from ..ops.attention import doc_starts

    pos = torch.cat([torch.arange(n) for n in lens])[:T].to(dev)
    return doc_starts(pos)


GEMM_SHAPES = (
    # name, N, K, kind: "nt" = x . W^T (W [N, K]), "nn" = g . W (W [K, N]), "geglu" (N = F), "dgeglu" (N = F)
    ("qkv_sliding", 16384, 5376, "nt"), ("qkv_global", 18432, 5376, "nt"), ("o_sliding", 5376, 8192, "nt"),
    ("o_global", 5376, 16384, "nt"), ("gate_up_geglu", 21504, 5376, "geglu"), ("down", 5376, 21504, "nt"),
    ("d_down_dgeglu", 21504, 5376, "dgeglu"), ("d_gate_up", 5376, 43008, "nn"), ("d_o_sliding", 8192, 5376, "nn"),
    ("d_qkv_sliding", 5376, 16384, "nn"), ("lm_head_chunk", 262144, 5376, "nt_m2048"),
)


def case_gemm(C, dev, it, pk, M=8192, only=None):
    """The decoder's projections at 8192 tokens (and one 2048-token LM-head chunk): the
    tcgen05 GEMM (with its fused GeGLU / GeGLU-backward epilogues) against cuBLAS
    (torch.matmul, plus the separate GeGLU kernels where the epilogue is fused)."""
    out = {}
    for name, N, K, kind in GEMM_SHAPES:
        if only and name not in only:
            continue
        m = 2048 if kind == "nt_m2048" else M
        A = torch.randn(m, K, device=dev).to(torch.bfloat16)
        if kind in ("nt", "nt_m2048"):
            W = (torch.randn(N, K, device=dev) / K ** 0.5).to(torch.bfloat16)
            ours, lib = (lambda: C.gemm(A, W, True, None)), (lambda: A @ W.t())
            flops = 2 * m * N * K
        elif kind == "nn":
            W = (torch.randn(K, N, device=dev) / K ** 0.5).to(torch.bfloat16)
            ours, lib = (lambda: C.gemm(A, W, False, None)), (lambda: A @ W)
            flops = 2 * m * N * K
        elif kind == "geglu":
            W = (torch.randn(2 * N, K, device=dev) / K ** 0.5).to(torch.bfloat16)
            ours = lambda: C.gemm_geglu(A, W, True)
            lib = lambda: C.geglu_fwd(A @ W.t())
            flops = 2 * m * 2 * N * K
        else:  # dgeglu
            W = (torch.randn(K, N, device=dev) / K ** 0.5).to(torch.bfloat16)
            gu = torch.randn(m, 2 * N, device=dev).to(torch.bfloat16)
            ours = lambda: C.gemm_dgeglu(A, W, gu)
            lib = lambda: C.geglu_bwd(A @ W, gu)
            flops = 2 * m * N * K
        row = {"M": m, "N": N, "K": K, "kind": kind}
        for tag, fn in (("tcgen05", ours), ("cublas", lib)):
            ms = _time(fn, it)
            row[tag] = {"ms": round(ms, 4), "tflops": round(flops / ms / 1e9, 1),
                        "frac_of_peak": round(flops / ms / 1e9 / pk["bf16_tflops"], 3)}
        row["speedup_vs_cublas"] = round(row["cublas"]["ms"] / row["tcgen05"]["ms"], 3)
        out[name] = row
        del A, W
    return out


def _attn_inputs(dev, D, Hk, T=8192, Hq=32):
    q = torch.randn(T, Hq, D, device=dev).to(torch.bfloat16)
    k = torch.randn(T, Hk, D, device=dev).to(torch.bfloat16)
    v = torch.randn(T, Hk, D, device=dev).to(torch.bfloat16)
    return q, k, v


def _attn_flops(ds, W, D, Hq):
    T = ds.numel()
    t = torch.arange(T, device=ds.device)
    lo = ds.long()
    if W:
        lo = torch.maximum(lo, t - W + 1)
    return 4.0 * float((t - lo + 1).double().sum()) * D * Hq


def case_attn_fwd(C, dev, it, pk):
    out = {}
    ds = _docs(8192, dev)
    for (D, Hk, W) in ((256, 16, 1024), (512, 4, 0)):
        q, k, v = _attn_inputs(dev, D, Hk)
        fl = _attn_flops(ds, W, D, 32)
        for name, fn in (("tcgen05", lambda: C.attn_fwd_tc(q, k, v, ds, W, 1.0)),
                         ("mma.sync", lambda: C.attn_fwd(q, k, v, ds, W, 1.0))):
            ms = _time(fn, it)
            out[f"hd{D} {name}"] = {"ms": round(ms, 4), "useful_tflops": round(fl / ms / 1e9, 1),
                                    "frac_of_peak": round(fl / ms / 1e9 / pk["bf16_tflops"], 3)}
    return out


def case_attn_bwd(C, dev, it, pk):
    from ..ops.attention import TILE_BUDGET

    out = {}
    ds = _docs(8192, dev)
    for (D, Hk, W) in ((256, 16, 1024), (512, 4, 0)):
        q, k, v = _attn_inputs(dev, D, Hk)
        o, lse = C.attn_fwd_tc(q, k, v, ds, W, 1.0)
        do = torch.randn_like(o)
        fl = 2.5 * _attn_flops(ds, W, D, 32)
        runs = [("mma.sync", lambda: C.attn_bwd(do, q, k, v, o, lse, ds, W, 1.0)),
                ("tcgen05 P/dS tiles", lambda: C.attn_bwd_mat(do, q, k, v, o, lse, ds, W, 1.0, TILE_BUDGET))]
        if D <= 256:
            runs.append(("tcgen05 fused", lambda: C.attn_bwd_tc(do, q, k, v, o, lse, ds, W, 1.0)))
        for name, fn in runs:
            ms = _time(fn, it)
            out[f"hd{D} bwd {name}"] = {"ms": round(ms, 4), "useful_tflops": round(fl / ms / 1e9, 1),
                                        "frac_of_peak": round(fl / ms / 1e9 / pk["bf16_tflops"], 3)}
    return out


def case_gate(C, dev, it, pk):
    """Fused scalar_sqrt gate at the microbenchmark size: 65536 tokens x d 5376."""
    N, d = 65536, 5376
    h = torch.randn(N, d, device=dev).to(torch.bfloat16)
    k = torch.randn_like(h)
    v = torch.randn_like(h) * 0.1
    s = torch.ones(d, device=dev)
    fwd_bytes = 4 * N * d * 2           # read h, k, v; write out
    bwd_bytes = 7 * N * d * 2           # read g, h, k, v; write dh, dk, dv
    out, st = C.engram_gate_fwd(h, k, v, s, s, None, True, None)
    r = {}
    ms = _time(lambda: C.engram_gate_fwd(h, k, v, s, s, None, True, None), it)
    r["gate fwd"] = {"ms": round(ms, 4), "gbs": round(fwd_bytes / ms / 1e6, 1),
                     "frac_of_hbm": round(fwd_bytes / ms / 1e6 / pk["hbm_gbs"], 3)}
    ms = _time(lambda: C.engram_gate_bwd(out, h, k, v, s, s, None, st, True), it)
    r["gate bwd"] = {"ms": round(ms, 4), "gbs": round(bwd_bytes / ms / 1e6, 1),
                     "frac_of_hbm": round(bwd_bytes / ms / 1e6 / pk["hbm_gbs"], 3)}
    return r


def case_ce(C, dev, it, pk):
    """One loss chunk: 256 tokens x 262144 vocab logits (bf16) -> softcapped LSE partials."""
    z = torch.randn(2048, 262144, device=dev).to(torch.bfloat16)
    lab = torch.randint(0, 262144, (2048,), device=dev)
    nbytes = z.numel() * 2
    ms = _time(lambda: C.ce_fwd(z, lab, 0, 30.0), it)
    return {"ce_fwd 2048x262144": {"ms": round(ms, 4), "gbs": round(nbytes / ms / 1e6, 1),
                                   "frac_of_hbm": round(nbytes / ms / 1e6 / pk["hbm_gbs"], 3)}}


def case_qkv(C, dev, it, pk):
    """q/k/v RMSNorm + RoPE, forward and backward, on one packed 8192-token step: a sliding layer
    (32 q heads, 16 k + 16 v heads of 256) and a global one (32 q heads of 512, 4 k heads, v = k)."""
    from ..models.gemma import GemmaConfig

    cfg, T = GemmaConfig(), 8192
    pos = torch.cat([torch.arange(n) for n in (2000, 3000, 1192, 2000)]).to(dev)
    r = {}
    for kind, D, Hk, shared in (("sliding", 256, 16, False), ("global", 512, 4, True)):
        Hq = 32
        HI, H = Hq + (1 if shared else 2) * Hk, Hq + 2 * Hk
        inv = cfg.inv_freq(f"{kind}_attention" if kind == "sliding" else "full_attention", D).to(dev)
        qkv = torch.randn(T, HI * D, device=dev).to(torch.bfloat16)
        w = torch.rand(D, device=dev) + 0.5
        q, k, v, rs = C.qkv_norm_rope(qkv, w, w, inv, pos, Hq, Hk, D, shared, 1e-6)
        fwd_bytes = T * HI * D * 2 + T * H * D * 2 + T * H * 4
        bwd_bytes = T * H * D * 2 + 2 * T * HI * D * 2 + T * H * 4
        ms = _time(lambda: C.qkv_norm_rope(qkv, w, w, inv, pos, Hq, Hk, D, shared, 1e-6), it)
        r[f"{kind} D{D} fwd"] = {"ms": round(ms, 4), "gbs": round(fwd_bytes / ms / 1e6, 1),
                                 "frac_of_hbm": round(fwd_bytes / ms / 1e6 / pk["hbm_gbs"], 3)}
        ms = _time(lambda: C.qkv_norm_rope_bwd(q, k, v, qkv, w, w, inv, pos, rs, Hq, Hk, D, shared), it)
        r[f"{kind} D{D} bwd"] = {"ms": round(ms, 4), "gbs": round(bwd_bytes / ms / 1e6, 1),
                                 "frac_of_hbm": round(bwd_bytes / ms / 1e6 / pk["hbm_gbs"], 3)}
    return r


def case_geglu(C, dev, it, pk):
    """GeGLU forward and backward on one 8192-token step of the 31B-class MLP (F = 21504)."""
    N, F = 8192, 21504
    gu = torch.randn(N, 2 * F, device=dev).to(torch.bfloat16)
    dm = torch.randn(N, F, device=dev).to(torch.bfloat16)
    fwd_bytes = N * 2 * F * 2 + N * F * 2
    bwd_bytes = N * 2 * F * 2 + N * F * 2 + N * 2 * F * 2
    r = {}
    ms = _time(lambda: C.geglu_fwd(gu), it)
    r["geglu fwd"] = {"ms": round(ms, 4), "gbs": round(fwd_bytes / ms / 1e6, 1),
                      "frac_of_hbm": round(fwd_bytes / ms / 1e6 / pk["hbm_gbs"], 3)}
    ms = _time(lambda: C.geglu_bwd(dm, gu), it)
    r["geglu bwd"] = {"ms": round(ms, 4), "gbs": round(bwd_bytes / ms / 1e6, 1),
                      "frac_of_hbm": round(bwd_bytes / ms / 1e6 / pk["hbm_gbs"], 3)}
    return r


CASES = {"gemm": case_gemm, "attn_fwd": case_attn_fwd, "attn_bwd": case_attn_bwd, "gate": case_gate, "ce": case_ce,
         "qkv": case_qkv, "geglu": case_geglu}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default="all", choices=["all"] + list(CASES))
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--gemm-shapes", default="", help="comma-separated subset of GEMM_SHAPES names")
    args = ap.parse_args(argv)
    from .. import native

    C = native()
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    pk = peaks()
    res = {"peaks": pk}
    for name, fn in CASES.items():
        if args.case in ("all", name):
            if name == "gemm" and args.gemm_shapes:
                res[name] = fn(C, dev, args.iters, pk, only=set(args.gemm_shapes.split(",")))
            else:
                res[name] = fn(C, dev, args.iters, pk)
    res["status"] = {"gemm": C.gemm_status(0).tolist(), "attn_tc": C.attn_tc_status(0).tolist()}
    print(json.dumps(res, indent=1))


if __name__ == "__main__":
    main()
