"""Kernel microbenchmarks of the sm_100a kernels on the 31B-class shapes, timed with CUDA
events (warm-up, synchronize on both sides) and reported against the measured roofline
(MEASURED_PEAKS.json: cuBLAS bf16 burst TFLOP/s and copy bandwidth; the recipe's fallback
figures otherwise). Also the workload that the committed ncu summaries in profiles/ capture.

  python -m micro_engram_fork_b200.utils.kernel_bench [--case all|gemm|attn_fwd|attn_bwd|gate|ce|qkv|geglu|rows|
                                                       norms|ce_bwd|nf4|ce_gemm|tp] [--iters N] [--small]
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


def case_gate(C, dev, it, pk, small=False):
    """Fused scalar_sqrt gate at the microbenchmark size: 65536 tokens x d 5376 (16384 with
    --small, the size an ncu capture replays)."""
    N, d = (16384 if small else 65536), 5376
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


def case_ce_gemm(C, dev, it, pk):
    """The loss's logits GEMM of one 2048-token chunk against 262144 tied-head rows (d 5376) with the
    softcapped-CE epilogue (per-tile partial sums and the target logit; logits kept for the
    backward), against the plain GEMM of the same shape."""
    H = torch.randn(2048, 5376, device=dev).to(torch.bfloat16)
    E = (torch.randn(262144, 5376, device=dev) * 0.02).to(torch.bfloat16)
    lab = torch.randint(0, 262144, (2048,), device=dev)
    flops = 2 * 2048 * 262144 * 5376
    r = {}
    for name, fn in (("gemm_ce (softcap 30, logits kept)", lambda: C.gemm_ce(H, E, lab, 0, 30.0, True, 262144)),
                     ("gemm_ce (softcap 30, no logits)", lambda: C.gemm_ce(H, E, lab, 0, 30.0, False, 262144)),
                     ("plain gemm", lambda: C.gemm(H, E, True, None))):
        ms = _time(fn, it)
        r[name] = {"ms": round(ms, 4), "tflops": round(flops / ms / 1e9, 1),
                   "frac_of_peak": round(flops / ms / 1e9 / pk["bf16_tflops"], 3)}
    return r


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


def _hbm(name, nbytes, ms, pk):
    return {name: {"ms": round(ms, 4), "gbs": round(nbytes / ms / 1e6, 1),
                   "frac_of_hbm": round(nbytes / ms / 1e6 / pk["hbm_gbs"], 3)}}


def case_rows(C, dev, it, pk, small=False):
    """The engram row path of one GPU at the module benchmark's size (65536 tokens, 24 tables of
    {1.57M, 4.19M, 4.19M} rows x dim 64 bf16, Zipf(1.1) ids): hash, gather, row-gradient push into
    the compact accumulator, touched-row Adam. Bytes count what each kernel must move: the ids
    and rows it reads, the rows it writes (scatter: fp32 row gradients added; Adam: per touched
    row, the bf16 row and moment read and written, the fp32 accumulator read). --small divides the
    table rows by 8 (still above L2) for ncu captures."""
    import numpy as np

    from micro_engram.module import MicroEngram

    from ..parallel.row_store import RowStore

    tables, N, dim = {2: 1572864, 3: 4194304, 4: 4194304}, 65536, 64
    if small:
        tables = {k: v // 8 for k, v in tables.items()}
    e = MicroEngram(model_dim=256, engram_dim=dim, num_heads=8, orders=(2, 3, 4), table_sizes=tables,
                    vocab_size=262144, gate="scalar_sqrt", build_tables=False, seed=0)
    rng = np.random.default_rng(0)
    p = np.arange(1, 262145, dtype=np.float64) ** -1.1
    ids = torch.from_numpy(np.searchsorted(np.cumsum(p / p.sum()), rng.random(N)).astype(np.int64)).to(dev)
    pos = torch.cat([torch.arange(n) for n in (2000, 3000, 1192, 2000)] * 8).to(dev)[None]
    canon, mults, orders, rows_t = e._consts(dev)
    nt = len(e.table_rows)
    r = {}
    ms = _time(lambda: C.engram_hash(ids[None], pos, canon, mults, orders, rows_t, 0), it)
    r.update(_hbm("hash", N * 16 + nt * N * 8, ms, pk))
    idx = C.engram_hash(ids[None], pos, canon, mults, orders, rows_t, 0).reshape(nt, N).contiguous()
    store = RowStore(e.table_rows, dim, torch.bfloat16, 0, 1, dev, capacity=N)
    for w in store.weights:
        w.normal_(0, 0.02)
    ms = _time(lambda: store.gather(idx, torch.bfloat16), it)
    r.update(_hbm("gather", nt * N * (8 + 2 * dim * 2), ms, pk))
    g = torch.randn(N, nt * dim, device=dev).to(torch.bfloat16)
    uniq = sum(int(torch.unique(idx[k]).numel()) for k in range(nt))
    m = [torch.zeros_like(w) for w in store.weights]
    v = [torch.zeros(w.shape[0], device=dev) for w in store.weights]

    def push_and_step():
        store.push_grads(g, idx, 1.0)
        for k in range(nt):
            C.engram_adam_touched(store.weights[k], m[k], v[k], store.acc[k], store.pos[k], store.list[k],
                                  store.count[k], None, 1e-3, 0.9, 0.999, 1e-8, 0.0, 0.1, 0.001, True, 0, 1, k)
        for c in store.count:
            c.zero_()

    def push_and_batched_step():
        store.push_grads(g, idx, 1.0)
        C.engram_adam_rows(store.weights, m, v, store.acc, store.pos, store.list, store.count, list(range(nt)),
                           [0.1] * nt, [0.001] * nt, [1] * nt, None, 1e-3, 0.9, 0.999, 1e-8, 0.0, True, 0)
        for c in store.count:
            c.zero_()

    moved = nt * N * (8 + dim * 2) + uniq * dim * (4 + 4 * 2 + 4)
    r.update(_hbm("scatter+adam (one launch per table)", moved, _time(push_and_step, it), pk))
    r.update(_hbm("scatter+adam_rows (all tables, one launch)", moved, _time(push_and_batched_step, it), pk))
    r["unique_rows"] = uniq
    r["lookups"] = nt * N
    return r


def case_norms(C, dev, it, pk):
    """The decoder's row norms on one 8192-token step at d 5376: RMSNorm forward/backward and the
    fused post-norm + residual add (+ the next layer's input norm) forward/backward."""
    T, d = 8192, 5376
    x = torch.randn(T, d, device=dev).to(torch.bfloat16)
    a = torch.randn_like(x)
    w = torch.rand(d, device=dev) + 0.5
    ls = torch.rand(1, device=dev) + 0.5
    y, rstd = C.rmsnorm_fwd(x, w, 1e-6)
    r = {}
    ms = _time(lambda: C.rmsnorm_fwd(x, w, 1e-6), it)
    r.update(_hbm("rmsnorm fwd", 2 * T * d * 2, ms, pk))
    ms = _time(lambda: C.rmsnorm_bwd(y, x, w, rstd, None), it)
    r.update(_hbm("rmsnorm bwd", 3 * T * d * 2, ms, pk))
    outs = C.post_norm_add(x, a, w, ls, w, 1e-6)
    ms = _time(lambda: C.post_norm_add(x, a, w, ls, w, 1e-6), it)
    r.update(_hbm("post_norm_add fwd", 4 * T * d * 2, ms, pk))
    xo, hn, ra, rx = outs[0], outs[1], outs[2], outs[3]
    ms = _time(lambda: C.post_norm_add_bwd(y, y, a, xo, w, ls, w, ra, rx), it)
    r.update(_hbm("post_norm_add bwd", 6 * T * d * 2, ms, pk))
    return r


def case_ce_bwd(C, dev, it, pk):
    """The in-place loss gradient of one 2048-token chunk against 262144 vocab rows (bf16 logits
    read and overwritten)."""
    z = torch.randn(2048, 262144, device=dev).to(torch.bfloat16)
    lab = torch.randint(0, 262144, (2048,), device=dev)
    lse = torch.full((2048,), 40.0, device=dev)
    wr = torch.ones(2048, device=dev)
    ms = _time(lambda: C.ce_bwd_inplace(z, lab, 0, 30.0, lse, wr), it)
    return _hbm("ce_bwd_inplace 2048x262144", 2 * z.numel() * 2, ms, pk)


def case_nf4(C, dev, it, pk):
    """NF4 dequantisation of one 31B-class MLP weight (gate|up, 43008 x 5376, block 64)."""
    w = (torch.randn(43008, 5376, device=dev) * 0.02).to(torch.bfloat16)
    codes, absmax = C.nf4_quantize(w)[:2]
    out = torch.empty_like(w)
    ms = _time(lambda: C.nf4_dequant(codes, absmax, out), it)
    return _hbm("nf4_dequant 43008x5376", codes.numel() * codes.element_size() + absmax.numel() * 4 + out.numel() * 2,
                ms, pk)


def case_tp(C, dev, it, pk):
    """The fused row-parallel linear's three kernels (scatter GEMM, slot sum, gather) for two
    ranks emulated on this GPU (every flag published beforehand, as in its GPU test), against
    the plain bf16 GEMM of one rank: the device time of the op without NVLink, and the host time
    of issuing it, to tell a launch-bound call from a GPU-bound one. o_proj at TP = 2."""
    import time

    world, N, K, flags = 2, 5376, 8192, 256
    r = {}
    for M in (64, 8192):
        rows = -(-M // world)
        slot, half = rows * N, (rows * N * 2 + 15) // 16 * 16
        xs = [torch.randn(M, K, device=dev).to(torch.bfloat16) for _ in range(world)]
        ws = [(torch.randn(N, K, device=dev) * K ** -0.5).to(torch.bfloat16) for _ in range(world)]
        rb = [torch.zeros(flags + 2 * world * slot * 4, dtype=torch.uint8, device=dev) for _ in range(world)]
        gb = [torch.zeros(flags + 2 * half, dtype=torch.uint8, device=dev) for _ in range(world)]
        for b in rb + gb:
            b[:flags].view(torch.int32)[:world] = 1 << 30  # every wait is already satisfied
        rbases = torch.tensor([b.data_ptr() for b in rb], dtype=torch.int64, device=dev)
        gbases = torch.tensor([b.data_ptr() for b in gb], dtype=torch.int64, device=dev)
        recv = torch.tensor([b.data_ptr() + flags for b in rb], dtype=torch.int64, device=dev)
        stages = [b[flags:flags + rows * N * 2].view(torch.bfloat16).view(rows, N) for b in gb]
        status = torch.zeros(2, dtype=torch.int32, device=dev)
        out = torch.empty(world * rows, N, dtype=torch.bfloat16, device=dev)

        def one_rank(rk=0):
            C.gemm_f32_scatter(xs[rk], ws[rk], recv, rows, rk, slot, True)
            C.p2p_sum_slots(rbases, rk, 2, flags, slot, stages[rk], 5.0, status)
            C.p2p_gather(gbases, rk, 2, flags, half, rows * N * 2 // 16, out, 5.0, status, True)

        ms = _time(one_rank, it)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(it):
            one_rank()
        host_us = (time.perf_counter() - t0) / it * 1e6
        torch.cuda.synchronize()
        gemm_ms = _time(lambda: C.gemm(xs[0], ws[0], True, None), it)
        flops = 2 * M * N * K
        r[f"M {M}"] = {"fused_ms": round(ms, 4), "host_us_per_call": round(host_us, 1),
                       "plain_gemm_ms": round(gemm_ms, 4), "fused_frac_of_peak": round(flops / ms / 1e9 / pk["bf16_tflops"], 3),
                       "status": status.tolist()}
    return r


CASES = {"gemm": case_gemm, "attn_fwd": case_attn_fwd, "attn_bwd": case_attn_bwd, "gate": case_gate, "ce": case_ce,
         "qkv": case_qkv, "geglu": case_geglu, "rows": case_rows, "norms": case_norms, "ce_bwd": case_ce_bwd,
         "nf4": case_nf4, "ce_gemm": case_ce_gemm, "tp": case_tp}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default="all", choices=["all"] + list(CASES))
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--gemm-shapes", default="", help="comma-separated subset of GEMM_SHAPES names")
    ap.add_argument("--small", action="store_true", help="smaller gate/rows problems (for ncu captures)")
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
            elif name in ("gate", "rows"):
                res[name] = fn(C, dev, args.iters, pk, small=args.small)
            else:
                res[name] = fn(C, dev, args.iters, pk)
    res["status"] = {"gemm": C.gemm_status(0).tolist(), "attn_tc": C.attn_tc_status(0).tolist()}
    print(json.dumps(res, indent=1))


if __name__ == "__main__":
    main()
