"""Packed-varlen causal attention (optionally sliding-window) for the Gemma-4 layers.

Layout: token-major q [T, Hq, D], k/v [T, Hk, D] (GQA: Hq % Hk == 0), straight from the
fused projection + norm/RoPE kernel, no transposes. Documents come from position_ids:
a document starts where pos[t] - pos[t-1] != 1 (transformers' packed-sequence rule), so
padding that continues the last document's positions stays in it. Token t attends to
s in [max(doc_start(t), t - window + 1), t]. Softmax scale is 1.0 (Gemma 4 normalises q
and k with RMSNorm instead).

The sm_100a kernels (csrc/attention.cu) do forward and backward on this layout with the
document bounds computed per tile from `doc_start`; the reference below builds the dense
mask and is used on CPU and as the oracle.
"""
import os

import torch

from .. import native


def doc_starts(pos):
    """[T] int32 first index of each token's document, from flat position ids [T]."""
    pos = pos.reshape(-1)
    T = pos.numel()
    idx = torch.arange(T, device=pos.device)
    new = torch.ones(T, dtype=torch.bool, device=pos.device)
    if T > 1:
        new[1:] = (pos[1:] - pos[:-1]) != 1
    starts = torch.where(new, idx, torch.zeros_like(idx))
    return torch.cummax(starts, dim=0).values.to(torch.int32)


def attention_ref(q, k, v, doc_start, window=None, scale=1.0):
    """Dense-mask reference: returns (o [T, Hq, D] in q's dtype, lse [Hq, T] fp32)."""
    T, Hq, D = q.shape
    Hk = k.shape[1]
    rep = Hq // Hk
    qf = q.float().transpose(0, 1)                       # [Hq, T, D]
    kf = k.float().transpose(0, 1).repeat_interleave(rep, 0)
    vf = v.float().transpose(0, 1).repeat_interleave(rep, 0)
    s = torch.matmul(qf, kf.transpose(1, 2)) * scale     # [Hq, T, T]
    t = torch.arange(T, device=q.device)
    ds = doc_start.long()
    allowed = (t[None, :] <= t[:, None]) & (t[None, :] >= ds[:, None])
    if window:
        allowed &= t[None, :] > (t[:, None] - window)
    s = s.masked_fill(~allowed[None], float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    p = torch.exp(s - lse[..., None])
    o = torch.matmul(p, vf).transpose(0, 1).to(q.dtype)
    return o, lse


def attention_torch(q, k, v, doc_start, window=None, scale=1.0):
    """Autograd-friendly reference (CPU model path): o [T, Hq, D]."""
    T, Hq, D = q.shape
    Hk = k.shape[1]
    rep = Hq // Hk
    qt = q.transpose(0, 1)
    kt = k.transpose(0, 1).repeat_interleave(rep, 0)
    vt = v.transpose(0, 1).repeat_interleave(rep, 0)
    t = torch.arange(T, device=q.device)
    ds = doc_start.long()
    allowed = (t[None, :] <= t[:, None]) & (t[None, :] >= ds[:, None])
    if window:
        allowed &= t[None, :] > (t[:, None] - window)
    s = torch.matmul(qt.float(), kt.float().transpose(1, 2)) * scale
    s = s.masked_fill(~allowed[None], float("-inf"))
    p = torch.softmax(s, dim=-1).to(q.dtype)
    return torch.matmul(p, vt).transpose(0, 1)


def attention_fwd(q, k, v, doc_start, window=None, scale=1.0):
    """(o [T, Hq, D] bf16, lse [Hq, T] fp32) on the tcgen05 kernel (csrc/attention_tc.cu):
    S and O accumulate in tensor memory, Q/K/V arrive by TMA."""
    return native().attn_fwd_tc(q, k, v, doc_start, int(window or 0), float(scale))


def attention_fwd_mma(q, k, v, doc_start, window=None, scale=1.0):
    """The first-generation warp-level mma.sync forward (kept for comparison and tests)."""
    return native().attn_fwd(q, k, v, doc_start, int(window or 0), float(scale))


# Byte budget of the P / dS tile buffers of the tiled backward (heads are processed in passes
# of whole GQA groups that fit; at least one group per pass).
TILE_BUDGET = int(float(os.environ.get("ME_ATTN_TILE_BUDGET_GIB", "2.5")) * 2**30)


def attention_bwd(do, q, k, v, o, lse, doc_start, window=None, scale=1.0):
    """(dq, dk, dv) on the sm_100a tcgen05/TMEM kernels. head_dim 256 and 512: the backward that
    writes the P and dS tiles to HBM once (bf16) and sums them into dQ, dK and dV as block-sparse
    GEMMs (5 tile products, no recomputation; 2.2x faster than the fused kernels at hd256 and the
    only tcgen05 form at hd512, whose 128 x 512 accumulator fills TMEM). Narrower heads: the fused
    backward (S and dP recomputed per output, nothing written but the gradients)."""
    if q.shape[-1] >= 256:
        return native().attn_bwd_mat(do, q, k, v, o, lse, doc_start, int(window or 0), float(scale), TILE_BUDGET)
    return native().attn_bwd_tc(do, q, k, v, o, lse, doc_start, int(window or 0), float(scale))


def attention_bwd_mma(do, q, k, v, o, lse, doc_start, window=None, scale=1.0):
    """The first-generation warp-level mma.sync backward (kept for comparison and tests)."""
    return native().attn_bwd(do, q, k, v, o, lse, doc_start, int(window or 0), float(scale))
