"""RMSNorm, the fused sub-block epilogue, q/k/v norm + partial RoPE, and GeGLU.

Native (sm_100a) forward/backward entry points used by the decoder's layer function, plus
plain PyTorch references with the same rounding points as HF's Gemma-4 modules
(transformers.models.gemma4.modeling_gemma4: Gemma4RMSNorm, apply_rotary_pos_emb,
Gemma4TextMLP), used on CPU and as the oracle in tests.
"""
import torch
import torch.nn.functional as F

from .. import native


# ------------------------------------------------------------------------- references
def rmsnorm_ref(x, w=None, eps=1e-6):
    xf = x.float()
    y = xf * torch.pow(xf.pow(2).mean(-1, keepdim=True) + eps, -0.5)
    if w is not None:
        y = y * w.float()
    return y.to(x.dtype)


def rope_ref(x, cos, sin):
    """HF's apply_rotary_pos_emb on [..., D] with cos/sin of the same dtype as x."""
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return (x * cos) + (rot * sin)


def rope_cos_sin(pos, inv_freq, dtype):
    """cos/sin [T, D] like Gemma4TextRotaryEmbedding: fp32 angles, cast to the compute dtype."""
    freqs = pos.float()[:, None] * inv_freq.float()[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def post_norm_add_ref(r, a, w_post, ls=None, w_next=None, eps=1e-6):
    x = r + rmsnorm_ref(a, w_post, eps)
    if ls is not None:
        x = x * ls.to(x.dtype)
    h = rmsnorm_ref(x, w_next, eps) if w_next is not None else None
    return x, h


def geglu_ref(gu):
    g, u = gu.chunk(2, dim=-1)
    return F.gelu(g, approximate="tanh") * u


def geglu_bwd_ref(dm, gu):
    """d gu = [dm * u * gelu'(g) | dm * gelu(g)] (tanh GELU), computed in fp32."""
    g, u = gu.float().chunk(2, dim=-1)
    dm = dm.float()
    k0, k1 = 0.7978845608028654, 0.044715
    t = torch.tanh(k0 * (g + k1 * g * g * g))
    gelu = 0.5 * g * (1.0 + t)
    dgelu = 0.5 * (1.0 + t) + 0.5 * g * (1.0 - t * t) * k0 * (1.0 + 3.0 * k1 * g * g)
    return torch.cat((dm * u * dgelu, dm * gelu), dim=-1).to(gu.dtype)


# ------------------------------------------------------------------------- native entry points
def rmsnorm(x, w=None, eps=1e-6):
    """(y, rstd) on CUDA."""
    return native().rmsnorm_fwd(x, w, eps)


def rmsnorm_bwd(dy, x, w, rstd, dx_add=None):
    return native().rmsnorm_bwd(dy, x, w, rstd, dx_add)


def post_norm_add(r, a, w_post, ls=None, w_next=None, eps=1e-6):
    """(x, h, rstd_a, rstd_x): x = (r + rms(a)*w_post) * ls; h = rms(x) * w_next."""
    return native().post_norm_add(r, a, w_post, ls, w_next, eps)


def post_norm_add_bwd(dx, dh, a, x, w_post, ls, w_next, rstd_a, rstd_x):
    """(d residual, d branch)."""
    return native().post_norm_add_bwd(dx, dh, a, x, w_post, ls, w_next, rstd_a, rstd_x)


def qkv_norm_rope(qkv, q_w, k_w, inv_freq, pos, hq, hk, d, kv_shared=False, eps=1e-6):
    """(q [T,Hq,D], k [T,Hk,D], v [T,Hk,D], rstd) from the fused projection output
    [T, (Hq + 2 Hk) D], or [T, (Hq + Hk) D] when v is the raw k (attention_k_eq_v)."""
    return native().qkv_norm_rope(qkv, q_w, k_w, inv_freq, pos, hq, hk, d, kv_shared, eps)


def qkv_norm_rope_bwd(dq, dk, dv, qkv, q_w, k_w, inv_freq, pos, rstd, hq, hk, d, kv_shared=False):
    return native().qkv_norm_rope_bwd(dq, dk, dv, qkv, q_w, k_w, inv_freq, pos, rstd, hq, hk, d, kv_shared)


def geglu(gu):
    return native().geglu_fwd(gu)


def geglu_bwd(dm, gu):
    return native().geglu_bwd(dm, gu)
