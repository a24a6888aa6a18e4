"""Projections on the persistent tcgen05 GEMM (csrc/gemm.cu), with plain PyTorch references.

The frozen base never needs weight gradients, so every projection is one of four products:

  linear(x, W)              x . W^T            forward of y = x W^T         (W [N, K], K-major)
  linear_t(g, W)            g . W              its input gradient dX        (W read N-major)
  geglu_linear(h, Wgu)      GeGLU(h . Wgu^T)   gate|up GEMM with the GeGLU in its epilogue
  dgeglu_linear(g, Wd, gu)  GeGLU'(gu) * (g . Wd)   down-projection dX with the GeGLU backward
                                                    in its epilogue
  projection(x, W)          x . W^T as an autograd op whose dX and dW (= dY^T . X, fp32
                            accumulation) also run on the tcgen05 GEMM: trained projections
                            such as the engram's key/value weights

CUDA tensors always run the native kernels (no silent fallback); CPU tensors run the reference.
The reference's base projections are HF ``nn.Linear`` layers over cuBLAS
(micro_engram/train/model.py:71-98 in Ready-Art/micro_engram_fork) with Liger's GeGLU
(micro_engram/train/vendor/gemma4_fused_attn.py:57-168).
"""
import torch
import torch.nn.functional as F

from .. import native
from ..parallel.sharded_base import carry_into_next_gemm
from . import use_native
from .norm import geglu_bwd_ref, geglu_ref


def _rows(x):
    return x.reshape(-1, x.shape[-1])


def _aligned(*ts):
    for t in ts:
        if t.dtype != torch.bfloat16 or t.stride(-1) != 1 or t.data_ptr() % 16 or (t.dim() > 1 and t.stride(0) % 8):
            return False
    return True


def linear(x, W, out=None):
    """x [..., K] . W[N, K]^T -> [..., N]."""
    if use_native(x, W):
        x2 = _rows(x).contiguous()
        if not _aligned(x2, W) or W.shape[0] % 8 or W.shape[1] % 8:
            raise RuntimeError("linear: the tcgen05 GEMM needs bf16, 16-byte aligned rows, N and K multiples of 8")
        carry_into_next_gemm(W)
        y = native().gemm(x2, W, True, out)
        return y.view(*x.shape[:-1], W.shape[0])
    return F.linear(x, W)


def linear_t(g, W, out=None):
    """g [..., N] . W[N, K] -> [..., K] (the input gradient of linear)."""
    if use_native(g, W):
        g2 = _rows(g).contiguous()
        if not _aligned(g2, W) or W.shape[0] % 8 or W.shape[1] % 8:
            raise RuntimeError("linear_t: the tcgen05 GEMM needs bf16, 16-byte aligned rows, N and K multiples of 8")
        carry_into_next_gemm(W)
        y = native().gemm(g2, W, False, out)
        return y.view(*g.shape[:-1], W.shape[1])
    return torch.matmul(g, W)


def geglu_linear(h, Wgu, save_gu=True):
    """(m, gu): gu = h . Wgu^T with Wgu = [gate; up] [2F, K], m = GeGLU(gu) [.., F]. gu is only
    materialised when save_gu (for the backward); m is bf16(bf16(gelu_tanh(gate)) * up)."""
    if use_native(h, Wgu):
        h2 = _rows(h).contiguous()
        carry_into_next_gemm(Wgu)
        m, gu = native().gemm_geglu(h2, Wgu, save_gu)
        lead = h.shape[:-1]
        return m.view(*lead, -1), (gu.view(*lead, -1) if save_gu else None)
    gu = F.linear(h, Wgu)
    return geglu_ref(gu), (gu if save_gu else None)


def dgeglu_linear(g, Wdown, gu):
    """d_gu = GeGLU backward of dm = g . Wdown (Wdown [d, F], the down projection's weight)."""
    if use_native(g, Wdown, gu):
        g2 = _rows(g).contiguous()
        carry_into_next_gemm(Wdown)
        return native().gemm_dgeglu(g2, Wdown, _rows(gu)).view(*g.shape[:-1], -1)
    return geglu_bwd_ref(torch.matmul(g, Wdown), gu)


class _Projection(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, W):
        ctx.save_for_backward(x, W)
        return linear(x, W)

    @staticmethod
    def backward(ctx, g):
        x, W = ctx.saved_tensors
        g2 = _rows(g).contiguous()
        dx = linear_t(g2, W).view(x.shape) if ctx.needs_input_grad[0] else None
        dW = None
        if ctx.needs_input_grad[1]:
            dW = native().gemm_tn_f32(g2, _rows(x).contiguous()).to(W.dtype)
        return dx, dW


def projection(x, W):
    """y = x . W^T with gradients for both x and W (W [N, K])."""
    if use_native(x, W):
        return _Projection.apply(x, W)
    return F.linear(x, W)
