"""Gemma-4-style text decoder (frozen base) for engram training, B200-first.

Architecture = HF transformers' Gemma4TextModel (modeling_gemma4.py): per layer
input_layernorm -> q/k/v proj -> q_norm/k_norm + RoPE, v_norm (no scale) -> attention
(scale 1.0; sliding-window layers with head_dim `head_dim`, global layers with
`global_head_dim`, `num_global_key_value_heads` and optionally v = k) -> o_proj ->
post_attention_layernorm + residual -> pre_feedforward_layernorm -> GeGLU MLP ->
post_feedforward_layernorm + residual -> * layer_scalar. Weight names match HF's, so
Gemma-4 safetensors load directly (`model.layers.N...` or `model.language_model.layers.N...`).

Execution:
  CUDA   one autograd Function per layer (`_LayerFn`) drives the sm_100a kernels: fused
         q/k/v projection (one GEMM against the concatenated weight), fused q/k/v norm +
         RoPE, packed-varlen attention, the post-norm + residual + next pre-norm epilogue,
         a fused gate|up GEMM + GeGLU, and a hand-written backward that only computes
         dX (the base is frozen: no weight gradients). Activation checkpointing saves just
         the layer input (which the trainer's offload hooks can move to pinned host memory)
         and recomputes the layer in the backward.
  CPU    the same math in plain PyTorch autograd (oracle, gloo tests).
The q/k/v and gate/up projections are stored fused; the HF-named Linear weights are views
into the fused buffers, so loading an HF state dict fills them in place.
"""
import json
import os
from dataclasses import dataclass, field

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..ops import use_native
from ..ops import norm as N
from ..ops.attention import attention_torch, doc_starts
from ..ops.linear import dgeglu_linear, geglu_linear, linear, linear_t


# ----------------------------------------------------------------------------- config
@dataclass
class GemmaConfig:
    vocab_size: int = 262_144
    hidden_size: int = 5376
    intermediate_size: int = 21504
    num_hidden_layers: int = 60
    num_attention_heads: int = 32
    num_key_value_heads: int = 16
    head_dim: int = 256
    global_head_dim: int = 512
    num_global_key_value_heads: int | None = 4
    attention_k_eq_v: bool = False
    sliding_window: int = 1024
    layer_types: list = None
    rope_parameters: dict = None
    rms_norm_eps: float = 1e-6
    final_logit_softcapping: float | None = 30.0
    pad_token_id: int | None = 0
    eos_token_id: int | None = 1
    bos_token_id: int | None = 2
    tie_word_embeddings: bool = True
    hidden_size_per_layer_input: int = 0
    num_kv_shared_layers: int = 0
    enable_moe_block: bool = False
    extra: dict = field(default_factory=dict)

    def __post_init__(self):
        if self.layer_types is None:
            self.layer_types = ["sliding_attention" if (i + 1) % 6 else "full_attention"
                                for i in range(self.num_hidden_layers)]
        if self.rope_parameters is None:
            self.rope_parameters = {
                "sliding_attention": {"rope_type": "default", "rope_theta": 10_000.0},
                "full_attention": {"rope_type": "proportional", "partial_rotary_factor": 0.25,
                                   "rope_theta": 1_000_000.0},
            }
        if self.hidden_size_per_layer_input:
            raise NotImplementedError("per-layer input embeddings (Gemma 4 E-series) are not supported")
        if self.enable_moe_block:
            raise NotImplementedError("MoE Gemma 4 variants are not supported")
        if self.num_kv_shared_layers:
            raise NotImplementedError("shared-KV layers are not supported in training")

    # HF-compatible fields used by the engram code
    @property
    def model_type(self):
        return "gemma4_text"

    @classmethod
    def from_dict(cls, d):
        d = dict(d)
        if "text_config" in d and isinstance(d["text_config"], dict):
            top = d
            d = dict(d["text_config"])
            d.setdefault("tie_word_embeddings", top.get("tie_word_embeddings", True))
        known = {f for f in cls.__dataclass_fields__ if f != "extra"}
        kw = {k: v for k, v in d.items() if k in known}
        eos = kw.get("eos_token_id")
        if isinstance(eos, list):
            kw["eos_token_id"] = eos[0] if eos else None
        kw["extra"] = {k: v for k, v in d.items() if k not in known}
        return cls(**kw)

    @classmethod
    def from_pretrained(cls, path):
        with open(os.path.join(path, "config.json")) as f:
            return cls.from_dict(json.load(f))

    def to_dict(self):
        d = {k: getattr(self, k) for k in self.__dataclass_fields__ if k != "extra"}
        return d

    def layer_is_sliding(self, i):
        return self.layer_types[i] == "sliding_attention"

    def attn_shape(self, i):
        """(head_dim, kv heads, v == k) of layer i, with HF's rule: global layers use
        global_head_dim, and num_global_key_value_heads only together with attention_k_eq_v."""
        if self.layer_is_sliding(i):
            return self.head_dim, self.num_key_value_heads, False
        kv_eq = bool(self.attention_k_eq_v)
        hd = self.global_head_dim or self.head_dim
        n_kv = self.num_global_key_value_heads if kv_eq else self.num_key_value_heads
        return hd, n_kv, kv_eq

    def inv_freq(self, layer_type, head_dim):
        """[head_dim/2] fp32 inverse frequencies (default and proportional RoPE)."""
        p = self.rope_parameters[layer_type]
        base = p["rope_theta"]
        if p.get("rope_type", "default") == "proportional":
            frac = p.get("partial_rotary_factor", 1.0)
            n_rot = int(frac * head_dim // 2)
            rot = 1.0 / (base ** (torch.arange(0, 2 * n_rot, 2, dtype=torch.int64, device="cpu").float() / head_dim))
            return torch.cat([rot, torch.zeros(head_dim // 2 - n_rot, device="cpu")])
        return 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.int64, device="cpu").float() / head_dim))


def tiny_config(**kw):
    """A small Gemma-4-style config (tests, smoke)."""
    base = dict(vocab_size=4096, hidden_size=256, intermediate_size=1024, num_hidden_layers=4,
                num_attention_heads=4, num_key_value_heads=2, head_dim=64, global_head_dim=128,
                num_global_key_value_heads=1, attention_k_eq_v=True, sliding_window=64,
                final_logit_softcapping=30.0,
                layer_types=["sliding_attention", "sliding_attention", "sliding_attention", "full_attention"])
    base.update(kw)
    return GemmaConfig(**base)


def config_31b():
    """The 31B-class config of the benchmark (60 layers, d 5376, FFN 21504, 32 q heads,
    sliding-1024 hd256 x16 KV interleaved 5:1 with global hd512 x4 KV, vocab 262144)."""
    return GemmaConfig(vocab_size=262_144, hidden_size=5376, intermediate_size=21504, num_hidden_layers=60,
                       num_attention_heads=32, num_key_value_heads=16, head_dim=256, global_head_dim=512,
                       num_global_key_value_heads=4, attention_k_eq_v=True, sliding_window=1024,
                       final_logit_softcapping=30.0)


# ----------------------------------------------------------------------------- modules
class _Norm(nn.Module):
    """RMSNorm weight, always kept in fp32 (the kernels apply it in fp32, as HF does)."""

    def __init__(self, dim):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim), requires_grad=False)

    def _apply(self, fn, *a, **kw):
        out = super()._apply(fn, *a, **kw)
        if self.weight.dtype != torch.float32:
            self.weight.data = self.weight.data.float()
        return out


class _Proj(nn.Module):
    """A bias-free linear whose weight is a view into a fused buffer."""

    def __init__(self, weight):
        super().__init__()
        self.weight = nn.Parameter(weight, requires_grad=False)

    def forward(self, x):
        return F.linear(x, self.weight)


class _Attn(nn.Module):
    def __init__(self, cfg, i, qkv, d):
        super().__init__()
        hd, n_kv, kv_eq = cfg.attn_shape(i)
        nq = cfg.num_attention_heads * hd
        nk = n_kv * hd
        self.q_proj = _Proj(qkv[:nq])
        self.k_proj = _Proj(qkv[nq:nq + nk])
        if not kv_eq:
            self.v_proj = _Proj(qkv[nq + nk:nq + 2 * nk])
        self.o_proj = _Proj(torch.empty(d, nq))
        self.q_norm = _Norm(hd)
        self.k_norm = _Norm(hd)


class _MLP(nn.Module):
    def __init__(self, gu, d, f):
        super().__init__()
        self.gate_proj = _Proj(gu[:f])
        self.up_proj = _Proj(gu[f:])
        self.down_proj = _Proj(torch.empty(d, f))


class GemmaLayer(nn.Module):
    def __init__(self, cfg, i):
        super().__init__()
        self.cfg, self.idx = cfg, i
        d, f = cfg.hidden_size, cfg.intermediate_size
        self.head_dim, self.n_kv, self.kv_eq = cfg.attn_shape(i)
        self.n_q = cfg.num_attention_heads
        self.sliding = cfg.layer_is_sliding(i)
        self.window = cfg.sliding_window if self.sliding else None
        rows = (self.n_q + (1 if self.kv_eq else 2) * self.n_kv) * self.head_dim
        self.register_buffer("qkv_weight", torch.empty(rows, d), persistent=False)
        self.register_buffer("gate_up_weight", torch.empty(2 * f, d), persistent=False)
        self.self_attn = _Attn(cfg, i, self.qkv_weight, d)
        self.mlp = _MLP(self.gate_up_weight, d, f)
        self.input_layernorm = _Norm(d)
        self.post_attention_layernorm = _Norm(d)
        self.pre_feedforward_layernorm = _Norm(d)
        self.post_feedforward_layernorm = _Norm(d)
        self.register_buffer("layer_scalar", torch.ones(1))
        self._inv_freq_cpu = cfg.inv_freq(cfg.layer_types[i], self.head_dim)  # fp32, never cast
        self._inv_freq_dev = {}
        self.gradient_checkpointing = False

    @property
    def inv_freq(self):
        dev = self.qkv_weight.device
        t = self._inv_freq_dev.get(str(dev))
        if t is None:
            t = self._inv_freq_cpu.to(dev)
            self._inv_freq_dev[str(dev)] = t
        return t

    def _apply(self, fn, *a, **kw):
        # keep the HF-named weights views of the fused buffers after .to()/.cuda()
        out = super()._apply(fn, *a, **kw)
        self._relink()
        return out

    def __setstate__(self, state):
        # copy.deepcopy / pickle rebuild the fused buffers and the HF-named weights as separate
        # tensors; make the names views of the buffers again
        super().__setstate__(state)
        self._relink()

    def _relink(self):
        nq = self.n_q * self.head_dim
        nk = self.n_kv * self.head_dim
        f = self.cfg.intermediate_size
        att = self.self_attn
        att.q_proj.weight.data = self.qkv_weight[:nq]
        att.k_proj.weight.data = self.qkv_weight[nq:nq + nk]
        if not self.kv_eq:
            att.v_proj.weight.data = self.qkv_weight[nq + nk:nq + 2 * nk]
        self.mlp.gate_proj.weight.data = self.gate_up_weight[:f]
        self.mlp.up_proj.weight.data = self.gate_up_weight[f:]

    # ---------------------------------------------------------------- forward
    def forward(self, x, pos, doc_start):
        """x [T, d] (one packed row), pos [T], doc_start [T] int32 -> [T, d]."""
        if use_native(x):
            if torch.is_grad_enabled() and x.requires_grad:
                ck = self.gradient_checkpointing
                mode = ck if ck in ("selective", "none", "full") else ("full" if ck else False)
                return _LayerFn.apply(x, pos, doc_start, self, mode)
            with torch.no_grad():
                return _layer_fwd(self, x, pos, doc_start)[0]
        if self.gradient_checkpointing and torch.is_grad_enabled() and x.requires_grad:
            from torch.utils.checkpoint import checkpoint

            return checkpoint(self._forward_torch, x, pos, doc_start, use_reentrant=False)
        return self._forward_torch(x, pos, doc_start)

    def _norm(self, x, norm, w_none=False):
        return N.rmsnorm_ref(x, None if w_none else norm.weight, self.cfg.rms_norm_eps)

    def _forward_torch(self, x, pos, doc_start):
        _materialize(self, force=True)
        cfg, att = self.cfg, self.self_attn
        T = x.shape[0]
        hd = self.head_dim
        h = self._norm(x, self.input_layernorm)
        q = F.linear(h, att.q_proj.weight).view(T, self.n_q, hd)
        k = F.linear(h, att.k_proj.weight).view(T, self.n_kv, hd)
        v = F.linear(h, att.v_proj.weight).view(T, self.n_kv, hd) if not self.kv_eq else k
        cos, sin = N.rope_cos_sin(pos, self.inv_freq, x.dtype)
        q = N.rope_ref(N.rmsnorm_ref(q, att.q_norm.weight, cfg.rms_norm_eps), cos[:, None], sin[:, None])
        k_n = N.rope_ref(N.rmsnorm_ref(k, att.k_norm.weight, cfg.rms_norm_eps), cos[:, None], sin[:, None])
        v = N.rmsnorm_ref(v, None, cfg.rms_norm_eps)
        a = attention_torch(q, k_n, v, doc_start, self.window, 1.0).reshape(T, -1)
        o = F.linear(a, att.o_proj.weight)
        x = x + self._norm(o, self.post_attention_layernorm)
        h = self._norm(x, self.pre_feedforward_layernorm)
        gu = F.linear(h, self.gate_up_weight)
        m = N.geglu_ref(gu)
        dn = F.linear(m, self.mlp.down_proj.weight)
        x = x + self._norm(dn, self.post_feedforward_layernorm)
        return x * self.layer_scalar.to(x.dtype)


def _ls(layer):
    return layer.layer_scalar.float().reshape(1).contiguous()


# ------------------------------------------------------------------ projections of a layer
# bf16 weights go through ops.linear; an NF4 base with the fused path hands the codes to the
# GEMM that dequantises them in-kernel (micro_engram_fork_b200/csrc/gemm_nf4.cu).
def _nf4_fused(layer):
    nf = getattr(layer, "_nf4", None)
    return nf if nf is not None and nf.fused else None


def _weight(layer, name):
    return {"qkv": layer.qkv_weight, "gate_up": layer.gate_up_weight, "o": layer.self_attn.o_proj.weight,
            "down": layer.mlp.down_proj.weight}[name]


def _proj(layer, name, x):
    """x . W^T for one of the layer's projections."""
    nf = _nf4_fused(layer)
    if nf is None:
        return linear(x, _weight(layer, name))
    from .. import native

    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    return native().gemm_nf4(x2, *nf.operand(name), True, None).view(*x.shape[:-1], -1)


def _proj_t(layer, name, g):
    """g . W: the input gradient of _proj."""
    nf = _nf4_fused(layer)
    if nf is None:
        return linear_t(g, _weight(layer, name))
    from .. import native

    g2 = g.reshape(-1, g.shape[-1]).contiguous()
    return native().gemm_nf4(g2, *nf.operand(name), False, None).view(*g.shape[:-1], -1)


def _geglu_proj(layer, h, save_gu):
    nf = _nf4_fused(layer)
    if nf is None:
        return geglu_linear(h, layer.gate_up_weight, save_gu=save_gu)
    from .. import native

    m, gu = native().gemm_geglu_nf4(h.reshape(-1, h.shape[-1]).contiguous(), *nf.operand("gate_up"), save_gu)
    return m, (gu if save_gu else None)


def _dgeglu_proj(layer, g, gu):
    nf = _nf4_fused(layer)
    if nf is None:
        return dgeglu_linear(g, layer.mlp.down_proj.weight, gu)
    from .. import native

    return native().gemm_dgeglu_nf4(g.reshape(-1, g.shape[-1]).contiguous(), *nf.operand("down"),
                                    gu.reshape(-1, gu.shape[-1]))


def _materialize(layer, direction=1, force=False):
    """Make this layer's full bf16 weights readable before it runs: an NF4 base expands them into
    the shared buffer; a sharded base gathers them from the peers (what the previous GEMMs did
    not already carry) and hands the next layer's gather (`direction` +1 forward, -1 backward)
    to this layer's GEMMs."""
    if getattr(layer, "_nf4", None) is not None:
        from .nf4 import materialize

        materialize(layer, force, direction)
    sb = getattr(layer, "_sharded", None)
    if sb is not None:
        sb.materialize(layer, direction)


def _layer_fwd(layer, x, pos, doc_start, keep=False, direction=1):
    """Native forward of one layer; returns (out, saved dict or None)."""
    from ..ops.attention import attention_fwd

    _materialize(layer, direction)
    cfg = layer.cfg
    eps = cfg.rms_norm_eps
    T = x.shape[0]
    hd = layer.head_dim
    att = layer.self_attn
    h1, r_in = N.rmsnorm(x, layer.input_layernorm.weight, eps)
    qkv = _proj(layer, "qkv", h1)
    q, k, v, r_qkv = N.qkv_norm_rope(qkv, att.q_norm.weight, att.k_norm.weight, layer.inv_freq, pos, layer.n_q,
                                     layer.n_kv, hd, layer.kv_eq, eps)
    a, lse = attention_fwd(q, k, v, doc_start, layer.window, 1.0)
    o = _proj(layer, "o", a.view(T, -1))
    x2, h2, r_o, r_x2 = N.post_norm_add(x, o, layer.post_attention_layernorm.weight, None,
                                        layer.pre_feedforward_layernorm.weight, eps)
    m, gu = _geglu_proj(layer, h2, keep)
    dn = _proj(layer, "down", m)
    x3, _, r_dn, _ = N.post_norm_add(x2, dn, layer.post_feedforward_layernorm.weight, _ls(layer), None, eps)
    saved = None
    if keep:
        saved = dict(r_in=r_in, qkv=qkv, q=q, k=k, v=v, r_qkv=r_qkv, a=a, lse=lse, o=o, x2=x2, r_o=r_o, r_x2=r_x2,
                     gu=gu, dn=dn, r_dn=r_dn)
    return x3, saved


_SAVE_KEYS = ("r_in", "qkv", "q", "k", "v", "r_qkv", "a", "lse", "o", "x2", "r_o", "r_x2", "gu", "dn", "r_dn")
# selective checkpointing keeps the expensive-to-recompute attention half of the layer on the GPU
_SELECTIVE_KEYS = ("qkv", "a", "lse", "o")


def _recompute_selective(layer, x, pos, kept, direction=-1):
    """Rebuild a layer's saved state from its input and the kept attention tensors: norms,
    RoPE and the MLP are recomputed; the q/k/v and o projections and attention are not."""
    _materialize(layer, direction)
    eps = layer.cfg.rms_norm_eps
    att = layer.self_attn
    _, r_in = N.rmsnorm(x, layer.input_layernorm.weight, eps)
    q, k, v, r_qkv = N.qkv_norm_rope(kept["qkv"], att.q_norm.weight, att.k_norm.weight, layer.inv_freq, pos,
                                     layer.n_q, layer.n_kv, layer.head_dim, layer.kv_eq, eps)
    x2, h2, r_o, r_x2 = N.post_norm_add(x, kept["o"], layer.post_attention_layernorm.weight, None,
                                        layer.pre_feedforward_layernorm.weight, eps)
    m, gu = _geglu_proj(layer, h2, True)
    dn = _proj(layer, "down", m)
    _, _, r_dn, _ = N.post_norm_add(x2, dn, layer.post_feedforward_layernorm.weight, _ls(layer), None, eps)
    return dict(r_in=r_in, qkv=kept["qkv"], q=q, k=k, v=v, r_qkv=r_qkv, a=kept["a"], lse=kept["lse"], o=kept["o"],
                x2=x2, r_o=r_o, r_x2=r_x2, gu=gu, dn=dn, r_dn=r_dn)


class _LayerFn(torch.autograd.Function):
    """One decoder layer on the sm_100a kernels with a hand-written dX-only backward.

    checkpoint: False (save everything), "full"/True (save only the input; recompute the
    layer), "selective" (save the input plus the q/k/v projection, attention output + LSE and
    o-proj output, kept on the GPU outside the saved-tensor hooks so activation offloading
    moves only the layer input; recompute norms, RoPE and the MLP)."""

    @staticmethod
    def forward(ctx, x, pos, doc_start, layer, checkpoint):
        ctx.layer, ctx.checkpoint = layer, checkpoint
        out, saved = _layer_fwd(layer, x, pos, doc_start, keep=checkpoint in (False, "selective", "none"))
        if checkpoint == "selective":
            ctx.save_for_backward(x, pos, doc_start)
            ctx.kept = {k: saved[k] for k in _SELECTIVE_KEYS}
        elif checkpoint == "none":
            # everything except q/k/v (cheap to rebuild from qkv), kept on the GPU
            ctx.save_for_backward(x, pos, doc_start)
            ctx.kept = {k: v for k, v in saved.items() if k not in ("q", "k", "v")}
        elif checkpoint:
            ctx.save_for_backward(x, pos, doc_start)
        else:
            ctx.save_for_backward(x, pos, doc_start, *[saved[k] for k in _SAVE_KEYS])
        return out

    @staticmethod
    def backward(ctx, g):
        from ..ops.attention import attention_bwd

        layer = ctx.layer
        _materialize(layer, -1)
        cfg = layer.cfg
        att = layer.self_attn
        tensors = ctx.saved_tensors
        x, pos, doc_start = tensors[:3]
        if ctx.checkpoint == "selective":
            with torch.no_grad():
                s = _recompute_selective(layer, x, pos, ctx.kept)
            ctx.kept = None
        elif ctx.checkpoint == "none":
            s = ctx.kept
            ctx.kept = None
            with torch.no_grad():
                s["q"], s["k"], s["v"], _ = N.qkv_norm_rope(
                    s["qkv"], att.q_norm.weight, att.k_norm.weight, layer.inv_freq, pos, layer.n_q, layer.n_kv,
                    layer.head_dim, layer.kv_eq, cfg.rms_norm_eps)
        elif ctx.checkpoint:
            with torch.no_grad():
                _, s = _layer_fwd(layer, x, pos, doc_start, keep=True, direction=-1)
        else:
            s = dict(zip(_SAVE_KEYS, tensors[3:]))
        T = x.shape[0]
        g = g.contiguous()
        # MLP block: x3 = (x2 + n(dn)) * ls
        d_x2_res, d_dn = N.post_norm_add_bwd(g, None, s["dn"], s["dn"], layer.post_feedforward_layernorm.weight,
                                             _ls(layer), None, s["r_dn"], None)
        d_gu = _dgeglu_proj(layer, d_dn, s["gu"])
        d_h2 = _proj_t(layer, "gate_up", d_gu)
        # attention block: x2 = x + n(o); h2 = n(x2)
        d_x_res, d_o = N.post_norm_add_bwd(d_x2_res, d_h2, s["o"], s["x2"], layer.post_attention_layernorm.weight,
                                           None, layer.pre_feedforward_layernorm.weight, s["r_o"], s["r_x2"])
        d_a = _proj_t(layer, "o", d_o).view_as(s["a"])
        dq, dk, dv = attention_bwd(d_a, s["q"], s["k"], s["v"], s["a"], s["lse"], doc_start, layer.window, 1.0)
        d_qkv = N.qkv_norm_rope_bwd(dq, dk, dv, s["qkv"], att.q_norm.weight, att.k_norm.weight, layer.inv_freq,
                                    pos, s["r_qkv"], layer.n_q, layer.n_kv, layer.head_dim, layer.kv_eq)
        d_h1 = _proj_t(layer, "qkv", d_qkv)
        dx = N.rmsnorm_bwd(d_h1, x, layer.input_layernorm.weight, s["r_in"], d_x_res)
        return dx, None, None, None, None


class GemmaTextModel(nn.Module):
    """The decoder stack + final norm. Takes inputs_embeds (the trainer's vocab shard embeds)."""

    def __init__(self, cfg):
        super().__init__()
        self.config = cfg
        self.layers = nn.ModuleList(GemmaLayer(cfg, i) for i in range(cfg.num_hidden_layers))
        self.norm = _Norm(cfg.hidden_size)

    @property
    def embed_scale(self):
        return float(self.config.hidden_size) ** 0.5

    def gradient_checkpointing_enable(self, upto=None, policy="full"):
        """Per-layer checkpointing for the layers after `upto` (the no-grad prefix needs none).
        policy: "full" (keep only the layer input), "selective" (also keep the attention half),
        "auto" (selective now; plan_checkpointing() later upgrades layers that fit in HBM)."""
        mode = {"auto": "selective", "selective": "selective", "none": "none"}.get(policy, "full")
        for i, layer in enumerate(self.layers):
            layer.gradient_checkpointing = mode if (upto is None or i > upto) else False

    @staticmethod
    def layer_saved_bytes(layer, tokens):
        """(selective, none) bytes a layer keeps on the GPU between its forward and backward."""
        cfg = layer.cfg
        d, f, hd = cfg.hidden_size, cfg.intermediate_size, layer.head_dim
        qkv_w = (layer.n_q + (1 if layer.kv_eq else 2) * layer.n_kv) * hd
        sel = tokens * (qkv_w * 2 + layer.n_q * hd * 2 + d * 2 + layer.n_q * 4 + (layer.n_q + 2 * layer.n_kv) * 4)
        mlp = tokens * (d * 2 + 2 * f * 2 + d * 2 + 4 * 4)
        return sel, sel + mlp

    def plan_checkpointing(self, tokens, budget_bytes, upto=None):
        """HBM-budgeted checkpointing: with `budget_bytes` free for saved activations, every
        trained layer keeps its attention half (selective) when that fits, and as many layers
        as then still fit keep their MLP activations too (no recompute at all). Returns the
        per-layer plan. The math is identical under every plan; only recompute vs memory moves."""
        layers = [l for i, l in enumerate(self.layers) if upto is None or i > upto]
        costs = [self.layer_saved_bytes(l, tokens) for l in layers]
        sel_total = sum(c[0] for c in costs)
        plan = {}
        if sel_total > budget_bytes:
            for l in layers:
                l.gradient_checkpointing = "full"
                plan[l.idx] = "full"
            return plan
        left = budget_bytes - sel_total
        for l, (sel, none) in zip(layers, costs):
            if none - sel <= left:
                l.gradient_checkpointing = "none"
                left -= none - sel
            else:
                l.gradient_checkpointing = "selective"
            plan[l.idx] = l.gradient_checkpointing
        return plan

    def forward(self, inputs_embeds, position_ids):
        """inputs_embeds [1, T, d] or [T, d]; position_ids [1, T] or [T] -> final hidden [T, d]."""
        x = inputs_embeds.reshape(-1, inputs_embeds.shape[-1])
        pos = position_ids.reshape(-1).to(x.device)
        ds = doc_starts(pos)
        d = x.shape[-1]
        for layer in self.layers:
            out = layer(x, pos, ds)
            x = (out[0] if isinstance(out, tuple) else out).reshape(-1, d)  # an engram hook may add a batch dim
        if use_native(x):
            return _FinalNorm.apply(x, self.norm.weight, self.config.rms_norm_eps)
        return N.rmsnorm_ref(x, self.norm.weight, self.config.rms_norm_eps)


class _FinalNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        y, r = N.rmsnorm(x.contiguous(), w, eps)
        ctx.save_for_backward(x, w, r)
        return y

    @staticmethod
    def backward(ctx, g):
        x, w, r = ctx.saved_tensors
        return N.rmsnorm_bwd(g.contiguous(), x, w, r, None), None, None


class GemmaForCausalLM(nn.Module):
    """model.{layers, norm} + a tied embedding (model.embed_tokens) — HF names."""

    def __init__(self, cfg, with_embedding=True):
        super().__init__()
        self.config = cfg
        self.model = GemmaTextModel(cfg)
        if with_embedding:
            self.model.embed_tokens = nn.Embedding(cfg.vocab_size, cfg.hidden_size)
            self.model.embed_tokens.weight.requires_grad_(False)

    def forward(self, input_ids, position_ids=None):
        """Full logits (small models / tests only)."""
        ids = input_ids.reshape(-1)
        if position_ids is None:
            position_ids = torch.arange(ids.numel(), device=ids.device)
        w = self.model.embed_tokens.weight
        emb = (w[ids] * torch.tensor(self.model.embed_scale, dtype=w.dtype)).to(w.dtype)
        h = self.model(emb, position_ids)
        z = (h.to(w.dtype) @ w.t()).float()
        cap = self.config.final_logit_softcapping
        if cap:
            z = torch.tanh(z / cap) * cap
        return z


# ----------------------------------------------------------------------------- init / loading
def text_of(model):
    return model.model if isinstance(model, GemmaForCausalLM) else model


@torch.no_grad()
def cast_projections_(model, dtype):
    """Projection weights (and the embedding) to `dtype`; norms stay fp32."""
    text = text_of(model)
    for layer in text.layers:
        layer.qkv_weight = layer.qkv_weight.to(dtype)
        layer.gate_up_weight = layer.gate_up_weight.to(dtype)
        layer.self_attn.o_proj.weight.data = layer.self_attn.o_proj.weight.data.to(dtype)
        layer.mlp.down_proj.weight.data = layer.mlp.down_proj.weight.data.to(dtype)
        layer._relink()
    emb = getattr(text, "embed_tokens", None)
    if emb is not None:
        emb.weight.data = emb.weight.data.to(dtype)
    return model


@torch.no_grad()
def init_random_(model, seed=0, std=0.02):
    """Random-init every base weight in place on its device (HF's initializer_range
    scheme): projections and embedding N(0, std), norm weights 1, layer scalars 1."""
    text = text_of(model)
    dev = text.layers[0].qkv_weight.device
    g = torch.Generator(device=dev).manual_seed(seed)
    for layer in text.layers:
        for t in (layer.qkv_weight, layer.gate_up_weight, layer.self_attn.o_proj.weight,
                  layer.mlp.down_proj.weight):
            t.normal_(0.0, std, generator=g)
        for n in (layer.input_layernorm, layer.post_attention_layernorm, layer.pre_feedforward_layernorm,
                  layer.post_feedforward_layernorm, layer.self_attn.q_norm, layer.self_attn.k_norm):
            n.weight.fill_(1.0)
        layer.layer_scalar.fill_(1.0)
        layer._relink()
    text.norm.weight.fill_(1.0)
    emb = getattr(text, "embed_tokens", None)
    if emb is not None:
        emb.weight.normal_(0.0, std, generator=g)


_PREFIXES = ("model.language_model.", "model.", "language_model.model.", "language_model.", "")


def hf_key_map(model):
    """{our state-dict key: HF candidates}."""
    out = {}
    for k in model.state_dict():
        base = k[len("model."):] if k.startswith("model.") else k
        out[k] = [p + base for p in _PREFIXES]
    return out


def load_hf_weights(model, folder, device=None, dtype=torch.bfloat16):
    """Fill `model` from an HF Gemma-4 safetensors folder (text weights only)."""
    import glob

    from safetensors import safe_open

    files = sorted(glob.glob(os.path.join(folder, "*.safetensors")))
    where = {}
    for f in files:
        with safe_open(f, framework="pt", device="cpu") as fh:
            for k in fh.keys():
                where[k] = f
    sd = model.state_dict()
    missing = []
    for key, cands in hf_key_map(model).items():
        src = next((c for c in cands if c in where), None)
        if src is None:
            if key.endswith("embed_tokens.weight") and "lm_head.weight" in where:
                src = "lm_head.weight"
            else:
                missing.append(key)
                continue
        with safe_open(where[src], framework="pt", device="cpu") as fh:
            t = fh.get_tensor(src)
        sd[key].copy_(t.to(sd[key].dtype))
    for layer in getattr(model, "model", model).layers:
        layer._relink()
    return missing
