"""Model side of micro_engram.train: the frozen Gemma-4-style base (our own decoder,
micro_engram_fork_b200.models.gemma, loaded from HF safetensors or random-initialised),
its placement on the GPUs, the vocab shard, the no-grad prefix and checkpointing.

Reference counterpart: micro_engram/train/model.py:1-285 (HF model + FSDP2 + kernel patches).
B200 placement: the base is frozen, so a GPU never needs its gradients or optimizer state.
With 180 GB of HBM a 31B bf16 base (62 GB) fits on every GPU, so `base_placement: auto`
replicates it (no per-layer all-gathers at all) unless it does not fit; `sharded` keeps FSDP2's
layout (each rank holds 1/world of every layer; the next layer's all-gather is carried by the
current layer's tcgen05 GEMMs, see micro_engram_fork_b200/parallel/sharded_base.py).
"""
import logging
import os
from contextlib import contextmanager

import torch
import torch.distributed as dist
import torch.nn as nn

from micro_engram_fork_b200.models import gemma as G

from ..module import find_text_layers

LOG = logging.getLogger("micro_engram.train")


def apply_kernel_patches(cfg, on_cuda):
    """The reference patched HF's Gemma 4 with Triton/Liger kernels; our decoder always runs
    the sm_100a kernels on CUDA, so the keys are accepted and only logged."""
    if on_cuda and cfg.kernels == "native":
        LOG.warning("[micro_engram] kernels: sm_100a fused q/k/v norm + RoPE, packed-varlen attention "
                    "(sliding hd256 / global hd512), RMSNorm epilogues, GeGLU, fused engram gate, fused CE")


def _base_config(path):
    cfg_file = os.path.join(path, "config.json")
    if not os.path.isfile(cfg_file):
        raise FileNotFoundError(f"base_model {path} has no config.json")
    conf = G.GemmaConfig.from_pretrained(path)
    return conf


def load_base(cfg, rank, local_rank, device):
    """(model, meta) — the frozen base on `device`, bf16 projections, fp32 norms."""
    conf = _base_config(cfg.base_model)
    if cfg.load_in_4bit:
        from micro_engram_fork_b200.models.nf4 import quantize_model_nf4

        LOG.warning("[micro_engram] load_in_4bit: NF4 (block 64, fp32 absmax) frozen base")
    with torch.device("meta"):
        model = G.GemmaForCausalLM(conf, with_embedding=True)
    model = model.to_empty(device=device)
    for layer in model.model.layers:
        layer._relink()
    G.cast_projections_(model, torch.bfloat16)
    efficient = cfg.fsdp_config.cpu_ram_efficient_loading and dist.is_initialized() and dist.get_world_size() > 1
    if cfg.base_init == "random":
        G.init_random_(model, seed=cfg.seed)
    elif not efficient or rank == 0:
        missing = G.load_hf_weights(model, cfg.base_model)
        if missing:
            raise ValueError(f"[micro_engram] base_model {cfg.base_model} is missing weights: {missing[:8]}")
    if efficient and cfg.base_init != "random":
        for t in list(model.parameters()) + list(model.buffers()):
            dist.broadcast(t.data, src=0)
    for p in model.parameters():
        p.requires_grad_(False)
    if cfg.load_in_4bit:
        quantize_model_nf4(model)
    return model, False


def text_model(model):
    """(name, the text decoder stack's owner): the module one level above the layer list."""
    layers_name, _ = find_text_layers(model)
    parent, _, _ = layers_name.rpartition(".")
    return parent, model.get_submodule(parent) if parent else model


def hybrid_attention(text, cfg):
    """Sliding and global layers always run the packed-varlen kernels (documents from
    position_ids); nothing to switch."""
    return


class _NoEmbedding(nn.Module):
    def __init__(self, num, dim):
        super().__init__()
        self.num_embeddings, self.embedding_dim = num, dim

    def forward(self, ids):  # pragma: no cover
        raise RuntimeError("micro_engram.train feeds inputs_embeds; the embedding lives in VocabShard")


def take_vocab(model, text, rank, world, device, broadcast=False, chunk_tokens=2048):
    """Split the tied embedding/head by rows over the GPUs (VocabShard); remove it from the model."""
    from .head import VocabShard

    emb = text.embed_tokens
    W = emb.weight.detach()
    softcap = getattr(text.config, "final_logit_softcapping", None)
    scale = float(text.config.hidden_size) ** 0.5
    if broadcast and world > 1:
        buf = W.to(device=device, dtype=torch.bfloat16) if rank == 0 else torch.empty(
            W.shape, dtype=torch.bfloat16, device=device)
        dist.broadcast(buf, src=0)
        W = buf
    shard = VocabShard(W, rank, world, embed_scale=scale, softcap=softcap, chunk_tokens=chunk_tokens,
                       device=device, dtype=torch.bfloat16)
    del W
    text.embed_tokens = _NoEmbedding(shard.V, shard.d)
    if getattr(model, "lm_head", None) is not None:
        model.lm_head = None
    return shard


@contextmanager
def grad_from_layer(text, first_layer, enabled):
    """Layers up to and including `first_layer` run without autograd; grad turns on right
    before that layer's engram injects (a prepended forward hook)."""
    if not enabled or first_layer is None:
        yield
        return
    before = torch.is_grad_enabled()

    def switch_on(_module, _args, _output):  # returns nothing, so the layer's output stands
        torch.set_grad_enabled(True)

    # forward hooks run in registration order: prepended, this one runs ahead of the engram's
    hook = text.layers[first_layer].register_forward_hook(switch_on, prepend=True)
    torch.set_grad_enabled(False)
    try:
        yield
    finally:
        torch.set_grad_enabled(before)
        hook.remove()


def checkpointing(model, text, cfg, no_grad_upto):
    """Per-layer activation checkpointing (only the layer input is kept), off for the prefix."""
    if not cfg.gradient_checkpointing:
        return
    text.gradient_checkpointing_enable(upto=no_grad_upto, policy=cfg.gradient_checkpointing_policy)


def base_bytes(text):
    return sum(t.numel() * t.element_size() for t in list(text.parameters()) + list(text.buffers()))


def place_base(text, cfg, device, world):
    """Place the frozen base: "replicated" (every GPU holds all of it; `auto` picks this when it
    fits in 60% of HBM) or "sharded" (FSDP2's layout: each GPU holds 1/world of every layer, the
    layer all-gathers ride inside the tcgen05 GEMMs; micro_engram_fork_b200.parallel.sharded_base).
    Returns the placement used. fsdp_config keys that the placement makes moot are reported."""
    mode = cfg.base_placement
    if mode == "auto":
        mode = "replicated"
        if device.type == "cuda" and world > 1:
            _, total = torch.cuda.mem_get_info(device)
            if base_bytes(text) >= 0.6 * total:
                mode = "sharded"
    fsdp = cfg.fsdp_config
    if fsdp.offload_params:
        LOG.warning("[micro_engram] fsdp_config.offload_params is not supported (the frozen base stays in HBM: "
                    "activations, not parameters, are offloaded); ignoring it")
    if mode == "sharded" and (world == 1 or device.type != "cuda"):
        LOG.warning("[micro_engram] base_placement: sharded needs CUDA and 2+ GPUs; the base stays replicated")
        mode = "replicated"
    if mode == "sharded" and cfg.load_in_4bit:
        raise ValueError("base_placement: sharded is for a bf16 base; an NF4 base (load_in_4bit) is replicated "
                         "(31B in NF4 is 17 GB)")
    if mode == "replicated":
        if world > 1 and not fsdp.reshard_after_forward:
            LOG.warning("[micro_engram] fsdp_config.reshard_after_forward has no effect: the base is replicated")
        return "replicated"
    if not fsdp.reshard_after_forward:
        LOG.warning("[micro_engram] fsdp_config.reshard_after_forward: false is not supported; each layer is "
                    "gathered again for its backward (two gather slots per GPU)")
    from micro_engram_fork_b200.parallel.sharded_base import ShardedBase, activate

    sb = ShardedBase(text.layers, dist.get_rank(), world, device)
    activate(sb)
    text._sharded_base = sb
    LOG.warning(f"[micro_engram] base_placement: sharded over {world} GPUs ({sb.nbytes() / 2 ** 30:.1f} GiB per GPU "
                "incl. two gather slots); layer all-gathers carried by the tcgen05 GEMMs")
    return "sharded"
