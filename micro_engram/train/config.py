"""YAML config of micro_engram.train.

Same key names, defaults and rules as the reference (micro_engram/train/config.py:1-196):
Axolotl-only keys are accepted and listed in one warning, fused-loss keys are accepted as
no-ops, LoRA keys and FSDP1 are errors, `load_in_8bit`, `liger_rope`,
`fsdp_config.activation_checkpointing` and `use_reentrant: true` are refused, and any other
unknown key is an error.

Keys this framework adds (all optional, defaults keep the reference's behaviour):
  base_init            "load" (weights from base_model) or "random" (random-init weights of
                       base_model's config.json: synthetic benchmarking)
  base_placement       "auto" | "replicated" | "sharded": the frozen base on every GPU, or
                       row-sharded over the GPUs with FSDP2 semantics (each layer gathered for
                       its forward and again for its backward; the gathers ride inside the
                       tcgen05 GEMMs of the previous layer); auto picks replicated when it
                       fits in HBM
  kernels              "native" (sm_100a kernels, the default on CUDA) or "reference"
                       (plain PyTorch ops; oracle runs)
  gradient_checkpointing_policy
                       "full" (default: keep each layer's input) or "selective" (also keep
                       the attention half of each layer on the GPU; recompute only the MLP)
                       or "auto" (HBM-budgeted mix of no recompute and selective)
  gradient_checkpointing_reserve_gib
                       HBM the auto plan leaves free for the backward's working set, the loss
                       chunks and the allocator (plus 4% of the GPU's memory)
  dense_allreduce      "p2p" (default on CUDA with 2+ GPUs: one kernel signals, waits and sums
                       every rank's gradients straight out of its memory over NVLink) or "nccl"
  table_moments_on_host
                       true | false | "auto": keep the lazy optimizer's table-sized moments of
                       the engram tables in pinned host memory (the touched-row update reads
                       and writes them over PCIe, a few MB per step); auto does so when the
                       HBM it frees lets the auto checkpointing plan drop recomputation
"""
import logging
import os
from typing import Any, Dict, List, Literal, Optional, Union

import yaml
from pydantic import BaseModel, ConfigDict, model_validator

from ..args import MicroEngramArgs

LOG = logging.getLogger("micro_engram.train")

IGNORED_KEYS = {
    "plugins", "strict", "tokenizer_type", "trust_remote_code", "bf16", "fp16", "save_safetensors",
    "eval_strategy", "freeze_mm_modules", "pad_to_sequence_len", "micro_engram_save_trainable_only",
    "micro_engram_save_steps", "train_on_inputs", "fsdp", "eval_sample_packing", "special_tokens",
    "chat_template", "flash_attention", "sdp_attention", "xformers_attention", "fsdp_version",
}
IGNORED_FSDP_KEYS = {
    "sync_module_states", "auto_wrap_policy", "transformer_layer_cls_to_wrap", "state_dict_type",
    "fsdp_version", "use_orig_params", "limit_all_gathers",
}
LOSS_KEYS = {"cut_cross_entropy", "liger_cross_entropy", "liger_fused_linear_cross_entropy",
             "chunked_cross_entropy", "chunked_cross_entropy_num_chunks"}
LORA_KEYS = {"adapter", "unfrozen_parameters"}
LORA_PREFIX = ("lora_", "peft_")


class DatasetConfig(BaseModel):
    model_config = ConfigDict(extra="forbid")
    path: str
    type: Literal["completion", "chat_template"]
    field: Optional[str] = None
    field_messages: Optional[str] = None
    message_property_mappings: Optional[Dict[str, str]] = None
    roles: Optional[Dict[str, List[str]]] = None
    roles_to_train: Optional[List[str]] = None
    split: Optional[str] = None
    ds_type: Optional[str] = None


class FsdpConfig(BaseModel):
    model_config = ConfigDict(extra="forbid")
    offload_params: bool = False
    cpu_ram_efficient_loading: bool = False
    reshard_after_forward: bool = True
    activation_checkpointing: Optional[bool] = None

    @model_validator(mode="before")
    @classmethod
    def _without_axolotl_only(cls, data):
        """Axolotl FSDP keys with no meaning here are dropped before the strict check."""
        if not isinstance(data, dict):
            return data
        return {k: data[k] for k in data.keys() - IGNORED_FSDP_KEYS}


class TrainConfig(MicroEngramArgs):
    model_config = ConfigDict(extra="forbid")

    # --- model ---
    base_model: str
    tokenizer_config: Optional[str] = None
    load_in_4bit: bool = False
    attn_implementation: Literal["sdpa", "flash_attention_2", "eager"] = "sdpa"
    gemma4_hybrid_attn_impl: bool = False
    large_head_attention: Optional[Literal["sdpa", "auto", "triton_flash"]] = None
    flash_attn_d512: Optional[bool] = None
    fused_attn_kernel: bool = True
    liger_rms_norm: bool = False
    liger_layer_norm: bool = False
    liger_glu_activation: bool = False
    liger_rope: bool = False
    tf32: bool = False
    base_init: Literal["load", "random"] = "load"
    base_placement: Literal["auto", "replicated", "sharded"] = "auto"
    kernels: Literal["native", "reference"] = "native"

    # --- data ---
    datasets: List[DatasetConfig]
    sequence_len: int = 2048
    sample_packing: bool = True
    dataset_prepared_path: Optional[str] = None
    axolotl_prepared_dataset: Optional[str] = None
    dataset_num_proc: Optional[int] = None
    chat_template_jinja: Optional[str] = None
    chat_template_kwargs: Optional[Dict[str, Any]] = None
    eot_tokens: Optional[List[str]] = None
    shuffle_each_epoch: bool = True

    # --- training ---
    output_dir: str
    micro_batch_size: int = 1
    gradient_accumulation_steps: int = 1
    num_epochs: float = 1
    max_steps: Optional[int] = None
    learning_rate: float = 1e-3
    micro_engram_dense_lr: Optional[float] = None
    micro_engram_train_scales: bool = True
    lr_scheduler: Literal["constant", "constant_with_warmup", "cosine", "linear",
                          "warmup_stable_decay"] = "constant_with_warmup"
    lr_scheduler_kwargs: Optional[Dict[str, Any]] = None
    cosine_min_lr_ratio: Optional[float] = None
    warmup_ratio: Optional[float] = None
    warmup_steps: Optional[int] = None
    weight_decay: float = 0.0
    adam_beta1: float = 0.9
    adam_beta2: float = 0.999
    adam_epsilon: float = 1e-8
    max_grad_norm: float = 1.0
    optimizer: Optional[str] = None
    seed: int = 42
    gradient_checkpointing: bool = True
    gradient_checkpointing_kwargs: Optional[Dict[str, Any]] = None
    # full: keep only each layer's input (the reference's behaviour); selective: also keep the
    # q/k/v projection, attention output + LSE and o-proj output on the GPU, recompute the rest
    # auto: selective where it fits in HBM, plus no recompute at all for as many layers as still fit
    gradient_checkpointing_policy: Literal["full", "selective", "auto"] = "full"
    gradient_checkpointing_reserve_gib: float = 23.0
    table_moments_on_host: Union[bool, Literal["auto"]] = "auto"
    dense_allreduce: Literal["p2p", "nccl"] = "p2p"
    activation_offloading: bool = False
    no_grad_prefix: bool = True
    sharded_vocab: bool = True
    sparse_row_grads: bool = True
    loss_chunk_tokens: int = 2048
    fsdp_config: FsdpConfig = FsdpConfig()

    # --- checkpoints / logging ---
    save_steps: Optional[int] = None
    save_total_limit: Optional[int] = None
    auto_resume_from_checkpoints: bool = True
    resume_from_checkpoint: Optional[str] = None
    logging_steps: int = 1
    profile_step: Optional[int] = None
    wandb_project: Optional[str] = None
    wandb_name: Optional[str] = None
    wandb_entity: Optional[str] = None
    wandb_mode: Optional[str] = None

    @model_validator(mode="after")
    def _check(self):
        for broken, why in _CONFIG_ERRORS:
            if broken(self):
                raise ValueError(why)
        return self

    @property
    def large_head_policy(self):
        """The hd-512 attention route: large_head_attention when set, else flash_attn_d512's
        legacy meaning (True: auto, unset or False: sdpa)."""
        return self.large_head_attention or ("auto" if self.flash_attn_d512 else "sdpa")

    def get(self, key, default=None):
        v = getattr(self, key, default)
        return default if v is None else v


# Combinations of valid keys that this trainer refuses, with the reason shown to the user.
_CONFIG_ERRORS = (
    (lambda c: bool(c.fsdp_config.activation_checkpointing),
     "fsdp_config.activation_checkpointing: set gradient_checkpointing: true instead (this trainer "
     "checkpoints each decoder layer itself, non-reentrant)"),
    (lambda c: c.micro_engram_dense_lr is not None and c.micro_engram_dense_lr <= 0,
     "micro_engram_dense_lr must be positive; to keep an engram fixed use micro_engram_frozen"),
    (lambda c: c.liger_rope,
     "liger_rope: RoPE is already applied inside the fused q/k/v norm kernel"),
    (lambda c: bool((c.gradient_checkpointing_kwargs or {}).get("use_reentrant")),
     "gradient_checkpointing_kwargs.use_reentrant: true is not supported (the frozen layers' inputs carry "
     "no gradient, so reentrant checkpointing would drop the engram's)"),
    (lambda c: c.micro_engram_sharding not in (None, "rows"),
     "micro_engram_sharding: tables are always row-sharded here; use rows or leave it out"),
    (lambda c: c.lr_scheduler == "warmup_stable_decay" and not c.micro_engram_lr_epoch_decay
     and "num_decay_steps" not in (c.lr_scheduler_kwargs or {}),
     "lr_scheduler: warmup_stable_decay needs lr_scheduler_kwargs.num_decay_steps (the length of its final "
     "decay)"),
)


def _read(path_or_dict):
    if isinstance(path_or_dict, dict):
        return dict(path_or_dict)
    with open(path_or_dict, encoding="utf-8") as f:
        return yaml.safe_load(f) or {}


def _screen(raw, announce):
    """Apply the key rules to a raw YAML mapping in place: LoRA keys, FSDP1 and 8-bit loading
    are errors; Axolotl-only keys and loss-implementation keys are dropped with one warning
    each (the loss here is always the fused, chunked, vocab-parallel one)."""
    lora = [k for k in raw if k in LORA_KEYS or k.startswith(LORA_PREFIX)]
    if lora:
        raise ValueError(f"{', '.join(sorted(lora))}: no adapter is trained or needed; the base stays frozen "
                         "(load_in_4bit: true quantizes it directly) and only the engram trains")
    if raw.get("fsdp_version") is not None and str(raw["fsdp_version"]) != "2":
        raise ValueError("fsdp_version: only 2 (FSDP2 semantics) is supported")
    if raw.pop("load_in_8bit", False):
        raise ValueError("load_in_8bit is not supported; use load_in_4bit (NF4)")
    dropped = {"ignoring Axolotl-only keys": sorted(k for k in raw if k in IGNORED_KEYS),
               "not needed (the loss is always fused, chunked and vocab-parallel)":
                   sorted(k for k in raw if k in LOSS_KEYS)}
    for what, keys in dropped.items():
        for k in keys:
            del raw[k]
        if keys and announce:
            LOG.warning(f"[micro_engram] {what}: {', '.join(keys)}")
    return raw


def load_config(path_or_dict):
    """TrainConfig from a YAML file or a dict (unknown keys are errors)."""
    raw = _screen(_read(path_or_dict), announce=os.environ.get("RANK", "0") == "0")
    return TrainConfig(**raw)
