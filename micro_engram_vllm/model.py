"""Gemma 4 with micro-engrams for vLLM (text path, Model Runner V2).

Reference behaviour: micro_engram_vllm/model.py (engram resolution :93-134, attachment
:138-214, weight loading :225-293, multimodal wrapper :293-326).

Each engram layer (listed by the engram config) gets its engram and a view of ONE shared
int32 history buffer [max_batched_tokens, max_order]. Before every step the model state
fills that buffer (micro_engram_vllm/ids.py); inside the compiled model each engram layer
then runs one custom op (`micro_engram_b200::serve_inject`): hash -> row read from the
owning TP rank's peer-mapped row store -> key/value projections -> gate -> residual add.
Without an engram config the classes behave like stock Gemma 4.

Selection (first match wins):
  1. --additional-config '{"micro_engram": "<config.json or its folder>"}' or
     MICRO_ENGRAM_CONFIG: weights from each engram's "weights" entry, base untouched.
  2. micro_engram_config.json next to the model weights (an assembled folder): the engram
     tensors come from the checkpoint itself.
MICRO_ENGRAM_OFF=1 loads the engram but skips it (A/B); {"micro_engram_offload": true} or
MICRO_ENGRAM_OFFLOAD=1 keeps the rows in pinned host memory read through UVA views.
"""
import json
import os

import torch

from vllm.config import VllmConfig
from vllm.distributed import (get_tensor_model_parallel_rank, get_tensor_model_parallel_world_size, get_tp_group,
                              tensor_model_parallel_all_reduce)
from vllm.logger import init_logger
from vllm.model_executor.models.gemma4 import Gemma4DecoderLayer, Gemma4ForCausalLM
from vllm.model_executor.models.gemma4_mm import Gemma4ForConditionalGeneration
from vllm.model_executor.models.utils import PPMissingLayer

from micro_engram.module import engram_from_spec
from micro_engram.weights import _local_name, base_mismatch, engram_specs, layer_of_key, load_engram_weights

from .ids import mask_media
from .tp import fused_ok, load_rows, serve_inject, tp_lookup

logger = init_logger("vllm.micro_engram")  # under "vllm." so vLLM's handler prints it

CONFIG_NAME = "micro_engram_config.json"
_WRAP = "._checkpoint_wrapped_module."


class EngramGemma4DecoderLayer(Gemma4DecoderLayer):
    """Gemma 4 decoder layer that adds its engram's gated memory to the layer output."""

    def forward(self, positions, hidden_states, residual, per_layer_input=None, **kwargs):
        hidden_states, residual = super().forward(positions, hidden_states, residual,
                                                  per_layer_input=per_layer_input, **kwargs)
        if not self.micro_engram_on:  # fixed at load time: a constant for the compiler
            return hidden_states, residual
        hist = self.micro_engram_ids[: hidden_states.shape[0]]
        keep = None
        if self.micro_engram_media is not None:
            hist, keep = mask_media(hist, self.micro_engram_media)
        engram = self.micro_engram
        if fused_ok(engram, hidden_states):
            return serve_inject(engram, hidden_states, hist, keep), residual
        return engram.inject(hidden_states, engram.hash_prev(hist), keep), residual


def _uses_v2_model_runner(vllm_config):
    """Model Runner V2? Newer vLLM drops the config flag; then look at who builds the model."""
    flag = getattr(vllm_config, "use_v2_model_runner", None)
    if flag is not None:
        return bool(flag)
    import inspect

    frames = [f.filename.replace("\\", "/") for f in inspect.stack(context=0)]
    if any(f.endswith("/v1/worker/gpu/model_runner.py") for f in frames):
        return True
    if any(f.endswith("/v1/worker/gpu_model_runner.py") for f in frames):
        return False
    logger.warning("[micro_engram] could not tell which vLLM model runner builds the model; assuming V2")
    return True


def _offload_wanted(vllm_config):
    extra = vllm_config.additional_config
    if isinstance(extra, dict) and "micro_engram_offload" in extra:
        return bool(extra["micro_engram_offload"])
    return os.environ.get("MICRO_ENGRAM_OFFLOAD", "0") == "1"


def _host_views(shards):
    """Device (UVA) views of pinned host rows: kernels read only the rows they index."""
    from vllm.utils.platform_utils import is_uva_available
    from vllm.utils.torch_utils import get_accelerator_view_from_cpu_tensor

    if not is_uva_available():
        raise RuntimeError("[micro_engram] micro_engram_offload needs UVA (pinned host memory the GPU can read); "
                           "serve without offload")
    return [get_accelerator_view_from_cpu_tensor(p.data) for p in shards]


def resolve_engram(additional_config, model_dir, environ=None):
    """(config dict, config path, weights from separate files?) or (None, None, False)."""
    environ = os.environ if environ is None else environ
    chosen = (additional_config.get("micro_engram") if isinstance(additional_config, dict) else None) or \
        environ.get("MICRO_ENGRAM_CONFIG")
    if chosen:
        path = os.path.join(chosen, CONFIG_NAME) if os.path.isdir(chosen) else chosen
        if not os.path.isfile(path):
            raise ValueError(f"[micro_engram] engram config not found: {path}")
        with open(path) as f:
            conf = json.load(f)
        for spec in engram_specs(conf, path):
            if not spec["weights"]:
                raise ValueError(
                    f"[micro_engram] {path}: the engram at layer {spec['layer']} has no \"weights\" (the copy "
                    f"written at the start of training has none): point at checkpoint-N/{CONFIG_NAME}, or set "
                    f"\"weights\" to a file or folder (relative to the config's folder)")
            if not os.path.exists(spec["weights"]):
                raise ValueError(f"[micro_engram] {path}: the weights of the engram at layer {spec['layer']} are "
                                 f"missing: {spec['weights']} (relative paths are relative to the config's folder)")
        return conf, path, True
    path = os.path.join(model_dir, CONFIG_NAME)
    if os.path.isfile(path):
        with open(path) as f:
            return json.load(f), path, False
    return None, None, False


class EngramGemma4ForCausalLM(Gemma4ForCausalLM):
    def __init__(self, *, vllm_config: VllmConfig, prefix: str = ""):
        super().__init__(vllm_config=vllm_config, prefix=prefix)
        self.micro_engram_slots = []
        self.micro_engram_separate = False
        self.micro_engram_conf = None
        self._micro_engram_ids = None
        conf, conf_path, separate = resolve_engram(vllm_config.additional_config, vllm_config.model_config.model)
        if conf is None:
            logger.info("[micro_engram] no engram configured: plain Gemma 4")
            return
        self.micro_engram_separate = separate
        self.micro_engram_conf = conf
        msg = base_mismatch(conf, vllm_config.model_config.model)
        if msg:
            logger.warning("[micro_engram] %s", msg)
        arch = vllm_config.model_config.architecture
        if arch not in ("Gemma4ForCausalLM", "Gemma4ForConditionalGeneration"):
            raise ValueError(f"[micro_engram] {arch} is not supported (the engram would never be fed); serve "
                             "Gemma4ForConditionalGeneration or Gemma4ForCausalLM")
        if not _uses_v2_model_runner(vllm_config):
            raise ValueError("[micro_engram] needs vLLM's Model Runner V2 (it fills the engram history before "
                             "every step); set VLLM_USE_V2_MODEL_RUNNER=1 (releases that default Gemma 4 to the V1 "
                             "runner need it; MICRO_ENGRAM_CONFIG sets it when the plugin loads)")
        specs = engram_specs(conf, conf_path)
        max_order = max(max(s["orders"]) for s in specs)
        tp_rank, tp_size = get_tensor_model_parallel_rank(), get_tensor_model_parallel_world_size()
        offload = _offload_wanted(vllm_config)
        on = os.environ.get("MICRO_ENGRAM_OFF", "0") != "1"
        text_cfg = getattr(self.config, "text_config", self.config)
        for spec in specs:
            layer = self.model.layers[spec["layer"]]
            if isinstance(layer, PPMissingLayer):
                continue  # pipeline parallel: the layer lives on another rank
            engram = engram_from_spec(spec, text_cfg.hidden_size, text_cfg.vocab_size,
                                      getattr(text_cfg, "pad_token_id", None) or 0, build_tables=False)
            ref = next(layer.parameters())
            engram.to(device=ref.device, dtype=ref.dtype)
            if offload:
                engram.shard_rows(tp_rank, tp_size, device="cpu", dtype=ref.dtype, requires_grad=False,
                                  empty=True, pin_memory=True)
                engram.__dict__["row_views"] = _host_views(engram.row_shards)
                engram.row_lookup_fn = tp_lookup(tensor_model_parallel_all_reduce)
            else:
                # peer-mapped row store across the TP group: the fused op reads owners' rows directly
                group = get_tp_group().cpu_group if tp_size > 1 else None
                engram.shard_rows(tp_rank, tp_size, device=ref.device, dtype=ref.dtype, requires_grad=False,
                                  empty=True, group=group)
            layer.add_module("micro_engram", engram)
            if self._micro_engram_ids is None:
                self._micro_engram_ids = torch.full((vllm_config.scheduler_config.max_num_batched_tokens, max_order),
                                                    -1, dtype=torch.int32, device=ref.device)
            layer.register_buffer("micro_engram_ids", self._micro_engram_ids, persistent=False)
            layer.micro_engram_on = on
            layer.micro_engram_media = None
            layer.__class__ = EngramGemma4DecoderLayer
            self.micro_engram_slots.append((spec, layer))
            held = sum(p.numel() * p.element_size() for p in engram.row_shards) / 2 ** 30
            logger.info("[micro_engram] layer %d: %s gate, %d tables x %d dims, rows per order %s; this rank holds "
                        "1/%d (%.2f GiB, %s), seed %d%s; weights from %s", spec["layer"], engram.gate,
                        len(engram.row_shards), engram.engram_dim, engram.order_sizes, tp_size, held,
                        "pinned host memory" if offload else "peer-mapped row store", spec["seed"],
                        "" if on else " (OFF: MICRO_ENGRAM_OFF=1)",
                        spec["weights"] if separate else "the model checkpoint")

    @property
    def micro_engram_ids(self):
        return self._micro_engram_ids

    def get_model_state_cls(self):
        from .model_state import EngramModelState

        return EngramModelState

    def load_weights(self, weights):
        if not self.micro_engram_slots:
            return super().load_weights(weights)
        found = {}

        def without_engram():
            for name, w in weights:
                name = name.replace(_WRAP, ".")
                if ".micro_engram." in name:
                    found.setdefault(layer_of_key(name), {})[_local_name(name)] = w
                else:
                    yield name, w

        loaded = super().load_weights(without_engram())
        if self.micro_engram_separate:
            if found:
                logger.warning("[micro_engram] the checkpoint has its own engram (%d tensors); using the "
                               "configured engram weights instead", sum(map(len, found.values())))
            if not getattr(self, "_micro_engram_loaded", False):  # the loader may call us once per name run
                self._micro_engram_loaded = True
                for spec, layer in self.micro_engram_slots:
                    loaded |= self._load_separate(spec, layer)
            return loaded
        done = self.__dict__.setdefault("_micro_engram_tables_done", {})
        for spec, layer in self.micro_engram_slots:
            part = found.get(spec["layer"])
            if not part:
                continue
            engram = layer.micro_engram
            got = done.setdefault(spec["layer"], set())
            got |= load_rows(engram, part, f"the checkpoint (layer {spec['layer']})", complete=False)
            loaded |= self._param_names(engram, part)
            logger.info("[micro_engram] layer %d: %d of %d tables loaded", spec["layer"], len(got),
                        len(engram.row_shards))
        return loaded

    def _param_names(self, engram, keys=None):
        prefix = next(n for n, m in self.named_modules() if m is engram)
        return {f"{prefix}.{n}" for n, _ in engram.named_parameters() if keys is None or n in keys}

    def _load_separate(self, spec, layer):
        engram = layer.micro_engram
        shared = sum(s["weights"] == spec["weights"] for s, _ in self.micro_engram_slots) > 1
        sd = load_engram_weights(spec["weights"], layer=spec["layer"], need_layer=shared)
        if not any(k.startswith("tables.") for k in sd):
            raise ValueError(f"[micro_engram] no engram weights for layer {spec['layer']} in {spec['weights']}")
        if "canon" not in sd and spec.get("token_merge"):
            canon_path = spec.get("canon_path")
            if not canon_path or not os.path.isfile(canon_path):
                raise ValueError("[micro_engram] the run merged tokens but the weights have no 'canon' and the "
                                 f"canon file is missing ({canon_path})")
            sd["canon"] = torch.load(canon_path, map_location="cpu")
        load_rows(engram, sd, spec["weights"])
        logger.info("[micro_engram] layer %d: loaded %d engram tensors from %s", spec["layer"], len(sd),
                    spec["weights"])
        return self._param_names(engram)


class EngramGemma4ForConditionalGeneration(Gemma4ForConditionalGeneration):
    """Multimodal Gemma 4: the language model inside is built through the registry (so it is
    EngramGemma4ForCausalLM); this wrapper exposes its history buffer and model state, and
    marks media placeholder ids (no engram on them; missing as history)."""

    def __init__(self, *, vllm_config: VllmConfig, prefix: str = ""):
        super().__init__(vllm_config=vllm_config, prefix=prefix)
        slots = getattr(self.language_model, "micro_engram_slots", None)
        if not slots:
            return
        media = sorted({int(t) for t in (getattr(self.config, n, None)
                                         for n in ("image_token_id", "video_token_id", "audio_token_id"))
                        if t is not None})
        for _, layer in slots:
            layer.__dict__.pop("micro_engram_media", None)
            layer.register_buffer("micro_engram_media",
                                  torch.tensor(media, dtype=torch.int32, device=layer.micro_engram_ids.device),
                                  persistent=False)
        logger.info("[micro_engram] multimodal model: no engram on media placeholder ids %s", media)

    @property
    def micro_engram_ids(self):
        return getattr(self.language_model, "micro_engram_ids", None)

    def get_model_state_cls(self):
        from .model_state import EngramModelState

        return EngramModelState
