"""Gemma 4 with micro-engrams inside vLLM (text path, Model Runner V2).

The plugin's public behaviour is the reference plugin's (Ready-Art/micro_engram_fork,
micro_engram_vllm/model.py: engram selection :93-134, attachment :138-214, weight loading
:225-293, multimodal wrapper :293-326): the same classes, keys, environment variables and
history rule, so existing command lines keep working. The serving path is this framework's:
every engram layer gets a view of ONE shared int32 history buffer [max_batched_tokens,
max_order] that the model state fills before each step (micro_engram_vllm/ids.py), and inside
the compiled model the layer runs one custom op (`micro_engram_b200::serve_inject`): hash ->
row read from the owning TP rank's peer-mapped row store -> key/value projections -> gate ->
residual add. Without an engram config the classes are stock Gemma 4.

Which engram (first match wins):
  1. --additional-config '{"micro_engram": "<config.json or its folder>"}', or
     MICRO_ENGRAM_CONFIG: each engram's weights come from its own "weights" entry;
  2. micro_engram_config.json beside the model weights (an assembled folder): the engram
     tensors are part of the checkpoint.
MICRO_ENGRAM_OFF=1 loads the engram but bypasses it (A/B runs); {"micro_engram_offload": true}
or MICRO_ENGRAM_OFFLOAD=1 keeps the rows in pinned host memory, read through UVA views.
"""
import json
import os
from dataclasses import dataclass

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

logger = init_logger("vllm.micro_engram")  # a "vllm." logger: vLLM's handler prints it

CONFIG_NAME = "micro_engram_config.json"
SUPPORTED_ARCHS = ("Gemma4ForCausalLM", "Gemma4ForConditionalGeneration")
MEDIA_TOKEN_FIELDS = ("image_token_id", "video_token_id", "audio_token_id")


# ============================================================================ selection
@dataclass
class EngramSelection:
    conf: dict
    path: str
    separate: bool  # weights in their own files (True) or inside the model checkpoint (False)


def _chosen_path(additional_config, environ):
    from_cli = additional_config.get("micro_engram") if isinstance(additional_config, dict) else None
    return from_cli or environ.get("MICRO_ENGRAM_CONFIG")


def _check_weights_exist(conf, path):
    for spec in engram_specs(conf, path):
        where = spec["weights"]
        if not where:
            raise ValueError(f"[micro_engram] {path}: the engram at layer {spec['layer']} names no \"weights\" (the "
                             f"copy written when training starts has none): use checkpoint-N/{CONFIG_NAME}, or set "
                             "\"weights\" to a file or folder (relative to the config's folder)")
        if not os.path.exists(where):
            raise ValueError(f"[micro_engram] {path}: the weights of the engram at layer {spec['layer']} are missing: "
                             f"{where} (relative paths start at the config's folder)")


def _read_json(path):
    with open(path) as f:
        return json.load(f)


def select_engram(additional_config, model_dir, environ=None):
    """The engram to serve, or None for plain Gemma 4: a config named by --additional-config or
    MICRO_ENGRAM_CONFIG (a file, or a folder holding one; weights in their own files), else a
    config beside the model (an assembled folder; weights inside the checkpoint)."""
    environ = os.environ if environ is None else environ
    chosen = _chosen_path(additional_config, environ)
    if not chosen:
        beside = os.path.join(model_dir, CONFIG_NAME)
        return EngramSelection(_read_json(beside), beside, separate=False) if os.path.isfile(beside) else None
    path = os.path.join(chosen, CONFIG_NAME) if os.path.isdir(chosen) else chosen
    if not os.path.isfile(path):
        raise ValueError(f"[micro_engram] engram config not found: {path}")
    conf = _read_json(path)
    _check_weights_exist(conf, path)
    return EngramSelection(conf, path, separate=True)


def resolve_engram(additional_config, model_dir, environ=None):
    """(config, config path, separate weights?) or (None, None, False)."""
    sel = select_engram(additional_config, model_dir, environ)
    return (sel.conf, sel.path, sel.separate) if sel else (None, None, False)


def runner_is_v2(vllm_config):
    """Does vLLM's Model Runner V2 build this model? The config says so in releases that have the
    flag; otherwise the caller's module tells (V2 lives in v1/worker/gpu/model_runner.py)."""
    flag = getattr(vllm_config, "use_v2_model_runner", None)
    if flag is not None:
        return bool(flag)
    import inspect

    callers = {f.filename.replace("\\", "/") for f in inspect.stack(context=0)}
    if any(c.endswith("/v1/worker/gpu/model_runner.py") for c in callers):
        return True
    if any(c.endswith("/v1/worker/gpu_model_runner.py") for c in callers):
        return False
    logger.warning("[micro_engram] could not tell which vLLM model runner builds the model; assuming V2")
    return True


def _offload_rows(vllm_config):
    extra = vllm_config.additional_config
    if isinstance(extra, dict) and "micro_engram_offload" in extra:
        return bool(extra["micro_engram_offload"])
    return os.environ.get("MICRO_ENGRAM_OFFLOAD", "0") == "1"


def _uva_views(shards):
    """Device (UVA) views of pinned host rows: kernels read only the rows they index."""
    from vllm.utils.platform_utils import is_uva_available
    from vllm.utils.torch_utils import get_accelerator_view_from_cpu_tensor

    if not is_uva_available():
        raise RuntimeError("[micro_engram] micro_engram_offload needs UVA (pinned host memory the GPU can read); "
                           "serve without it")
    return [get_accelerator_view_from_cpu_tensor(p.data) for p in shards]


def fused_tp_wanted(vllm_config, environ=None):
    """Replace the row-parallel linears' GEMM + all-reduce with the fused peer-memory op?
    additional_config {"micro_engram_fused_tp": true} or MICRO_ENGRAM_FUSED_TP=1; off by default."""
    environ = os.environ if environ is None else environ
    extra = getattr(vllm_config, "additional_config", None)
    if isinstance(extra, dict) and "micro_engram_fused_tp" in extra:
        return bool(extra["micro_engram_fused_tp"])
    return environ.get("MICRO_ENGRAM_FUSED_TP", "0") == "1"


def _fusable(lin):
    """A plain bf16 row-parallel linear whose output vLLM all-reduces."""
    w = getattr(lin, "weight", None)
    return (getattr(lin, "input_is_parallel", False) and getattr(lin, "reduce_results", False)
            and getattr(lin, "bias", None) is None and w is not None and w.dim() == 2 and w.dtype == torch.bfloat16
            and w.shape[0] % 8 == 0 and w.shape[1] % 8 == 0)


def _route_row_parallel(lin, handle, rows):
    """lin.forward -> the fused op for bf16 inputs of at most `rows` rows (else vLLM's own path)."""
    from micro_engram_fork_b200.ops.registry import tp_row_linear

    plain = lin.forward

    def forward(input_):
        if input_.dim() != 2 or input_.dtype != torch.bfloat16 or input_.shape[0] > rows:
            return plain(input_)
        y = tp_row_linear(input_.contiguous(), lin.weight, handle)
        return (y, None) if lin.return_bias else y

    lin.forward = forward


def fuse_row_parallel(model, vllm_config):
    """Route every decoder layer's o_proj and down_proj through one shared TPRowLinear (the GEMM's
    epilogue reduce-scatters over NVLink; no NCCL all-reduce). Needs TP > 1 and eager execution:
    the host-side call counter that pairs the ranks' buffers would be frozen by a CUDA graph.
    Returns the number of linears routed."""
    tp_size = get_tensor_model_parallel_world_size()
    if tp_size == 1 or not fused_tp_wanted(vllm_config):
        return 0
    if not getattr(vllm_config.model_config, "enforce_eager", False):
        logger.warning("[micro_engram] micro_engram_fused_tp needs enforce_eager=True (CUDA graphs would freeze "
                       "its call counter); vLLM's all-reduce is kept")
        return 0
    from micro_engram_fork_b200.ops.registry import add_tp_linear
    from micro_engram_fork_b200.parallel.tp_linear import TPRowLinear

    rows = vllm_config.scheduler_config.max_num_batched_tokens
    lins = []
    for layer in model.model.layers:
        if isinstance(layer, PPMissingLayer):
            continue
        pair = (getattr(getattr(layer, "self_attn", None), "o_proj", None),
                getattr(getattr(layer, "mlp", None), "down_proj", None))
        lins += [lin for lin in pair if lin is not None and _fusable(lin)]
    if not lins:
        return 0
    n_out = {lin.weight.shape[0] for lin in lins}
    if len(n_out) != 1:
        raise ValueError(f"[micro_engram] micro_engram_fused_tp: row-parallel outputs differ {sorted(n_out)}")
    shared = TPRowLinear(rows, n_out.pop(), lins[0].weight.device, group=get_tp_group().cpu_group)
    handle = add_tp_linear(shared)
    model.__dict__["micro_engram_tp_linear"] = shared
    for lin in lins:
        _route_row_parallel(lin, handle, rows)
    logger.info("[micro_engram] %d row-parallel linears fused with their all-reduce (GEMM epilogue "
                "reduce-scatter over NVLink, %d rows max)", len(lins), rows)
    return len(lins)


def _dummy_rows(engram, seed):
    """load_format="dummy" (random weights for benchmarking) never calls load_weights, so the
    row shards, allocated empty, get N(0, 0.02) rows here instead of whatever memory held."""
    with torch.no_grad():
        for shard in engram.row_shards:
            g = torch.Generator(device=shard.device).manual_seed(seed)
            shard.copy_(torch.randn(shard.shape, generator=g, device=shard.device).to(shard.dtype) * 0.02)


# ============================================================================ the layer
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


# ============================================================================ weights
class _EngramTensors:
    """Routes a checkpoint stream: base tensors on to vLLM's loader, engram tensors aside by
    layer (checkpoint names, with or without activation-checkpoint wrappers)."""

    WRAPPED = "._checkpoint_wrapped_module."

    def __init__(self):
        self.by_layer = {}

    def base_only(self, weights):
        for name, tensor in weights:
            name = name.replace(self.WRAPPED, ".")
            if ".micro_engram." in name:
                self.by_layer.setdefault(layer_of_key(name), {})[_local_name(name)] = tensor
            else:
                yield name, tensor

    def count(self):
        return sum(len(v) for v in self.by_layer.values())


def _with_canon(spec, sd):
    """A merged-token engram needs its canon map: from the weights, else the run's canon file."""
    if "canon" in sd or not spec.get("token_merge"):
        return sd
    canon_path = spec.get("canon_path")
    if not canon_path or not os.path.isfile(canon_path):
        raise ValueError("[micro_engram] this engram merges tokens but its weights carry no 'canon' and the canon "
                         f"file is missing ({canon_path})")
    sd["canon"] = torch.load(canon_path, map_location="cpu")
    return sd


# ============================================================================ the models
class EngramGemma4ForCausalLM(Gemma4ForCausalLM):
    def __init__(self, *, vllm_config: VllmConfig, prefix: str = ""):
        super().__init__(vllm_config=vllm_config, prefix=prefix)
        fuse_row_parallel(self, vllm_config)
        self.micro_engram_slots = []
        self.micro_engram_separate = False
        self.micro_engram_conf = None
        self._micro_engram_ids = None
        self._engram_files_loaded = False
        self._engram_tables_loaded = {}
        sel = select_engram(vllm_config.additional_config, vllm_config.model_config.model)
        if sel is None:
            logger.info("[micro_engram] no engram configured: plain Gemma 4")
            return
        self._check_serving(vllm_config, sel)
        self.micro_engram_separate, self.micro_engram_conf = sel.separate, sel.conf
        specs = engram_specs(sel.conf, sel.path)
        history_width = max(max(s["orders"]) for s in specs)
        for spec in specs:
            layer = self.model.layers[spec["layer"]]
            if isinstance(layer, PPMissingLayer):
                continue  # pipeline parallel: another rank holds this layer
            self._attach(vllm_config, spec, layer, history_width, sel.separate)

    def _check_serving(self, vllm_config, sel):
        note = base_mismatch(sel.conf, vllm_config.model_config.model)
        if note:
            logger.warning("[micro_engram] %s", note)
        arch = vllm_config.model_config.architecture
        if arch not in SUPPORTED_ARCHS:
            raise ValueError(f"[micro_engram] {arch} is not supported (its layers would never see the engram "
                             f"history); serve one of {', '.join(SUPPORTED_ARCHS)}")
        if not runner_is_v2(vllm_config):
            raise ValueError("[micro_engram] vLLM's Model Runner V2 is required (it fills the engram history before "
                             "each step); set VLLM_USE_V2_MODEL_RUNNER=1 (set automatically when the plugin loads "
                             "with MICRO_ENGRAM_CONFIG)")

    def _attach(self, vllm_config, spec, layer, history_width, separate):
        text_cfg = getattr(self.config, "text_config", self.config)
        tp_rank, tp_size = get_tensor_model_parallel_rank(), get_tensor_model_parallel_world_size()
        engram = engram_from_spec(spec, text_cfg.hidden_size, text_cfg.vocab_size,
                                  getattr(text_cfg, "pad_token_id", None) or 0, build_tables=False)
        ref = next(layer.parameters())
        engram.to(device=ref.device, dtype=ref.dtype)
        offload = _offload_rows(vllm_config)
        if offload:
            engram.shard_rows(tp_rank, tp_size, device="cpu", dtype=ref.dtype, requires_grad=False, empty=True,
                              pin_memory=True)
            engram.__dict__["row_views"] = _uva_views(engram.row_shards)
            engram.row_lookup_fn = tp_lookup(tensor_model_parallel_all_reduce)
        else:  # rows in a row store mapped across the TP group: the fused op reads owners' rows directly
            group = get_tp_group().cpu_group if tp_size > 1 else None
            engram.shard_rows(tp_rank, tp_size, device=ref.device, dtype=ref.dtype, requires_grad=False,
                              empty=True, group=group)
        if getattr(getattr(vllm_config, "load_config", None), "load_format", None) == "dummy":
            _dummy_rows(engram, spec["seed"] * 1_000_003 + tp_rank)
        layer.add_module("micro_engram", engram)
        if self._micro_engram_ids is None:
            rows = vllm_config.scheduler_config.max_num_batched_tokens
            self._micro_engram_ids = torch.full((rows, history_width), -1, dtype=torch.int32, device=ref.device)
        layer.register_buffer("micro_engram_ids", self._micro_engram_ids, persistent=False)
        layer.micro_engram_on = os.environ.get("MICRO_ENGRAM_OFF", "0") != "1"
        layer.micro_engram_media = None
        layer.__class__ = EngramGemma4DecoderLayer
        self.micro_engram_slots.append((spec, layer))
        gib = sum(p.numel() * p.element_size() for p in engram.row_shards) / 2 ** 30
        logger.info("[micro_engram] layer %d: %s gate, %d tables x %d dims, rows per order %s; this rank holds 1/%d "
                    "(%.2f GiB, %s), seed %d%s; weights from %s", spec["layer"], engram.gate, len(engram.row_shards),
                    engram.engram_dim, engram.order_sizes, tp_size, gib,
                    "pinned host memory" if offload else "peer-mapped row store", spec["seed"],
                    "" if layer.micro_engram_on else " (OFF: MICRO_ENGRAM_OFF=1)",
                    spec["weights"] if separate else "the model checkpoint")

    @property
    def micro_engram_ids(self):
        return self._micro_engram_ids

    def get_model_state_cls(self):
        from .model_state import EngramModelState

        return EngramModelState

    # ------------------------------------------------------------------ weights
    def load_weights(self, weights):
        if not self.micro_engram_slots:
            return super().load_weights(weights)
        aside = _EngramTensors()
        loaded = super().load_weights(aside.base_only(weights))
        if self.micro_engram_separate:
            if aside.count():
                logger.warning("[micro_engram] the checkpoint carries an engram of its own (%d tensors); the "
                               "configured engram weights are used instead", aside.count())
            if not self._engram_files_loaded:  # vLLM may call load_weights once per run of names
                self._engram_files_loaded = True
                for spec, layer in self.micro_engram_slots:
                    loaded |= self._load_from_files(spec, layer)
            return loaded
        for spec, layer in self.micro_engram_slots:
            loaded |= self._load_from_stream(spec, layer, aside.by_layer.get(spec["layer"]))
        return loaded

    def _param_names(self, engram, only=None):
        owner = next(n for n, m in self.named_modules() if m is engram)
        return {f"{owner}.{n}" for n, _ in engram.named_parameters() if only is None or n in only}

    def _load_from_stream(self, spec, layer, part):
        """Engram tensors that arrived with the checkpoint (an assembled model; possibly over
        several load_weights calls)."""
        if not part:
            return set()
        engram = layer.micro_engram
        tables = self._engram_tables_loaded.setdefault(spec["layer"], set())
        tables |= load_rows(engram, part, f"the checkpoint (layer {spec['layer']})", complete=False)
        logger.info("[micro_engram] layer %d: %d of %d tables loaded", spec["layer"], len(tables),
                    len(engram.row_shards))
        return self._param_names(engram, part)

    def _load_from_files(self, spec, layer):
        engram = layer.micro_engram
        shared_file = sum(s["weights"] == spec["weights"] for s, _ in self.micro_engram_slots) > 1
        sd = load_engram_weights(spec["weights"], layer=spec["layer"], need_layer=shared_file)
        if not any(k.startswith("tables.") for k in sd):
            raise ValueError(f"[micro_engram] {spec['weights']} holds no engram tables for layer {spec['layer']}")
        load_rows(engram, _with_canon(spec, sd), spec["weights"])
        logger.info("[micro_engram] layer %d: %d engram tensors from %s", spec["layer"], len(sd), spec["weights"])
        return self._param_names(engram)


class EngramGemma4ForConditionalGeneration(Gemma4ForConditionalGeneration):
    """Multimodal Gemma 4: its language model comes from the registry (so it is
    EngramGemma4ForCausalLM); this wrapper exposes the history buffer and the model state, and
    keeps the engram off media placeholder ids (no memory on them; treated as missing history)."""

    def __init__(self, *, vllm_config: VllmConfig, prefix: str = ""):
        super().__init__(vllm_config=vllm_config, prefix=prefix)
        slots = getattr(self.language_model, "micro_engram_slots", None)
        if not slots:
            return
        media = sorted({int(t) for t in (getattr(self.config, f, None) for f in MEDIA_TOKEN_FIELDS) if t is not None})
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
