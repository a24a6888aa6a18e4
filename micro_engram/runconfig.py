"""Which engrams a run trains, how each one is built and attached, and the run's
micro_engram_config.json.

A run asks for one main engram (the micro_engram_* keys) and any number of extra ones
(micro_engram_extra). Each request becomes an `EngramRequest`; `build_slot` turns it into a
live engram attached to its decoder layer, either fresh or rebuilt from trained weights
(init_from), and returns a `Slot`. `run_config` renders the JSON every loader reads.

The JSON layout, the inheritance rules of extra engrams and the init_from precedence are the
public contract of Ready-Art/micro_engram_fork (micro_engram/runconfig.py:1-259):
  * the first engram's settings are repeated at the top level (older loaders read only those),
    and every engram is listed under "engrams" with its own "weights";
  * a frozen engram's "weights" is the file it was loaded from; a trained one's is where this
    run writes it;
  * an extra engram without table sizes inherits the main engram's (unless it sets its own
    single table_size), and dim / heads / gate fall back to the main engram's;
  * with init_from, the trained engram's architecture (sizes, gate, seed, ...) wins over the YAML.
"""
import json
import logging
import os
from collections.abc import Mapping
from dataclasses import dataclass

import torch

from .module import attach_engram, check_loaded, engram_from_spec, resolve_order_sizes
from .weights import (CONFIG_NAME, base_fingerprint, default_seed, load_engram_weights, norm_table_sizes,
                      resolve_engram_source)

LOG = logging.getLogger(__package__)

__all__ = ["CONFIG_NAME", "EngramRequest", "Slot", "run_config", "build_config", "write_config", "check_canon",
           "epoch_step_scheduler", "engram_requests", "build_slot", "engram_params", "fingerprint_or_none"]

# settings that define an engram's shape and hashing: a trained engram's values win
ARCH_FIELDS = ("table_size", "table_sizes", "engram_dim", "num_heads", "orders", "gate", "seed")


@dataclass
class EngramRequest:
    """One engram the config asks for. `spec` is the JSON form (keys starting with "_" stay
    private); init_from / frozen say where it starts and whether it trains."""
    spec: dict
    init_from: str | None = None
    frozen: bool = False

    @property
    def layer(self):
        return self.spec["layer"]


@dataclass
class Slot:
    """A built engram of the run."""
    spec: dict
    engram: torch.nn.Module
    frozen: bool = False
    source: str | None = None   # absolute path of the weights it was built from (init_from)
    where: str | None = None    # module name of the decoder layer it is attached to

    @property
    def layer(self):
        return self.spec["layer"]

    def file_name(self, step=None):
        """The .pt name of this engram: the main one keeps the historical name."""
        stem = "micro_engram" if self.spec.get("_main") else f"micro_engram_L{self.layer}"
        return stem + (f"-step{step}" if step is not None else "") + ".pt"


# ------------------------------------------------------------------------- config JSON
def _public(spec):
    return {k: v for k, v in spec.items() if not k.startswith("_")}


def run_config(base, slots, weights_for):
    """The micro_engram_config.json mapping. `weights_for(slot)` is where a trained engram's
    tensors live relative to the file's folder (None: inside a model checkpoint there)."""
    listed = [dict(_public(s.spec), weights=(s.source if s.frozen else weights_for(s))) for s in slots]
    head = listed[0]
    conf = dict(base)
    conf.update({k: v for k, v in head.items() if k != "weights"})
    conf["engrams"] = listed
    if head["weights"]:
        conf["weights"] = head["weights"]
    return conf


build_config = run_config  # the name the trainer and tools use


def write_config(conf, folder, weights=None):
    """Write `conf` as folder/micro_engram_config.json (`weights`: the single-engram form's
    top-level weights path)."""
    os.makedirs(folder, exist_ok=True)
    if weights:
        conf = {**conf, "weights": weights}
    path = os.path.join(folder, CONFIG_NAME)
    with open(path, "w") as f:
        json.dump(conf, f, indent=2)
    LOG.info(f"[micro_engram] wrote {path}")


# ------------------------------------------------------------------------- small helpers
def engram_params(engram):
    """All trainable tensors of an engram, its row shards included."""
    every = getattr(engram, "all_parameters", None)
    return every() if every is not None else list(engram.parameters())


def fingerprint_or_none(path):
    """The base weights' fingerprint, or None (a folder without safetensors, or any failure:
    a fingerprint is advisory and never stops a run)."""
    if not path or not os.path.isdir(path):
        return None
    try:
        return base_fingerprint(path)
    except Exception as e:  # noqa: BLE001
        LOG.warning(f"[micro_engram] base fingerprint unavailable: {e}")
        return None


def check_canon(canon, vocab_size):
    """Validate a token-merge map read from disk: a 1-D id tensor over the whole vocabulary
    whose canonical ids map to themselves."""
    ok = torch.is_tensor(canon) and canon.dim() == 1 and canon.numel() == vocab_size
    if not ok:
        raise ValueError(f"[micro_engram] the canon file must hold one id per vocabulary entry ({vocab_size})")
    canon = canon.long()
    if bool((canon < 0).any()) or bool((canon >= vocab_size).any()):
        raise ValueError("[micro_engram] the canon map points outside the vocabulary")
    if not bool((canon[canon] == canon).all()):
        raise ValueError("[micro_engram] the canon map is not idempotent: a canonical id must map to itself")
    return canon


def epoch_step_scheduler(optimizer, num_training_steps, warmup_steps, epochs, factor):
    """LambdaLR: linear warmup from 0, then the LR times factor**(completed epochs), with an
    epoch measured in optimizer steps."""
    from torch.optim.lr_scheduler import LambdaLR

    steps_per_epoch = max(1, round(num_training_steps / max(epochs, 1e-9)))
    warm = int(warmup_steps or 0)

    def factor_at(step):
        return step / warm if step < warm else factor ** (step // steps_per_epoch)

    LOG.warning(f"[micro_engram] LR: {warm} warmup steps, then x{factor} every {steps_per_epoch} steps "
                f"(at {list(range(steps_per_epoch, num_training_steps, steps_per_epoch))})")
    return LambdaLR(optimizer, factor_at)


# ------------------------------------------------------------------------- requests
def _mapping(entry):
    if isinstance(entry, Mapping):
        return dict(entry)
    dump = getattr(entry, "model_dump", None)
    return dump() if callable(dump) else dict(vars(entry))


def _main_request(cfg):
    spec = dict(layer=cfg.micro_engram_layer, table_size=cfg.micro_engram_table_size,
                table_sizes=norm_table_sizes(cfg.micro_engram_table_sizes), engram_dim=cfg.micro_engram_dim,
                num_heads=cfg.micro_engram_heads, gate=cfg.micro_engram_gate, seed=cfg.micro_engram_seed, _main=True)
    return EngramRequest(spec, cfg.micro_engram_init_from, bool(cfg.micro_engram_frozen))


def _extra_request(entry, main):
    e = _mapping(entry)
    if e.get("table_sizes"):
        sizes = norm_table_sizes(e["table_sizes"])
    elif e.get("table_size"):
        sizes = None          # its own single size for every order
    else:
        sizes = main["table_sizes"]
    spec = dict(layer=int(e["layer"]), table_size=e.get("table_size") or main["table_size"], table_sizes=sizes,
                engram_dim=e.get("dim") or main["engram_dim"], num_heads=e.get("heads") or main["num_heads"],
                gate=e.get("gate") or main["gate"], seed=e.get("seed"))
    return EngramRequest(spec, e.get("init_from"), bool(e.get("frozen")))


def engram_requests(cfg):
    """[EngramRequest] for the main engram and each micro_engram_extra entry, validated: one
    engram per layer, no frozen engram without trained weights, a default seed per layer."""
    main = _main_request(cfg)
    reqs = [main] + [_extra_request(e, main.spec) for e in (cfg.micro_engram_extra or [])]
    seen = set()
    for r in reqs:
        if r.layer in seen:
            raise ValueError(f"[micro_engram] layer {r.layer} has two engrams; each layer takes at most one")
        seen.add(r.layer)
        if r.frozen and not r.init_from:
            raise ValueError(f"[micro_engram] layer {r.layer}: frozen needs init_from (an untrained frozen engram "
                             "would only add its zero-initialised output)")
        if r.spec["seed"] is None:
            r.spec["seed"] = default_seed(r.layer)
    return reqs


# ------------------------------------------------------------------------- building
def _same(a, b):
    if isinstance(a, dict) or isinstance(b, dict):
        return norm_table_sizes(a) == norm_table_sizes(b)
    if isinstance(a, (list, tuple)) and isinstance(b, (list, tuple)):
        return tuple(a) == tuple(b)
    return a == b


def _adopt_trained_spec(spec, trained):
    """The trained engram's architecture replaces the YAML's (with one warning listing what
    changed)."""
    diff = [f"{k} {spec[k]} -> {trained[k]}" for k in ARCH_FIELDS
            if spec.get(k) is not None and trained.get(k) is not None and not _same(spec[k], trained[k])]
    if diff:
        LOG.warning(f"[micro_engram] layer {spec['layer']}: the trained engram's settings replace the YAML's: "
                    + ", ".join(diff))
    for k in ARCH_FIELDS:
        if trained.get(k) is not None:
            spec[k] = trained[k]
    spec["table_sizes"] = norm_table_sizes(trained.get("table_sizes"))


def _spec_from_tensors(spec, sd, source):
    """Bare weights without a config: table shapes give sizes and dim; the gate kind follows
    from which tensors exist; heads and orders come from the YAML and must fit the count."""
    n_tables = sum(1 for k in sd if k.startswith("tables."))
    rows = [int(sd[f"tables.{i}.weight"].shape[0]) for i in range(n_tables)]
    first = sd["tables.0.weight"]
    spec["table_size"], spec["engram_dim"] = int(first.shape[0]), int(first.shape[1])
    orders = list(resolve_order_sizes(spec["table_size"], spec.get("orders") or (2, 3), spec.get("table_sizes")))
    heads = spec["num_heads"]
    if heads * len(orders) != n_tables:
        raise ValueError(f"[micro_engram] {source} holds {n_tables} tables, which is not {heads} heads x "
                         f"{len(orders)} orders {orders}; set the table sizes of these weights")
    spec["orders"] = orders
    spec["table_sizes"] = {n: rows[i * heads] for i, n in enumerate(orders)}
    if "up.weight" in sd:
        spec["gate"] = "ple"
    else:
        spec["gate"] = "scalar_sqrt" if "q_scale" in sd else "scalar"


def _load_trained(spec, init_from):
    """(absolute source path, state dict) of a trained engram; `spec` is updated to match it."""
    source, trained = resolve_engram_source(init_from, spec["layer"])
    source = os.path.abspath(source)
    if trained is not None:
        _adopt_trained_spec(spec, trained)
    sd = load_engram_weights(source, layer=spec["layer"])
    if not any(k.startswith("tables.") for k in sd):
        raise ValueError(f"[micro_engram] {source} has no engram tables for layer {spec['layer']}")
    if trained is None:
        _spec_from_tensors(spec, sd, source)
    return source, sd


def _check_trained_canon(spec, sd, canon):
    if "canon" in sd:
        if canon is not None and not torch.equal(sd["canon"].long(), canon):
            LOG.warning(f"[micro_engram] layer {spec['layer']} keeps the token-merge map it was trained with "
                        "(it differs from micro_engram_canon_path)")
    elif canon is None and spec.get("token_merge"):
        raise ValueError(f"[micro_engram] layer {spec['layer']} was trained with merged tokens but its weights carry "
                         "no canon map; set micro_engram_canon_path")


def build_slot(request, model, text_cfg, canon, dtype=None, sharding=None, get_ids=None, device=None, group=None,
               row_capacity=None):
    """Build the requested engram (fresh or from init_from), row-shard its tables when asked,
    and attach it to its decoder layer."""
    spec, frozen = request.spec, request.frozen
    source = sd = None
    if request.init_from:
        source, sd = _load_trained(spec, request.init_from)
    engram = engram_from_spec(spec, text_cfg.hidden_size, text_cfg.vocab_size, text_cfg.pad_token_id or 0, canon,
                              build_tables=not (sharding and sd is None))
    if sd is not None:
        _check_trained_canon(spec, sd, canon)
        check_loaded(engram, sd, source)
        LOG.warning(f"[micro_engram] layer {spec['layer']}: starts from {source} "
                    + ("(frozen)" if frozen else "(continues training)"))
    spec.update(orders=list(engram.orders), table_sizes=dict(engram.order_sizes), table_size=engram.table_size,
                pad_id=engram.pad_id, token_merge=not torch.equal(engram.canon, torch.arange(engram.canon.numel())),
                frozen=frozen, init_from=source)
    dt = {"fp32": torch.float32, "bf16": torch.bfloat16}.get(dtype)
    if sharding:
        _shard_tables(engram, model, spec["layer"], dt, not frozen, device, group, row_capacity)
    where, _ = attach_engram(model, engram, spec["layer"], dtype=dt, get_ids=get_ids)
    count = sum(p.numel() for p in engram_params(engram))
    LOG.warning(f"[micro_engram] {where}: {count / 1e6:.1f}M engram parameters, {spec['gate']} gate, seed "
                f"{spec['seed']}" + (", frozen" if frozen else ""))
    return Slot(spec=spec, engram=engram, frozen=frozen, source=source, where=where)


def _shard_tables(engram, model, layer, dtype, trainable, device, group, row_capacity):
    from .module import find_text_layers, layer_device_dtype
    from .rows import dist_rank_world

    rank, world = dist_rank_world()
    if device is None:
        device = (torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0))) if torch.cuda.is_available()
                  else torch.device("cpu"))
    if dtype is None:
        dtype = layer_device_dtype(find_text_layers(model)[1][layer])[1]
    engram.shard_rows(rank, world, device=device, dtype=dtype, requires_grad=trainable, group=group,
                      row_capacity=row_capacity)
