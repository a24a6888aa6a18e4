"""Engram weights from wherever they were saved, keyed by their name inside the engram
(tables.0.weight, key.weight, canon, ...), plus the engram specs of a run config, checkpoint
discovery and the base-model fingerprint.

Formats (micro_engram/weights.py:1-328 of the reference): a `.pt` with local or full names,
a `.safetensors` file or folder (merged / assembled model), and a DCP folder (checkpoint-N/
micro_engram_rows or an FSDP checkpoint), from which only the engram tensors are read.
"""
import glob
import hashlib
import json
import os
import re

import torch

TAG = "micro_engram."
CONFIG_NAME = "micro_engram_config.json"
SEED_STRIDE = 10007  # default seed = 10007 * layer (layer 0 -> 0)

_LAYER_RE = re.compile(r"(?:^|\.)layers\.(\d+)\.(?:_checkpoint_wrapped_module\.)?micro_engram\.")
_CKPT_RE = re.compile(r"checkpoint-(\d+)$")
_SPEC_KEYS = ("layer", "table_size", "table_sizes", "engram_dim", "num_heads", "orders", "gate", "seed",
              "pad_id", "token_merge", "canon_path", "frozen", "init_from")


def _flatten(d, prefix=""):
    flat = {}
    for k, v in d.items():
        if isinstance(v, dict):
            flat.update(_flatten(v, f"{prefix}{k}."))
        else:
            flat[f"{prefix}{k}"] = v
    return flat


def _local_name(key):
    """'...layers.0._checkpoint_wrapped_module.micro_engram.tables.0.weight' -> 'tables.0.weight';
    None for keys outside an engram."""
    marker = "." + TAG
    if marker in key:
        return key.split(marker, 1)[1]
    if key.startswith(TAG):
        return key[len(TAG):]
    return None


def layer_of_key(key):
    """The decoder layer an engram key belongs to, or None when the key has no layer."""
    m = _LAYER_RE.search(key)
    return int(m.group(1)) if m else None


def _wanted(key, layer):
    if _local_name(key) is None:
        return False
    if layer is None:
        return True
    k_layer = layer_of_key(key)
    return k_layer is None or k_layer == layer


def _from_full_keys(sd, layer=None):
    return {_local_name(k): v for k, v in sd.items() if torch.is_tensor(v) and _wanted(k, layer)}


def _load_dcp(path, layer=None):
    import torch.distributed.checkpoint as dcp
    from torch.distributed.checkpoint.metadata import TensorStorageMetadata

    reader = dcp.FileSystemReader(path)
    meta = reader.read_metadata().state_dict_metadata
    want = {k: torch.empty(tuple(m.size), dtype=m.properties.dtype) for k, m in meta.items()
            if isinstance(m, TensorStorageMetadata) and _wanted(k, layer)}
    if want:
        dcp.load(want, storage_reader=reader, no_dist=True)  # every process reads alone
    return _from_full_keys(want, layer)


def _load_safetensors(files, layer=None):
    from safetensors import safe_open

    sd = {}
    for f in files:
        with safe_open(f, framework="pt", device="cpu") as fh:
            for k in fh.keys():
                if _wanted(k, layer):
                    sd[_local_name(k)] = fh.get_tensor(k)
    return sd


def engram_layers_in(path):
    """Layer indices of the engrams stored at `path` (empty when the keys carry none)."""
    path = os.path.abspath(path)
    if os.path.isdir(path) and os.path.isfile(os.path.join(path, ".metadata")):
        import torch.distributed.checkpoint as dcp

        keys = list(dcp.FileSystemReader(path).read_metadata().state_dict_metadata)
    elif os.path.isdir(path) or path.endswith(".safetensors"):
        from safetensors import safe_open

        files = sorted(glob.glob(os.path.join(path, "*.safetensors"))) if os.path.isdir(path) else [path]
        keys = []
        for f in files:
            with safe_open(f, framework="pt", device="cpu") as fh:
                keys.extend(fh.keys())
    else:
        keys = list(_flatten(torch.load(path, map_location="cpu", weights_only=True)))
    layers = {layer_of_key(k) for k in keys if _local_name(k) is not None}
    return sorted(x for x in layers if x is not None)


def _no_layer(sd, path, layer, need_layer):
    if need_layer and layer is not None and any(k.startswith("tables.") for k in sd):
        raise ValueError(f"[micro_engram] {path} is used by several engrams, but its tensor names have no layer "
                         f"number (e.g. {next(iter(sd))}), so it can't tell which is layer {layer}'s. Give each "
                         f"engram its own file, or keep the full names (...layers.{layer}.micro_engram.tables.0.weight)")
    return sd


def load_engram_weights(path, layer=None, need_layer=False):
    """{local name: tensor} of the engram at `path` (only layer `layer`'s with full names)."""
    path = os.path.abspath(path)
    if os.path.isdir(path):
        if os.path.isfile(os.path.join(path, ".metadata")):
            return _load_dcp(path, layer)
        return _load_safetensors(sorted(glob.glob(os.path.join(path, "*.safetensors"))), layer)
    if path.endswith(".safetensors"):
        sd = _load_safetensors([path], layer)
        if not sd:
            from safetensors.torch import load_file

            sd = _no_layer(load_file(path), path, layer, need_layer)
        return sd
    flat = _flatten(torch.load(path, map_location="cpu", weights_only=True))
    full = _from_full_keys(flat, layer)
    return full or _no_layer({k: v for k, v in flat.items() if torch.is_tensor(v)}, path, layer, need_layer)


def resolve_weights_path(conf, conf_path):
    """The config's "weights" entry resolved against the config file's folder, or None."""
    w = conf.get("weights")
    if not w:
        return None
    return w if os.path.isabs(w) else os.path.join(os.path.dirname(os.path.abspath(conf_path)), w)


def norm_table_sizes(sizes):
    """{int order: rows or None}, or None for no per-order sizes."""
    if not sizes:
        return None
    return {int(k): (int(v) if v else None) for k, v in dict(sizes).items()}


def default_seed(layer):
    return SEED_STRIDE * int(layer)


def engram_specs(conf, conf_path=None):
    """One spec dict per engram of a micro_engram_config.json ("engrams" list, or the old
    single-engram top level). Missing seeds are 0 (configs from before seeds were recorded)."""
    top = {k: conf.get(k) for k in _SPEC_KEYS}
    entries = conf.get("engrams") or [{**top, "weights": conf.get("weights")}]
    specs = []
    for e in entries:
        spec = dict(top)
        spec.update({k: v for k, v in e.items() if v is not None or k == "weights"})
        spec["layer"] = int(spec.get("layer") or 0)
        spec["orders"] = tuple(spec.get("orders") or (2, 3))
        spec["table_sizes"] = norm_table_sizes(spec.get("table_sizes"))
        spec["gate"] = spec.get("gate") or "scalar"
        spec["seed"] = 0 if spec.get("seed") is None else int(spec["seed"])
        w = e.get("weights")
        if w and conf_path and not os.path.isabs(w):
            w = os.path.join(os.path.dirname(os.path.abspath(conf_path)), w)
        spec["weights"] = w or None
        specs.append(spec)
    layers = [s["layer"] for s in specs]
    if len(set(layers)) != len(layers):
        raise ValueError(f"[micro_engram] two engrams in the same layer: {layers}")
    return specs


def latest_checkpoint(folder):
    """The newest COMPLETE checkpoint-N in `folder` (trainer_state.json written last), or None."""
    done = []
    for c in glob.glob(os.path.join(folder, "checkpoint-*")):
        m = _CKPT_RE.search(c)
        if m and os.path.isfile(os.path.join(c, "trainer_state.json")):
            done.append((int(m.group(1)), c))
    return max(done)[1] if done else None


def _spec_for_layer(conf_path, layer):
    with open(conf_path) as f:
        specs = engram_specs(json.load(f), conf_path)
    for spec in specs:
        if spec["layer"] == layer:
            return spec
    raise ValueError(f"[micro_engram] {conf_path} has no engram at layer {layer} "
                     f"(it has layers {[s['layer'] for s in specs]})")


def resolve_engram_source(path, layer):
    """(weights path, spec or None) of the trained engram of decoder `layer`.

    `path`: a micro_engram_config.json, a folder holding one (checkpoint-N, assembled model,
    output_dir -> its newest checkpoint), or the weights themselves."""
    path = os.path.abspath(path)
    conf_path = path if path.endswith(".json") else os.path.join(path, CONFIG_NAME)
    if os.path.isdir(path) and not os.path.isfile(os.path.join(path, ".metadata")):
        has_conf = os.path.isfile(conf_path)
        has_weights = bool(glob.glob(os.path.join(path, "*.safetensors")))
        ckpt = None if has_weights else latest_checkpoint(path)
        if ckpt is not None:
            weights, spec = resolve_engram_source(ckpt, layer)
            if spec is None and has_conf:
                spec = _spec_for_layer(conf_path, layer)
            return weights, spec
    if os.path.isfile(conf_path):
        spec = _spec_for_layer(conf_path, layer)
        return spec["weights"] or os.path.dirname(conf_path), spec
    return path, None


# ----------------------------------------------------------------------------- base fingerprint
_FP_LAYER = re.compile(r"^(.*\.layers\.)(\d+)\.(self_attn\.[qkvo]_proj|mlp\.(?:gate|up|down)_proj)\.weight$")
_FP_ROWS = 64


def _weight_files(model_dir):
    index = os.path.join(model_dir, "model.safetensors.index.json")
    if os.path.isfile(index):
        with open(index) as f:
            return {k: os.path.join(model_dir, v) for k, v in json.load(f)["weight_map"].items()}
    from safetensors import safe_open

    files = {}
    for path in sorted(glob.glob(os.path.join(model_dir, "*.safetensors"))):
        with safe_open(path, framework="pt", device="cpu") as fh:
            for k in fh.keys():
                files[k] = path
    return files


def base_fingerprint(model_dir):
    """sha256 (16 hex chars) of the first 64 rows of the embedding and of every attention/MLP
    projection of the first, middle and last text layer, hashed by role (not by name), so
    folder names and multimodal wrappers don't change it. None without safetensors."""
    from safetensors import safe_open

    if not os.path.isdir(model_dir):
        return None
    files = {k: f for k, f in _weight_files(model_dir).items()
             if TAG not in k and "vision" not in k and "audio" not in k}
    if not files:
        return None
    roles = {"embed": k for k in files if k.endswith("embed_tokens.weight")}
    by_layer = {}
    for k in files:
        m = _FP_LAYER.match(k)
        if m:
            by_layer.setdefault(int(m.group(2)), {})[m.group(3)] = k
    if by_layer:
        ids = sorted(by_layer)
        for where, i in (("first", ids[0]), ("middle", ids[len(ids) // 2]), ("last", ids[-1])):
            roles.update({f"{where}.{r}": k for r, k in by_layer[i].items()})
    if not roles:
        return None
    h = hashlib.sha256()
    for role in sorted(roles):
        k = roles[role]
        with torch.device("cpu"), safe_open(files[k], framework="pt", device="cpu") as fh:
            t = fh.get_slice(k)[:_FP_ROWS].contiguous().cpu()
        h.update(role.encode())
        h.update(str((t.dtype, tuple(t.shape))).encode())
        h.update(t.view(torch.uint8).numpy().tobytes())
    return h.hexdigest()[:16]


def base_mismatch(conf, model_dir):
    """A warning text when the engram was trained on other base weights, else None."""
    want = conf.get("base_fingerprint")
    if not want:
        return None
    try:
        have = base_fingerprint(model_dir)
    except Exception as e:  # noqa: BLE001 - a warning check never stops loading
        return f"could not check which base weights this engram was trained on ({type(e).__name__}: {e})"
    if have is None or have == want:
        return None
    return (f"this engram was trained on different base weights (trained on {conf.get('base_model', '?')}, "
            f"fingerprint {want}; this model: {have}). It still loads, but it injects into hidden states it "
            f"never saw: expect worse output unless this is really the same base.")
