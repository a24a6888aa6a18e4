"""Reading engram weights from any of the places they are saved, the engram specs of a run
config, checkpoint discovery, and the base-model fingerprint.

Sources (the formats of Ready-Art/micro_engram_fork, micro_engram/weights.py:1-328):
  * a `.pt` file, with full module names (...layers.3.micro_engram.tables.0.weight) or names
    local to the engram (tables.0.weight);
  * a `.safetensors` file, or a folder of them (a merged or assembled model);
  * a DCP folder (`.metadata` inside: checkpoint-N/micro_engram_rows or an FSDP checkpoint).
Each is wrapped in a small reader class with `names()` and `read(names)`; everything above it
(layer filtering, local names) is format-independent. Only engram tensors are ever read.
"""
import glob
import hashlib
import json
import os
import re

import torch

TAG = "micro_engram."
CONFIG_NAME = "micro_engram_config.json"
SEED_STRIDE = 10007  # an engram's default hash seed is 10007 x its layer index

LAYER_IN_KEY = re.compile(r"(?:^|\.)layers\.(\d+)\.(?:_checkpoint_wrapped_module\.)?micro_engram\.")
CHECKPOINT_DIR = re.compile(r"checkpoint-(\d+)$")
SPEC_FIELDS = ("layer", "table_size", "table_sizes", "engram_dim", "num_heads", "orders", "gate", "seed",
               "pad_id", "token_merge", "canon_path", "frozen", "init_from")


# ------------------------------------------------------------------------- names
def _local_name(key):
    """The name inside the engram ('tables.0.weight') of a full or local key; None when the
    key is not an engram tensor."""
    head, sep, tail = key.partition("." + TAG)
    if sep:
        return tail
    return key[len(TAG):] if key.startswith(TAG) else None


def layer_of_key(key):
    """Decoder layer index carried by an engram key, or None."""
    hit = LAYER_IN_KEY.search(key)
    return int(hit.group(1)) if hit else None


def _belongs(key, layer):
    """An engram key of `layer` (keys without a layer number belong to every layer)."""
    if _local_name(key) is None:
        return False
    own = layer_of_key(key)
    return layer is None or own is None or own == layer


# ------------------------------------------------------------------------- readers
class _PtReader:
    def __init__(self, path):
        def flat(d, prefix=""):
            for k, v in d.items():
                if isinstance(v, dict):
                    yield from flat(v, f"{prefix}{k}.")
                else:
                    yield f"{prefix}{k}", v

        self.items = dict(flat(torch.load(path, map_location="cpu", weights_only=True)))

    def names(self):
        return [k for k, v in self.items.items() if torch.is_tensor(v)]

    def read(self, names):
        return {k: self.items[k] for k in names}


class _SafetensorsReader:
    def __init__(self, files):
        from safetensors import safe_open

        self.where = {}
        for f in files:
            with safe_open(f, framework="pt", device="cpu") as fh:
                for k in fh.keys():
                    self.where[k] = f

    def names(self):
        return list(self.where)

    def read(self, names):
        from safetensors import safe_open

        out = {}
        for f in sorted({self.where[k] for k in names}):
            with safe_open(f, framework="pt", device="cpu") as fh:
                for k in names:
                    if self.where[k] == f:
                        out[k] = fh.get_tensor(k)
        return out


class _DcpReader:
    def __init__(self, folder):
        import torch.distributed.checkpoint as dcp
        from torch.distributed.checkpoint.metadata import TensorStorageMetadata

        self.reader = dcp.FileSystemReader(folder)
        meta = self.reader.read_metadata().state_dict_metadata
        self.meta = {k: m for k, m in meta.items() if isinstance(m, TensorStorageMetadata)}

    def names(self):
        return list(self.meta)

    def read(self, names):
        import torch.distributed.checkpoint as dcp

        out = {k: torch.empty(tuple(self.meta[k].size), dtype=self.meta[k].properties.dtype) for k in names}
        if out:
            dcp.load(out, storage_reader=self.reader, no_dist=True)  # each process reads on its own
        return out


def _is_dcp(path):
    return os.path.isdir(path) and os.path.isfile(os.path.join(path, ".metadata"))


def _reader(path):
    if _is_dcp(path):
        return _DcpReader(path)
    if os.path.isdir(path):
        return _SafetensorsReader(sorted(glob.glob(os.path.join(path, "*.safetensors"))))
    if path.endswith(".safetensors"):
        return _SafetensorsReader([path])
    return _PtReader(path)


# ------------------------------------------------------------------------- loading
def engram_layers_in(path):
    """Layer indices of the engram tensors stored at `path` (empty when names carry none)."""
    names = _reader(os.path.abspath(path)).names()
    return sorted({layer_of_key(k) for k in names if _local_name(k) is not None} - {None})


def load_engram_weights(path, layer=None, need_layer=False):
    """{local name: tensor} of the engram stored at `path` (only layer `layer`'s when the names
    carry layers). A file whose tensors are already local (no engram prefix) is returned whole;
    with need_layer such a file is refused when several engrams would share it."""
    path = os.path.abspath(path)
    src = _reader(path)
    names = src.names()
    mine = [k for k in names if _belongs(k, layer)]
    if mine:
        return {_local_name(k): t for k, t in src.read(mine).items()}
    if _is_dcp(path) or os.path.isdir(path):
        return {}
    local = src.read(names)  # bare tensors named tables.0.weight, key.weight, ...
    if need_layer and layer is not None and any(k.startswith("tables.") for k in local):
        raise ValueError(f"[micro_engram] several engrams use {path}, but its tensor names carry no layer "
                         f"(e.g. {next(iter(local))}), so layer {layer}'s tensors cannot be told apart; give each "
                         f"engram its own file or keep full names (...layers.{layer}.micro_engram.tables.0.weight)")
    return local


# ------------------------------------------------------------------------- configs and specs
def resolve_weights_path(conf, conf_path):
    """A config's "weights" entry, relative paths taken from the config's folder; or None."""
    w = conf.get("weights")
    if not w:
        return None
    return w if os.path.isabs(w) else os.path.join(os.path.dirname(os.path.abspath(conf_path)), w)


def norm_table_sizes(sizes):
    """{int order: int rows or None}; None when no per-order sizes are given."""
    if not sizes:
        return None
    return {int(order): (int(rows) if rows else None) for order, rows in dict(sizes).items()}


def default_seed(layer):
    return SEED_STRIDE * int(layer)


def _entry_spec(top, entry, conf_path):
    spec = dict(top)
    spec.update({k: v for k, v in entry.items() if v is not None or k == "weights"})
    spec["layer"] = int(spec.get("layer") or 0)
    spec["orders"] = tuple(spec.get("orders") or (2, 3))
    spec["table_sizes"] = norm_table_sizes(spec.get("table_sizes"))
    spec["gate"] = spec.get("gate") or "scalar"
    spec["seed"] = int(spec["seed"]) if spec.get("seed") is not None else 0  # configs older than recorded seeds
    w = entry.get("weights")
    if w and conf_path and not os.path.isabs(w):
        w = os.path.join(os.path.dirname(os.path.abspath(conf_path)), w)
    spec["weights"] = w or None
    return spec


def engram_specs(conf, conf_path=None):
    """One spec per engram of a micro_engram_config.json: its "engrams" list, or the older
    single-engram form at the top level."""
    top = {k: conf.get(k) for k in SPEC_FIELDS}
    entries = conf.get("engrams") or [dict(top, weights=conf.get("weights"))]
    specs = [_entry_spec(top, e, conf_path) for e in entries]
    layers = [s["layer"] for s in specs]
    if len(layers) != len(set(layers)):
        raise ValueError(f"[micro_engram] the config lists two engrams for one layer: {layers}")
    return specs


def latest_checkpoint(folder):
    """The newest complete checkpoint-N under `folder` (complete = its trainer_state.json, which
    is written last, exists), or None."""
    best = None
    for c in glob.glob(os.path.join(folder, "checkpoint-*")):
        hit = CHECKPOINT_DIR.search(c)
        if hit and os.path.isfile(os.path.join(c, "trainer_state.json")):
            if best is None or int(hit.group(1)) > best[0]:
                best = (int(hit.group(1)), c)
    return best[1] if best else None


def _spec_of_layer(conf_path, layer):
    with open(conf_path) as f:
        specs = engram_specs(json.load(f), conf_path)
    hit = [s for s in specs if s["layer"] == layer]
    if not hit:
        raise ValueError(f"[micro_engram] {conf_path} has no engram at layer {layer} "
                         f"(layers: {[s['layer'] for s in specs]})")
    return hit[0]


def resolve_engram_source(path, layer):
    """(weights path, spec or None) of the trained engram for decoder `layer`. `path` may be a
    micro_engram_config.json, a folder holding one (a checkpoint, an assembled model, or an
    output_dir, which means its newest complete checkpoint), or the weights themselves."""
    path = os.path.abspath(path)
    conf_path = path if path.endswith(".json") else os.path.join(path, CONFIG_NAME)
    is_plain_dir = os.path.isdir(path) and not _is_dcp(path)
    if is_plain_dir and not glob.glob(os.path.join(path, "*.safetensors")):
        ckpt = latest_checkpoint(path)
        if ckpt is not None:
            weights, spec = resolve_engram_source(ckpt, layer)
            if spec is None and os.path.isfile(conf_path):
                spec = _spec_of_layer(conf_path, layer)
            return weights, spec
    if os.path.isfile(conf_path):
        spec = _spec_of_layer(conf_path, layer)
        return (spec["weights"] or os.path.dirname(conf_path)), spec
    return path, None


# ------------------------------------------------------------------------- base fingerprint
# The fingerprint is a stored format: configs written by either framework carry it, so its
# steps are fixed (the first 64 rows of the embedding and of every q/k/v/o and gate/up/down
# projection of the first, middle and last text layer, each hashed as role name, (dtype,
# shape) text and raw bytes, roles in sorted order; sha256, 16 hex digits).
PROJ_KEY = re.compile(r"^(.*\.layers\.)(\d+)\.(self_attn\.[qkvo]_proj|mlp\.(?:gate|up|down)_proj)\.weight$")
FINGERPRINT_ROWS = 64


def _tensor_files(model_dir):
    """{tensor name: file} of a safetensors model folder (index file when present)."""
    index = os.path.join(model_dir, "model.safetensors.index.json")
    if os.path.isfile(index):
        with open(index) as f:
            return {k: os.path.join(model_dir, v) for k, v in json.load(f)["weight_map"].items()}
    return _SafetensorsReader(sorted(glob.glob(os.path.join(model_dir, "*.safetensors")))).where


def _fingerprint_roles(names):
    roles = {"embed": k for k in names if k.endswith("embed_tokens.weight")}
    layers = {}
    for k in names:
        hit = PROJ_KEY.match(k)
        if hit:
            layers.setdefault(int(hit.group(2)), {})[hit.group(3)] = k
    if layers:
        idx = sorted(layers)
        for label, i in (("first", idx[0]), ("middle", idx[len(idx) // 2]), ("last", idx[-1])):
            for role, k in layers[i].items():
                roles[f"{label}.{role}"] = k
    return roles


def base_fingerprint(model_dir):
    """16-hex-digit fingerprint of a base model folder's text weights (None without any)."""
    from safetensors import safe_open

    if not os.path.isdir(model_dir):
        return None
    files = {k: f for k, f in _tensor_files(model_dir).items()
             if TAG not in k and "vision" not in k and "audio" not in k}
    roles = _fingerprint_roles(list(files))
    if not roles:
        return None
    digest = hashlib.sha256()
    for role in sorted(roles):
        name = roles[role]
        with safe_open(files[name], framework="pt", device="cpu") as fh:
            rows = fh.get_slice(name)[:FINGERPRINT_ROWS].contiguous().cpu()
        digest.update(role.encode())
        digest.update(str((rows.dtype, tuple(rows.shape))).encode())
        digest.update(rows.view(torch.uint8).numpy().tobytes())
    return digest.hexdigest()[:16]


def base_mismatch(conf, model_dir):
    """A warning when the engram's config records other base weights than `model_dir`'s."""
    want = conf.get("base_fingerprint")
    if not want:
        return None
    try:
        have = base_fingerprint(model_dir)
    except Exception as e:  # noqa: BLE001 - advisory only
        return f"the base weights this engram was trained on could not be checked ({type(e).__name__}: {e})"
    if have in (None, want):
        return None
    return (f"this engram was trained on other base weights (recorded base {conf.get('base_model', '?')}, "
            f"fingerprint {want}; this model's is {have}); it loads, but it will inject into hidden states it "
            f"was not trained on, so expect worse output unless the bases really are the same")
