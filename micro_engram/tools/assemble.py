"""A servable model folder = base weights (symlinked, or copied) + a trained engram
(reference: assemble_engram_model.py:80-146).

    python -m micro_engram.tools.assemble --base BASE --engram ENGRAM --out OUT [--config C] [--copy] [--force]

ENGRAM: a DCP checkpoint folder (checkpoint-N/pytorch_model_fsdp_0), a folder of
.safetensors holding engram tensors, or a .pt. The engram config comes from --config, else
from next to the engram (its folder or that folder's parent), else from the base folder.

OUT gets every base file (symlinks), micro_engram.safetensors with full key names under the
base's decoder-layer prefix, model.safetensors.index.json extended with those keys, and the
engram config without "weights" (the engram now lives inside the folder).
"""
import argparse
import glob
import json
import os
import re
import shutil

from micro_engram.weights import CONFIG_NAME, base_mismatch, engram_specs, load_engram_weights

INDEX = "model.safetensors.index.json"
ENGRAM_FILE = "micro_engram.safetensors"
TAG = "micro_engram."
_LAYERS = re.compile(r"^(.*\.layers\.)(\d+)\.")


def find_config(engram, base, explicit=None):
    eng = os.path.abspath(engram)
    here = eng if os.path.isdir(eng) else os.path.dirname(eng)
    tried = ([explicit] if explicit else []) + [os.path.join(here, CONFIG_NAME),
                                                os.path.join(os.path.dirname(here), CONFIG_NAME),
                                                os.path.join(base, CONFIG_NAME)]
    for c in tried:
        if os.path.isfile(c):
            return c
    raise SystemExit(f"{CONFIG_NAME} not found (looked in {', '.join(tried)}); pass --config")


def base_weight_map(base):
    """The base's safetensors index (built from the shard headers when there is none)."""
    path = os.path.join(base, INDEX)
    if os.path.isfile(path):
        with open(path) as f:
            return json.load(f)
    from safetensors import safe_open

    files = sorted(glob.glob(os.path.join(base, "*.safetensors")))
    if not files:
        raise SystemExit(f"no safetensors weights in {base}")
    wmap = {}
    for fn in files:
        with safe_open(fn, framework="pt", device="cpu") as fh:
            for k in fh.keys():
                wmap[k] = os.path.basename(fn)
    return {"metadata": {"total_size": sum(os.path.getsize(f) for f in files)}, "weight_map": wmap}


def layer_prefix(weight_map, layer):
    """'<text decoder layers prefix><layer>.' of the base checkpoint (language model over towers)."""
    found = set()
    for k in weight_map:
        m = _LAYERS.match(k)
        if m and TAG not in k and "vision" not in m.group(1) and "audio" not in m.group(1):
            found.add(m.group(1))
    if not found:
        raise SystemExit("no decoder layers found in the base checkpoint")
    best = min(found, key=lambda p: ("language_model" not in p, len(p)))
    return f"{best}{layer}."


def _place(src, dst, copy):
    if os.path.lexists(dst):
        if os.path.isdir(dst) and not os.path.islink(dst):
            shutil.rmtree(dst)
        else:
            os.remove(dst)
    if copy:
        (shutil.copytree if os.path.isdir(src) else shutil.copy2)(src, dst)
    else:
        os.symlink(src, dst)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--base", required=True)
    ap.add_argument("--engram", required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--config", default=None)
    ap.add_argument("--copy", action="store_true", help="copy the base files instead of symlinking them")
    ap.add_argument("--force", action="store_true", help="write into a non-empty --out")
    args = ap.parse_args(argv)
    from safetensors.torch import save_file

    base, out = os.path.abspath(args.base), os.path.abspath(args.out)
    if os.path.isdir(out) and os.listdir(out) and not args.force:
        raise SystemExit(f"{out} is not empty (--force writes into it)")
    conf_path = find_config(args.engram, base, args.config)
    with open(conf_path) as f:
        conf = json.load(f)
    specs = engram_specs(conf, conf_path)
    msg = base_mismatch(conf, base)
    if msg:
        print(f"WARNING: {msg}")
    index = base_weight_map(base)
    wmap = {k: v for k, v in index["weight_map"].items() if TAG not in k}  # an older engram is replaced
    tensors = {}
    for spec in specs:
        several = len(specs) > 1
        src = (spec["weights"] or args.engram) if several else args.engram
        sd = load_engram_weights(src, layer=spec["layer"] if several else None)
        if not any(k.startswith("tables.") for k in sd):
            raise SystemExit(f"no engram tables for layer {spec['layer']} in {src}")
        prefix = layer_prefix(wmap, spec["layer"]) + TAG
        for k, v in sd.items():
            tensors[prefix + k] = v.contiguous()
        print(f"layer {spec['layer']}: {len(sd)} tensors from {src}")
    os.makedirs(out, exist_ok=True)
    for src in sorted(glob.glob(os.path.join(base, "*"))):
        if os.path.basename(src) not in (INDEX, CONFIG_NAME, ENGRAM_FILE):
            _place(src, os.path.join(out, os.path.basename(src)), args.copy)
    save_file(tensors, os.path.join(out, ENGRAM_FILE), metadata={"format": "pt"})
    nbytes = sum(v.numel() * v.element_size() for v in tensors.values())
    wmap.update(dict.fromkeys(tensors, ENGRAM_FILE))
    meta = dict(index.get("metadata", {}))
    meta["total_size"] = int(meta.get("total_size", 0)) + nbytes
    with open(os.path.join(out, INDEX), "w") as f:
        json.dump({"metadata": meta, "weight_map": dict(sorted(wmap.items()))}, f, indent=2)
    new = {k: v for k, v in conf.items() if k != "weights"}
    if new.get("engrams"):
        new["engrams"] = [{k: v for k, v in e.items() if k != "weights"} for e in new["engrams"]]
    with open(os.path.join(out, CONFIG_NAME), "w") as f:
        json.dump(new, f, indent=2)
    print(f"engram: {len(tensors)} tensors, {nbytes / 2 ** 30:.2f} GiB, keys like {next(iter(tensors))}")
    print(f"config: {conf_path} (" + "; ".join(f"layer {s['layer']}, {s['gate']} gate, seed {s['seed']}"
                                            for s in specs) + ")")
    print(f"wrote {out} ({'copied' if args.copy else 'symlinked'} base files from {base})")


if __name__ == "__main__":
    main()
