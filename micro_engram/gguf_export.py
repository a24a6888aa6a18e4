"""Add trained micro-engram(s) to a Gemma 4 GGUF (reference: llama_cpp/gguf_add_engram.py).

    python engram_runtime/gguf_add_engram.py --gguf base.gguf --engram CKPT_OR_CONFIG --out out.gguf
        [--dtype bf16|f16|f32] [--force]

--engram: a checkpoint-N folder, an assembled model folder or an engram config (every
engram it lists is added, each from its own "weights"). The base file's metadata and tensors
are copied unchanged (any quantization); the engram goes in as --dtype (norm scales F32).

The layout is the one the engram runtime (engram_runtime/) and the llama.cpp patch read, and
it is identical to the reference's so either build loads either file:
  metadata arrays micro_engram.{layers, table_size, table_rows, dim, n_tables, gate, pad_id,
  table_orders, mults (max_order per table, zero padded), canon} + micro_engram.max_order;
  tensors blk.L.engram_kv.mengram_{tables [all tables' rows, dim], key, value | down, up} and
  blk.L.engram_gate.mengram_{q_scale, k_scale} (the scales themselves, not the stored deltas).
One GGUF holds one token-merge map, so every engram must share it.
"""
import argparse
import json
import os
import sys

import numpy as np
import torch

from micro_engram.module import check_loaded, engram_from_spec
from micro_engram.weights import CONFIG_NAME, engram_specs, load_engram_weights

GATE_CODE = {"scalar": 0, "scalar_sqrt": 1, "ple": 2}
PREFIX = "micro_engram."


def find_config(path):
    path = os.path.abspath(path)
    conf = path if path.endswith(".json") else os.path.join(path, CONFIG_NAME)
    if not os.path.isfile(conf):
        raise SystemExit(f"{CONFIG_NAME} not found at {conf}")
    return conf


def _trained_engram(spec, conf, src, n_embd, several):
    """The MicroEngram of one spec with the weights found at `src` (the canon map from the
    weights when they carry one, else from the spec's canon_path when it merged tokens)."""
    sd = load_engram_weights(src, layer=spec["layer"] if several else None)
    if not any(k.startswith("tables.") for k in sd):
        raise SystemExit(f"no engram weights for layer {spec['layer']} in {src}")
    if "canon" in sd:
        vocab, canon = int(sd["canon"].numel()), None
    else:
        vocab = int(conf.get("vocab_size") or 262144)
        canon = torch.load(spec["canon_path"], map_location="cpu") if spec.get("token_merge") else None
    eng = engram_from_spec(spec, n_embd, vocab, conf.get("pad_id") or 0, canon)
    check_loaded(eng, sd, src)
    return eng


def load_engrams(conf_path, n_embd):
    """[(spec, MicroEngram with its trained weights)] in layer order."""
    with open(conf_path) as f:
        conf = json.load(f)
    specs = sorted(engram_specs(conf, conf_path), key=lambda sp: sp["layer"])
    loaded = []
    for spec in specs:
        src = spec["weights"] or os.path.dirname(conf_path)
        eng = _trained_engram(spec, conf, src, n_embd, len(specs) > 1)
        print(f"layer {spec['layer']}: {spec['gate']} gate, {len(eng.tables)} tables, rows per order "
              f"{eng.order_sizes} x {eng.engram_dim}, seed {spec['seed']}, from {src}")
        loaded.append((spec, eng))
    return loaded


def _array(t, dtype):
    """(numpy array, raw GGML type or None) of a tensor in the requested storage type."""
    import gguf

    t = t.detach().float().cpu()
    if dtype == "f32":
        return t.numpy(), None
    if dtype == "f16":
        return t.half().numpy(), None
    return t.bfloat16().view(torch.int16).numpy().view(np.uint16), gguf.GGMLQuantizationType.BF16


def engram_tensors(layer, eng, dtype="bf16"):
    """{GGUF tensor name: (array, raw type)} for one engram."""
    kv, gv = f"blk.{layer}.engram_kv.mengram_", f"blk.{layer}.engram_gate.mengram_"
    out = {kv + "tables": _array(torch.cat([t.weight for t in eng.tables], dim=0), dtype)}
    if eng.gate == "ple":
        out[kv + "down"] = _array(eng.down.weight, dtype)
        out[kv + "up"] = _array(eng.up.weight, dtype)
    else:
        out[kv + "key"] = _array(eng.key.weight, dtype)
        out[kv + "value"] = _array(eng.value.weight, dtype)
        if eng.gate == "scalar_sqrt":
            qs, ks = eng.norm_scales()
            out[gv + "q_scale"] = _array(qs, "f32")
            out[gv + "k_scale"] = _array(ks, "f32")
    return out


def engram_metadata(engrams):
    """({key: (values, element type)}, max_order) of the micro_engram.* arrays."""
    import gguf

    T = gguf.GGUFValueType
    max_order = max(max(e.orders) for _, e in engrams)
    orders, mults, rows = [], [], []
    for _, e in engrams:
        m = e.mults.long()
        for k, n in enumerate(e._table_orders):
            orders.append(int(n))
            rows.append(int(e.table_rows[k]))
            mults.extend([int(v) for v in m[k, :n]] + [0] * (max_order - n))
    canon = engrams[0][1].canon
    return {
        "layers": ([s["layer"] for s, _ in engrams], T.UINT32),
        "table_size": ([int(e.table_size or 0) for _, e in engrams], T.UINT32),
        "table_rows": (rows, T.UINT32),
        "dim": ([int(e.engram_dim) for _, e in engrams], T.UINT32),
        "n_tables": ([len(e.table_rows) for _, e in engrams], T.UINT32),
        "gate": ([GATE_CODE[e.gate] for _, e in engrams], T.UINT32),
        "pad_id": ([int(e.pad_id) for _, e in engrams], T.INT32),
        "table_orders": (orders, T.UINT32),
        "mults": (mults, T.UINT64),
        "canon": ([int(v) for v in canon.long()], T.INT32),
    }, max_order


def _field(reader, key):
    f = reader.fields.get(key)
    return None if f is None else f.contents()


def add_engrams(src, engram, out, dtype="bf16", force=False):
    import gguf

    if os.path.exists(out) and not force:
        raise SystemExit(f"{out} exists (use --force)")
    reader = gguf.GGUFReader(src)
    arch = _field(reader, gguf.Keys.General.ARCHITECTURE)
    if arch != "gemma4":
        raise SystemExit(f"{src} is a {arch!r} model; the engram GGUF layout is defined for gemma4")
    if _field(reader, "split.count"):
        raise SystemExit("split GGUFs are not supported: merge it first")
    if any(k.startswith(PREFIX) for k in reader.fields) and not force:
        raise SystemExit(f"{src} already has an engram (use --force to replace it)")
    n_embd = int(_field(reader, f"{arch}.embedding_length"))
    n_layer = int(_field(reader, f"{arch}.block_count"))
    engrams = load_engrams(find_config(engram), n_embd)
    canon = engrams[0][1].canon
    for spec, e in engrams[1:]:
        if not torch.equal(e.canon, canon):
            raise SystemExit(f"the engram at layer {spec['layer']} uses another token-merge map; one GGUF holds one")
    for spec, _ in engrams:
        if spec["layer"] >= n_layer:
            raise SystemExit(f"engram layer {spec['layer']} but the model has {n_layer} layers")
    toks = _field(reader, gguf.Keys.Tokenizer.LIST)
    if toks is not None and len(toks) != canon.numel():
        print(f"WARNING: the GGUF vocabulary has {len(toks)} tokens, the token-merge map {canon.numel()}")
    meta, max_order = engram_metadata(engrams)
    T = gguf.GGUFValueType
    w = gguf.GGUFWriter(out, arch=arch, endianess=reader.endianess)
    for field in reader.fields.values():
        name = field.name
        if name == gguf.Keys.General.ARCHITECTURE or name.startswith("GGUF.") or name.startswith(PREFIX):
            continue
        vt = field.types[0]
        w.add_key_value(name, field.contents(), vt, sub_type=field.types[-1] if vt == T.ARRAY else None)
    for key, (vals, sub) in meta.items():
        w.add_key_value(PREFIX + key, vals, T.ARRAY, sub_type=sub)
    w.add_key_value(PREFIX + "max_order", max_order, T.UINT32)
    base = [t for t in reader.tensors if ".mengram_" not in t.name]
    new = {}
    for spec, e in engrams:
        new.update(engram_tensors(spec["layer"], e, dtype))
    for t in base:
        w.add_tensor_info(t.name, t.data.shape, t.data.dtype, t.data.nbytes, t.tensor_type)
    for name, (arr, raw) in new.items():
        w.add_tensor_info(name, arr.shape, arr.dtype, arr.nbytes, raw)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_ti_data_to_file()
    for t in base:
        w.write_tensor_data(t.data, tensor_endianess=reader.endianess)
    for arr, _ in new.values():
        w.write_tensor_data(arr)
    w.close()
    size = sum(a.nbytes for a, _ in new.values()) / 2 ** 30
    print(f"wrote {out}: {len(base)} base tensors + {len(new)} engram tensors ({size:.2f} GiB, {dtype})")


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gguf", required=True)
    ap.add_argument("--engram", required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--dtype", choices=["bf16", "f16", "f32"], default="bf16")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args(argv)
    try:
        import gguf  # noqa: F401
    except ImportError as e:
        sys.exit(f"the gguf package is needed ({e}); pip install gguf, or PYTHONPATH=<llama.cpp>/gguf-py")
    add_engrams(args.gguf, args.engram, args.out, args.dtype, args.force)


if __name__ == "__main__":
    main()
