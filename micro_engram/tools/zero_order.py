"""Copy of an engram with n-gram orders zeroed and/or its injection scaled (ablations;
reference: zero_ngram_order.py:59-131).

    python -m micro_engram.tools.zero_order SRC --order 4 --out DIR
    python -m micro_engram.tools.zero_order SRC --scale 0.5 --out DIR
    python -m micro_engram.tools.zero_order SRC --order 4 --layer-scale 29=0.5 --out DIR

SRC: an engram config, or a folder with one (checkpoint-N, an output_dir = its newest
checkpoint, or an assembled model). --order N zeroes every table of order N (repeatable);
--scale S multiplies the output projection (value, or up for ple) of every engram;
--layer-scale L=S sets it for layer L. DIR gets consolidated.pth (all engrams, full key
names) and the config pointing at it, plus zeroed_orders / injection_scale / zeroed_from.
"""
import argparse
import json
import os

import torch

from micro_engram.weights import CONFIG_NAME, engram_specs, latest_checkpoint, load_engram_weights

OUT_WEIGHTS = "consolidated.pth"


def find_config(src):
    src = os.path.abspath(src)
    if src.endswith(".json"):
        return src
    if os.path.isfile(os.path.join(src, CONFIG_NAME)):
        return os.path.join(src, CONFIG_NAME)
    ckpt = latest_checkpoint(src)
    if ckpt and os.path.isfile(os.path.join(ckpt, CONFIG_NAME)):
        return os.path.join(ckpt, CONFIG_NAME)
    raise SystemExit(f"no {CONFIG_NAME} in {src} (give the config, a checkpoint-N folder or an output_dir)")


def table_orders(spec):
    """Order of every table in the module layout (order-major, then head)."""
    return [n for n in sorted(int(o) for o in spec["orders"]) for _ in range(int(spec["num_heads"]))]


def _layer_scales(items):
    out = {}
    for it in items:
        try:
            layer, val = it.split("=")
            out[int(layer)] = float(val)
        except ValueError:
            raise SystemExit(f"--layer-scale wants L=S, e.g. 29=0.5 (got {it!r})") from None
    return out


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("src")
    ap.add_argument("--order", type=int, action="append", default=[])
    ap.add_argument("--scale", type=float, default=1.0)
    ap.add_argument("--layer-scale", action="append", default=[], metavar="L=S")
    ap.add_argument("--out", required=True)
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args(argv)
    conf_path = find_config(args.src)
    with open(conf_path) as f:
        conf = json.load(f)
    specs = engram_specs(conf, conf_path)
    if os.path.exists(os.path.join(args.out, OUT_WEIGHTS)) and not args.force:
        raise SystemExit(f"{args.out} already has {OUT_WEIGHTS} (use --force)")
    zero, per_layer = set(args.order), _layer_scales(args.layer_scale)
    if not zero and args.scale == 1.0 and not per_layer:
        raise SystemExit("nothing to do: give --order, --scale and/or --layer-scale")
    os.makedirs(args.out, exist_ok=True)
    merged = {}
    for spec in specs:
        layer = spec["layer"]
        src = spec["weights"] or os.path.dirname(conf_path)
        sd = load_engram_weights(src, layer=layer, need_layer=len(specs) > 1)
        orders = table_orders(spec)
        n_tables = sum(k.startswith("tables.") for k in sd)
        if n_tables != len(orders):
            raise SystemExit(f"layer {layer}: {n_tables} tables in {src}, the config's orders x heads give "
                             f"{len(orders)}")
        absent = zero - set(orders)
        if zero and absent:
            print(f"layer {layer}: has no order {sorted(absent)} (orders {sorted(set(orders))})")
        rows = 0
        for k, n in enumerate(orders):
            if n in zero:
                sd[f"tables.{k}.weight"].zero_()
                rows += sd[f"tables.{k}.weight"].shape[0]
        scale = per_layer.get(layer, args.scale)
        if scale != 1.0:
            proj = "value.weight" if "value.weight" in sd else "up.weight"
            sd[proj] = (sd[proj].float() * scale).to(sd[proj].dtype)
        print(f"layer {layer}: zeroed {rows:,} rows of order(s) {sorted(zero & set(orders))}, injection x{scale:g} "
              f"({len(orders)} tables, from {src})")
        merged.update({f"model.language_model.layers.{layer}.micro_engram.{k}": v for k, v in sd.items()})
    torch.save(merged, os.path.join(args.out, OUT_WEIGHTS))
    new = dict(conf, weights=OUT_WEIGHTS)
    if new.get("engrams"):
        new["engrams"] = [dict(e, weights=OUT_WEIGHTS) for e in new["engrams"]]
    new["zeroed_orders"] = sorted(zero)
    new["injection_scale"] = {str(s["layer"]): per_layer.get(s["layer"], args.scale) for s in specs}
    new["zeroed_from"] = conf_path
    with open(os.path.join(args.out, CONFIG_NAME), "w") as f:
        json.dump(new, f, indent=2)
    print(f"wrote {args.out}/{OUT_WEIGHTS} and {CONFIG_NAME} ({len(specs)} engram(s))")


if __name__ == "__main__":
    main()
