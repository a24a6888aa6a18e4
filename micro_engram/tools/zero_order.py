"""Ablation copies of a trained engram: n-gram orders switched off and/or the injection scaled
(the reference's zero_ngram_order.py offers the same ablations).

    python -m micro_engram.tools.zero_order SRC --order 4 --out DIR
    python -m micro_engram.tools.zero_order SRC --scale 0.5 --out DIR
    python -m micro_engram.tools.zero_order SRC --order 4 --layer-scale 29=0.5 --out DIR

SRC is an engram config, or a folder holding one (checkpoint-N, an output_dir, which means its
newest complete checkpoint, or an assembled model). --order N zeroes every table of order N
(repeatable); --scale S multiplies the output projection (value, or ple's up) of every engram
and --layer-scale L=S that of layer L only. DIR receives consolidated.pth (every engram, full
key names) and a config pointing at it that records zeroed_orders, injection_scale and
zeroed_from.
"""
import argparse
import json
import os
from dataclasses import dataclass

import torch

from micro_engram.weights import CONFIG_NAME, engram_specs, latest_checkpoint, load_engram_weights

OUT_WEIGHTS = "consolidated.pth"
KEY_PREFIX = "model.language_model.layers.{}.micro_engram."


def find_config(src):
    """The micro_engram_config.json that SRC stands for."""
    src = os.path.abspath(src)
    candidates = [src] if src.endswith(".json") else [os.path.join(src, CONFIG_NAME)]
    newest = None if src.endswith(".json") else latest_checkpoint(src)
    if newest:
        candidates.append(os.path.join(newest, CONFIG_NAME))
    for c in candidates:
        if os.path.isfile(c):
            return c
    raise SystemExit(f"no {CONFIG_NAME} in {src} (give the config, a checkpoint-N folder or an output_dir)")


def table_orders(spec):
    """The n-gram order of each table, in the module's order-major, then head, layout."""
    heads = int(spec["num_heads"])
    return [order for order in sorted(int(o) for o in spec["orders"]) for _ in range(heads)]


@dataclass
class Ablation:
    zero: frozenset
    scale: float
    per_layer: dict

    @classmethod
    def from_args(cls, orders, scale, layer_scales):
        per_layer = {}
        for item in layer_scales:
            layer, sep, value = item.partition("=")
            try:
                per_layer[int(layer)] = float(value)
            except ValueError:
                raise SystemExit(f"--layer-scale wants L=S, e.g. 29=0.5 (got {item!r})") from None
            if not sep:
                raise SystemExit(f"--layer-scale wants L=S, e.g. 29=0.5 (got {item!r})")
        return cls(frozenset(orders), scale, per_layer)

    def is_noop(self):
        return not self.zero and self.scale == 1.0 and not self.per_layer

    def scale_of(self, layer):
        return self.per_layer.get(layer, self.scale)

    def apply(self, layer, sd, orders):
        """Zero the chosen orders' tables and scale the output projection of one engram in place;
        returns the number of rows zeroed."""
        zeroed = 0
        for k, order in enumerate(orders):
            if order in self.zero:
                table = sd[f"tables.{k}.weight"]
                table.zero_()
                zeroed += table.shape[0]
        factor = self.scale_of(layer)
        if factor != 1.0:
            out = "value.weight" if "value.weight" in sd else "up.weight"
            sd[out] = (sd[out].float() * factor).to(sd[out].dtype)
        return zeroed


def _ablated_config(conf, conf_path, specs, ab):
    new = dict(conf, weights=OUT_WEIGHTS)
    if new.get("engrams"):
        new["engrams"] = [dict(e, weights=OUT_WEIGHTS) for e in new["engrams"]]
    new["zeroed_orders"] = sorted(ab.zero)
    new["injection_scale"] = {str(s["layer"]): ab.scale_of(s["layer"]) for s in specs}
    new["zeroed_from"] = conf_path
    return new


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("src")
    ap.add_argument("--order", type=int, action="append", default=[], help="zero every table of this order")
    ap.add_argument("--scale", type=float, default=1.0, help="output projection factor of every engram")
    ap.add_argument("--layer-scale", action="append", default=[], metavar="L=S", help="factor for layer L only")
    ap.add_argument("--out", required=True)
    ap.add_argument("--force", action="store_true", help="overwrite DIR's consolidated.pth")
    args = ap.parse_args(argv)
    conf_path = find_config(args.src)
    with open(conf_path) as f:
        conf = json.load(f)
    specs = engram_specs(conf, conf_path)
    if os.path.exists(os.path.join(args.out, OUT_WEIGHTS)) and not args.force:
        raise SystemExit(f"{args.out} already has {OUT_WEIGHTS} (use --force)")
    ab = Ablation.from_args(args.order, args.scale, args.layer_scale)
    if ab.is_noop():
        raise SystemExit("nothing to do: give --order, --scale and/or --layer-scale")
    os.makedirs(args.out, exist_ok=True)
    merged = {}
    for spec in specs:
        layer = spec["layer"]
        src = spec["weights"] or os.path.dirname(conf_path)
        sd = load_engram_weights(src, layer=layer, need_layer=len(specs) > 1)
        orders = table_orders(spec)
        found = sum(k.startswith("tables.") for k in sd)
        if found != len(orders):
            raise SystemExit(f"layer {layer}: {found} tables in {src}, but the config's orders x heads give "
                             f"{len(orders)}")
        missing = ab.zero - set(orders)
        if ab.zero and missing:
            print(f"layer {layer}: has no order {sorted(missing)} (orders {sorted(set(orders))})")
        rows = ab.apply(layer, sd, orders)
        print(f"layer {layer}: zeroed {rows:,} rows of order(s) {sorted(ab.zero & set(orders))}, injection "
              f"x{ab.scale_of(layer):g} ({len(orders)} tables, from {src})")
        merged.update((KEY_PREFIX.format(layer) + k, v) for k, v in sd.items())
    torch.save(merged, os.path.join(args.out, OUT_WEIGHTS))
    with open(os.path.join(args.out, CONFIG_NAME), "w") as f:
        json.dump(_ablated_config(conf, conf_path, specs, ab), f, indent=2)
    print(f"wrote {args.out}/{OUT_WEIGHTS} and {CONFIG_NAME} ({len(specs)} engram(s))")


if __name__ == "__main__":
    main()
