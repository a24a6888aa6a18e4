"""Generation with HF transformers plus trained engram(s) (reference: infer_engram.py:90-334).

    python -m micro_engram.tools.infer --model MERGED_DIR --prompt "Hello"
    python -m micro_engram.tools.infer --model BASE_DIR --engram-pt micro_engram.pt --prompt "Hello" [--no-engram]

Settings are resolved per key as: explicit flag > engram config > what the saved tensors
show (table count / shape, gate parameters) > defaults. A config listing several engrams
loads each from its own "weights" by layer. On a GPU the engram runs on the sm_100a kernels
(native hash and fused gate); the history of the current generation is kept, and only the
tail that new positions' n-grams can reach is hashed each step.
"""
import argparse
import glob
import json
import os
import re

import torch

from micro_engram.module import MicroEngram, check_loaded, engram_from_spec, find_text_layers, layer_device_dtype
from micro_engram.weights import CONFIG_NAME, base_mismatch, engram_specs, resolve_weights_path
from micro_engram.weights import load_engram_weights as load_engram_file

_LAYER_KEY = re.compile(r"layers\.(\d+)\.micro_engram\.")


def first(*values):
    for v in values:
        if v is not None:
            return v
    return None


def load_engram_weights(model_path, engram_pt=None):
    """(engram state dict with local names, layer seen in the key names or None)."""
    if engram_pt:
        return load_engram_file(engram_pt), None
    sd, layer = {}, None

    def take(key, val):
        nonlocal layer
        m = _LAYER_KEY.search(key)
        if m:
            layer = int(m.group(1))
        sd[key.split("micro_engram.", 1)[1]] = val

    from safetensors import safe_open

    for fn in sorted(glob.glob(os.path.join(model_path, "*.safetensors"))):
        with safe_open(fn, framework="pt", device="cpu") as fh:
            for k in fh.keys():
                if "micro_engram." in k:
                    take(k, fh.get_tensor(k))
    if not sd:
        for fn in sorted(glob.glob(os.path.join(model_path, "*.bin"))):
            for k, v in torch.load(fn, map_location="cpu").items():
                if "micro_engram." in k:
                    take(k, v)
    return sd, layer


def _read_conf(args):
    path = args.engram_config or os.path.join(args.model, CONFIG_NAME)
    if os.path.isfile(path):
        with open(path) as f:
            return json.load(f), path
    if args.engram_config:
        raise SystemExit(f"--engram-config file not found: {args.engram_config}")
    return {}, path


def shape_settings(sd, orders):
    """What the saved tensors say about the engram's layout."""
    n_tables = sum(1 for k in sd if k.startswith("tables.") and k.endswith(".weight"))
    t0 = sd.get("tables.0.weight")
    rows = [int(sd[f"tables.{k}.weight"].shape[0]) for k in range(n_tables) if f"tables.{k}.weight" in sd]
    heads = n_tables // len(orders) if n_tables else None
    gate = ("ple" if "up.weight" in sd else "scalar_sqrt" if "q_scale" in sd else "scalar" if "value.weight" in sd
            else None)
    return {"table_size": int(t0.shape[0]) if t0 is not None else None,
            "table_sizes": ({n: rows[i * heads] for i, n in enumerate(orders)}
                            if rows and heads and len(set(rows)) > 1 else None),
            "engram_dim": int(t0.shape[1]) if t0 is not None else None, "num_heads": heads, "gate": gate}


def resolve_settings(args, sd, layer_from_key):
    conf, path = _read_conf(args)
    orders = tuple(conf.get("orders", (2, 3)))
    shp = shape_settings(sd, orders)
    s = {"layer": first(args.layer, conf.get("layer"), layer_from_key, 0),
         "table_size": first(args.table_size, conf.get("table_size"), shp["table_size"], 65_536),
         "table_sizes": None if args.table_size else first(conf.get("table_sizes"), shp["table_sizes"]),
         "engram_dim": first(args.dim, conf.get("engram_dim"), shp["engram_dim"], 128),
         "num_heads": first(args.heads, conf.get("num_heads"), shp["num_heads"], 4),
         "orders": orders, "pad_id": conf.get("pad_id"), "model_dim": conf.get("model_dim"),
         "token_merge": conf.get("token_merge"), "canon_path": conf.get("canon_path"),
         "gate": first(getattr(args, "gate", None), conf.get("gate"), shp["gate"], "scalar"),
         "seed": first(conf.get("seed"), 0)}
    if conf:
        print(f"[engram] settings: {path} (explicit flags override it)")
    elif shp["table_size"] is not None:
        print("[engram] no engram config: settings read from the saved tensors (orders 2 and 3 assumed)")
    else:
        print("[engram] no config and no tensors to read: defaults")
    print("[engram] using: " + str({k: v for k, v in s.items() if k not in ("pad_id", "model_dim", "canon_path")}))
    return s


class EngramRunner:
    """Attaches engram(s) to an HF model and keeps the token history of one generation.

    EngramRunner(model, engram, layer) or EngramRunner(model, [(engram, layer), ...])."""

    def __init__(self, model, engrams, layer_idx=None):
        self.model = model
        self.engrams = [(engrams, layer_idx)] if layer_idx is not None else list(engrams)
        self.engram = self.engrams[0][0]
        self.hist = None
        self.enabled = True
        _, layers = find_text_layers(model)
        model.register_forward_pre_hook(self._grab, with_kwargs=True)
        for engram, layer in self.engrams:
            target = layers[layer]
            device, dtype = layer_device_dtype(target)
            engram.to(device=device, dtype=dtype)
            target.add_module("micro_engram", engram)
            target.register_forward_hook(self._hook(engram))

    def reset(self):
        self.hist = None

    def _grab(self, _mod, args, kwargs):
        ids = kwargs.get("input_ids")
        if ids is None and args:
            ids = args[0]
        if ids is not None:
            self.hist = ids if self.hist is None else torch.cat([self.hist, ids.to(self.hist.device)], dim=1)

    def _hook(self, engram):
        def inject(_mod, _args, output):
            if not self.enabled or self.hist is None:
                return output
            hidden = output[0] if isinstance(output, tuple) else output
            new = self.forward(engram, hidden)
            return (new,) + tuple(output[1:]) if isinstance(output, tuple) else new
        return inject

    @torch.no_grad()
    def forward(self, engram, hidden):
        T = hidden.shape[1]
        tail = self.hist[:, -(T + max(engram.orders) - 1):]  # all that T new positions' n-grams reach
        idx = [i[:, -T:] for i in engram.hash_ids(tail.to(hidden.device))]
        return engram.inject(hidden, idx)


def plan_engrams(args):
    """[(settings, state dict)] per engram, read before the model load so bad paths fail fast."""
    explicit = args.engram_pt
    if not args.engram_pt and args.engram_config:
        with open(args.engram_config) as f:
            args.engram_pt = resolve_weights_path(json.load(f), args.engram_config)
    conf, conf_path = _read_conf(args)
    if conf:
        msg = base_mismatch(conf, args.model)
        if msg:
            print(f"[engram] WARNING: {msg}")
    if len(conf.get("engrams") or []) > 1:
        plans = []
        for spec in engram_specs(conf, conf_path):
            src = explicit or spec["weights"] or args.model
            sd = load_engram_file(src, layer=spec["layer"])
            if not any(k.startswith("tables.") for k in sd):
                raise SystemExit(f"no engram weights for layer {spec['layer']} in {src}")
            spec["model_dim"] = conf.get("model_dim")
            print(f"[engram] layer {spec['layer']}: {spec['gate']} gate, {spec['num_heads']} heads, seed "
                  f"{spec['seed']}, from {src}")
            plans.append((spec, sd))
        return plans
    sd, layer = load_engram_weights(args.model, args.engram_pt)
    if not sd:
        raise SystemExit("no micro_engram weights found (wrong path, or they were not saved)")
    return [(resolve_settings(args, sd, layer), sd)]


def attach_planned(plans, model):
    text_cfg = getattr(model.config, "text_config", model.config)
    pairs = []
    for s, sd in plans:
        if s.get("model_dim") and s["model_dim"] != text_cfg.hidden_size:
            raise SystemExit(f"the config says model_dim {s['model_dim']}, the model has hidden_size "
                             f"{text_cfg.hidden_size}")
        canon = None
        if "canon" not in sd and s.get("token_merge"):
            path = s.get("canon_path")
            if not path or not os.path.isfile(path):
                raise SystemExit(f"training merged tokens but the weights have no 'canon' and the canon file is "
                                 f"missing ({path}); copy it and fix canon_path in {CONFIG_NAME}")
            canon = torch.load(path, map_location="cpu")
        engram = engram_from_spec(s, text_cfg.hidden_size, text_cfg.vocab_size,
                                  first(getattr(text_cfg, "pad_token_id", None), 0), canon)
        check_loaded(engram, sd, f"layer {s['layer']} weights")
        out = engram.up if engram.gate == "ple" else engram.value
        print(f"[engram] layer {s['layer']}: {len(sd)} tensors, output-weight magnitude "
              f"{out.weight.float().abs().mean().item():.6f} ({engram.gate} gate; 0 = untrained or not loaded)")
        pairs.append((engram, s["layer"]))
    return EngramRunner(model, pairs)


def add_engram_args(ap):
    ap.add_argument("--model", required=True, help="merged model dir (or the base with --engram-pt)")
    ap.add_argument("--engram-pt", default=None, help=".pt, .safetensors, a safetensors folder or a DCP folder")
    ap.add_argument("--engram-config", default=None)
    ap.add_argument("--layer", type=int, default=None)
    ap.add_argument("--table-size", type=int, default=None)
    ap.add_argument("--dim", type=int, default=None)
    ap.add_argument("--heads", type=int, default=None)
    ap.add_argument("--gate", choices=MicroEngram.GATES, default=None)


def load_model(args):
    from transformers import AutoModelForCausalLM, AutoTokenizer

    plans = plan_engrams(args)
    tok = AutoTokenizer.from_pretrained(args.model)
    model = AutoModelForCausalLM.from_pretrained(args.model, dtype=torch.bfloat16, device_map="auto").eval()
    return model, tok, attach_planned(plans, model)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    add_engram_args(ap)
    ap.add_argument("--prompt", required=True)
    ap.add_argument("--raw", action="store_true", help="no chat template")
    ap.add_argument("--no-engram", action="store_true")
    ap.add_argument("--max-new-tokens", type=int, default=2000)
    ap.add_argument("--temperature", type=float, default=0.8)
    ap.add_argument("--top-p", type=float, default=0.95)
    args = ap.parse_args(argv)
    model, tok, runner = load_model(args)
    runner.enabled = not args.no_engram
    print(f"[engram] enabled: {runner.enabled}")
    if args.raw or not getattr(tok, "chat_template", None):
        ids = tok(args.prompt, return_tensors="pt").input_ids
    else:
        ids = tok.apply_chat_template([{"role": "user", "content": args.prompt}], add_generation_prompt=True,
                                      return_tensors="pt")
        if not torch.is_tensor(ids):
            ids = ids["input_ids"]
    ids = ids.to(next(model.parameters()).device)
    runner.reset()
    with torch.no_grad():
        out = model.generate(input_ids=ids, max_new_tokens=args.max_new_tokens, do_sample=args.temperature > 0,
                             temperature=args.temperature if args.temperature > 0 else None, top_p=args.top_p,
                             use_cache=True)
    print("\n--- output ---")
    print(tok.decode(out[0, ids.shape[1]:], skip_special_tokens=True))


if __name__ == "__main__":
    main()
