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
from collections import ChainMap

import torch

from micro_engram.module import MicroEngram, check_loaded, engram_from_spec, find_text_layers, layer_device_dtype
from micro_engram.weights import CONFIG_NAME, base_mismatch, engram_specs, resolve_weights_path
from micro_engram.weights import load_engram_weights as read_engram_source

_ENGRAM_KEY = re.compile(r"layers\.(\d+)\.micro_engram\.(.+)$")
DEFAULTS = {"layer": 0, "table_size": 65_536, "engram_dim": 128, "num_heads": 4, "gate": "scalar", "seed": 0}
_FROM_CONFIG = ("layer", "table_size", "table_sizes", "engram_dim", "num_heads", "gate", "seed")
_PASSED_THROUGH = ("pad_id", "model_dim", "token_merge", "canon_path")


def _present(d):
    """The entries of d that say something (None means: not given here)."""
    return {k: v for k, v in d.items() if v is not None}


# ------------------------------------------------------------------ where the engram comes from
def _model_folder_tensors(model_path):
    """(local-name state dict, layer) of the engram inside a model folder's own shards:
    safetensors first, .bin only when those hold none."""
    from safetensors import safe_open

    def shards():
        for fn in sorted(glob.glob(os.path.join(model_path, "*.safetensors"))):
            with safe_open(fn, framework="pt", device="cpu") as fh:
                yield from ((k, fh.get_tensor(k)) for k in fh.keys() if "micro_engram." in k)

    def bins():
        for fn in sorted(glob.glob(os.path.join(model_path, "*.bin"))):
            yield from ((k, v) for k, v in torch.load(fn, map_location="cpu").items() if "micro_engram." in k)

    for source in (shards, bins):
        found, layer = {}, None
        for key, tensor in source():
            m = _ENGRAM_KEY.search(key)
            if m:
                layer = int(m.group(1))
            found[key.split("micro_engram.", 1)[1]] = tensor
        if found:
            return found, layer
    return {}, None


def load_engram_weights(model_path, engram_pt=None):
    """(engram state dict with local names, layer named by the keys or None)."""
    return (read_engram_source(engram_pt), None) if engram_pt else _model_folder_tensors(model_path)


def _config_of(args):
    """(engram config dict, its path): --engram-config, else the one beside the model, else {}."""
    path = args.engram_config or os.path.join(args.model, CONFIG_NAME)
    if not os.path.isfile(path):
        if args.engram_config:
            raise SystemExit(f"--engram-config file not found: {args.engram_config}")
        return {}, path
    with open(path) as f:
        return json.load(f), path


def shape_settings(sd, orders):
    """What the saved tensors say about the engram's layout (None where they say nothing)."""
    gate = "ple" if "up.weight" in sd else "scalar_sqrt" if "q_scale" in sd else "scalar" if "value.weight" in sd \
        else None
    tables = [sd[f"tables.{k}.weight"] for k in range(len(sd)) if f"tables.{k}.weight" in sd]
    if not tables:
        return {"table_size": None, "table_sizes": None, "engram_dim": None, "num_heads": None, "gate": gate}
    heads = len(tables) // len(orders)
    rows = [int(t.shape[0]) for t in tables]
    per_order = {n: rows[i * heads] for i, n in enumerate(orders)} if heads and len(set(rows)) > 1 else None
    return {"table_size": rows[0], "table_sizes": per_order, "engram_dim": int(tables[0].shape[1]),
            "num_heads": heads or None, "gate": gate}


def resolve_settings(args, sd, layer_from_key):
    """One engram's settings, each key from the first layer that gives it: flags, the engram
    config, the saved tensors, DEFAULTS."""
    conf, path = _config_of(args)
    orders = tuple(conf.get("orders", (2, 3)))
    flags = _present({"layer": args.layer, "table_size": args.table_size, "engram_dim": args.dim,
                      "num_heads": args.heads, "gate": getattr(args, "gate", None)})
    seen = _present({**shape_settings(sd, orders), "layer": layer_from_key})
    chain = ChainMap(flags, _present({k: conf.get(k) for k in _FROM_CONFIG}), seen, DEFAULTS)
    settings = {k: chain.get(k) for k in (*DEFAULTS, "table_sizes")}
    if args.table_size:  # an explicit size is one size for every order
        settings["table_sizes"] = None
    settings.update({"orders": orders}, **{k: conf.get(k) for k in _PASSED_THROUGH})
    if conf:
        print(f"[engram] settings: {path} (explicit flags override it)")
    elif "table_size" in seen:
        print("[engram] no engram config: settings read from the saved tensors (orders 2 and 3 assumed)")
    else:
        print("[engram] no config and no tensors to read: defaults")
    shown = {k: v for k, v in settings.items() if k not in ("pad_id", "model_dim", "canon_path")}
    print(f"[engram] using: {shown}")
    return settings


def plan_engrams(args):
    """[(settings, state dict)] per engram, read before the model loads so a bad path fails fast."""
    given_pt = args.engram_pt
    if not args.engram_pt and args.engram_config:
        with open(args.engram_config) as f:
            args.engram_pt = resolve_weights_path(json.load(f), args.engram_config)
    conf, conf_path = _config_of(args)
    note = base_mismatch(conf, args.model) if conf else None
    if note:
        print(f"[engram] WARNING: {note}")
    if len(conf.get("engrams") or []) <= 1:
        sd, layer = load_engram_weights(args.model, args.engram_pt)
        if not sd:
            raise SystemExit("no micro_engram weights found (wrong path, or they were not saved)")
        return [(resolve_settings(args, sd, layer), sd)]
    plans = []
    for spec in engram_specs(conf, conf_path):  # several engrams: each from its own weights, by layer
        where = given_pt or spec["weights"] or args.model
        sd = read_engram_source(where, layer=spec["layer"])
        if not any(k.startswith("tables.") for k in sd):
            raise SystemExit(f"no engram weights for layer {spec['layer']} in {where}")
        spec["model_dim"] = conf.get("model_dim")
        print(f"[engram] layer {spec['layer']}: {spec['gate']} gate, {spec['num_heads']} heads, seed "
              f"{spec['seed']}, from {where}")
        plans.append((spec, sd))
    return plans


# ------------------------------------------------------------------ the generation session
class EngramSession:
    """Engrams attached to one HF model, plus the token history of the generation in flight.

    A pre-hook on the model appends every call's input_ids to the history (prefill, then one
    token per decode step); a hook after each engram's layer adds the engram's gated memory,
    hashing only the tail of the history that the call's new positions' n-grams reach."""

    def __init__(self, model, attached):
        self.model, self.attached = model, list(attached)  # [(engram, layer)]
        self.history, self.enabled = None, True
        _, layers = find_text_layers(model)
        model.register_forward_pre_hook(self._see_inputs, with_kwargs=True)
        for engram, layer in self.attached:
            block = layers[layer]
            device, dtype = layer_device_dtype(block)
            block.add_module("micro_engram", engram.to(device=device, dtype=dtype))
            block.register_forward_hook(self._after_layer(engram))

    def new_sequence(self):
        self.history = None

    def _see_inputs(self, _mod, args, kwargs):
        ids = kwargs.get("input_ids")
        if ids is None:
            ids = args[0] if args else None
        if ids is None:
            return
        self.history = ids if self.history is None else torch.cat([self.history, ids.to(self.history.device)], 1)

    def _after_layer(self, engram):
        def add_memory(_mod, _args, output):
            if not self.enabled or self.history is None:
                return output
            if isinstance(output, tuple):
                return (self.with_memory(engram, output[0]),) + tuple(output[1:])
            return self.with_memory(engram, output)

        return add_memory

    @torch.no_grad()
    def with_memory(self, engram, hidden):
        """hidden [B, T, d] of the newest T positions + the engram's gated memory."""
        T = hidden.shape[1]
        reach = self.history[:, -(T + max(engram.orders) - 1):].to(hidden.device)
        return engram.inject(hidden, [i[:, -T:] for i in engram.hash_ids(reach)])


def attach_planned(plans, model):
    """Build every planned engram for `model`, check it against its tensors, attach them."""
    text_cfg = getattr(model.config, "text_config", model.config)
    pad = getattr(text_cfg, "pad_token_id", None)
    attached = []
    for s, sd in plans:
        if s.get("model_dim") and s["model_dim"] != text_cfg.hidden_size:
            raise SystemExit(f"the config says model_dim {s['model_dim']}, the model has hidden_size "
                             f"{text_cfg.hidden_size}")
        canon = None
        if s.get("token_merge") and "canon" not in sd:
            path = s.get("canon_path")
            if not (path and os.path.isfile(path)):
                raise SystemExit(f"training merged tokens but the weights have no 'canon' and the canon file is "
                                 f"missing ({path}); copy it and fix canon_path in {CONFIG_NAME}")
            canon = torch.load(path, map_location="cpu")
        engram = engram_from_spec(s, text_cfg.hidden_size, text_cfg.vocab_size, 0 if pad is None else pad, canon)
        check_loaded(engram, sd, f"layer {s['layer']} weights")
        out_w = (engram.up if engram.gate == "ple" else engram.value).weight
        print(f"[engram] layer {s['layer']}: {len(sd)} tensors, output-weight magnitude "
              f"{out_w.float().abs().mean().item():.6f} ({engram.gate} gate; 0 = untrained or not loaded)")
        attached.append((engram, s["layer"]))
    return EngramSession(model, attached)


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
    """(model, tokenizer, EngramSession) for the engram(s) `args` name."""
    from transformers import AutoModelForCausalLM, AutoTokenizer

    plans = plan_engrams(args)
    tok = AutoTokenizer.from_pretrained(args.model)
    model = AutoModelForCausalLM.from_pretrained(args.model, dtype=torch.bfloat16, device_map="auto").eval()
    return model, tok, attach_planned(plans, model)


def _prompt_ids(tok, prompt, raw):
    if raw or not getattr(tok, "chat_template", None):
        return tok(prompt, return_tensors="pt").input_ids
    ids = tok.apply_chat_template([{"role": "user", "content": prompt}], add_generation_prompt=True,
                                  return_tensors="pt")
    return ids if torch.is_tensor(ids) else ids["input_ids"]


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
    model, tok, session = load_model(args)
    session.enabled = not args.no_engram
    print(f"[engram] enabled: {session.enabled}")
    ids = _prompt_ids(tok, args.prompt, args.raw).to(next(model.parameters()).device)
    session.new_sequence()
    sample = args.temperature > 0
    with torch.no_grad():
        out = model.generate(input_ids=ids, max_new_tokens=args.max_new_tokens, do_sample=sample,
                             temperature=args.temperature if sample else None, top_p=args.top_p, use_cache=True)
    print("\n--- output ---")
    print(tok.decode(out[0, ids.shape[1]:], skip_special_tokens=True))


if __name__ == "__main__":
    main()
