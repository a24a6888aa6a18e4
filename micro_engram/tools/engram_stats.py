"""Engram weight statistics of checkpoints on disk (CPU only; safe while training runs;
reference: engram_stats.py:57-130).

    python -m micro_engram.tools.engram_stats OUTPUT_DIR            # newest complete checkpoint
    python -m micro_engram.tools.engram_stats OUTPUT_DIR --all      # every checkpoint on disk
    python -m micro_engram.tools.engram_stats OUTPUT_DIR --watch 120
    python -m micro_engram.tools.engram_stats micro_engram.pt --config micro_engram_config.json

Columns: out|w| (mean |weight| of value, or up for ple; 0 = untrained), rms Ng (RMS of the
N-gram tables; they start at 0.02), learned Ng (share of rows whose RMS passed 1.5x the
start), scales (mean gate norm scales, scalar_sqrt). Frozen engrams are skipped.
"""
import argparse
import glob
import json
import os
import re
import time

from micro_engram.stats import format_stats, weight_stats
from micro_engram.weights import CONFIG_NAME, engram_specs, load_engram_weights, resolve_weights_path

_CKPT = re.compile(r"checkpoint-(\d+)$")
_STEP_PT = re.compile(r"micro_engram-step(\d+)\.pt$")


def _conf(path):
    if path and os.path.isfile(path):
        with open(path) as f:
            return json.load(f)
    return {}


def checkpoint_weights(ckpt):
    """Where one checkpoint folder keeps its engram tensors (None if nowhere)."""
    cp = os.path.join(ckpt, CONFIG_NAME)
    w = resolve_weights_path(_conf(cp), cp)
    if w and os.path.exists(w):
        return w
    for cand in ("pytorch_model_fsdp_0", "micro_engram.pt"):
        if os.path.exists(os.path.join(ckpt, cand)):
            return os.path.join(ckpt, cand)
    return ckpt if glob.glob(os.path.join(ckpt, "*.safetensors")) else None


def find_snapshots(path):
    """[(step or None, weights, config path)], oldest first; only complete checkpoints
    (trainer_state.json is written last)."""
    path = os.path.abspath(path)
    if not os.path.isdir(path):
        return [(None, path, None)]
    m = _CKPT.search(path)
    if m:
        return [(int(m.group(1)), checkpoint_weights(path), os.path.join(path, CONFIG_NAME))]
    snaps = []
    for ckpt in glob.glob(os.path.join(path, "checkpoint-*")):
        m = _CKPT.search(ckpt)
        if m and os.path.isfile(os.path.join(ckpt, "trainer_state.json")):
            w = checkpoint_weights(ckpt)
            if w:
                snaps.append((int(m.group(1)), w, os.path.join(ckpt, CONFIG_NAME)))
    for pt in glob.glob(os.path.join(path, "micro_engram-step*.pt")):
        snaps.append((int(_STEP_PT.search(pt).group(1)), pt, os.path.join(path, CONFIG_NAME)))
    if not snaps and checkpoint_weights(path):
        snaps.append((None, checkpoint_weights(path), os.path.join(path, CONFIG_NAME)))
    return sorted(snaps, key=lambda s: s[0] or 0)


def stats_line(step, weights, conf_path, override=None):
    """One line per trained engram of a snapshot."""
    path = override or conf_path
    conf = _conf(override) or _conf(conf_path)
    if not conf:
        path = os.path.join(os.path.dirname(os.path.dirname(weights)), CONFIG_NAME)
        conf = _conf(path)
    label = f"step {step:>6}" if step is not None else os.path.basename(weights)
    specs = engram_specs(conf, path) if conf else [{"layer": None, "orders": (2, 3), "num_heads": None,
                                                     "weights": None, "frozen": False}]
    several = len(specs) > 1
    lines = []
    for spec in specs:
        if spec.get("frozen"):
            continue
        src = (spec["weights"] or weights) if several else weights
        sd = load_engram_weights(src, layer=spec["layer"] if several else None)
        tag = f"{label} L{spec['layer']}" if several else label
        if not any(k.startswith("tables.") for k in sd):
            lines.append(f"{tag}: no engram tensors found")
            continue
        lines.append(f"{tag}  " + format_stats(weight_stats(sd, tuple(spec.get("orders") or (2, 3)),
                                                            spec.get("num_heads"))))
    return "\n".join(lines) or f"{label}: every engram is frozen"


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("path")
    ap.add_argument("--config", default=None)
    ap.add_argument("--all", action="store_true")
    ap.add_argument("--watch", type=float, default=0, metavar="SECONDS")
    args = ap.parse_args(argv)
    seen = set()
    while True:
        snaps = find_snapshots(args.path)
        if not snaps and not args.watch:
            raise SystemExit(f"no complete checkpoint with engram weights under {args.path}")
        for step, w, cp in (snaps if args.all or args.watch else snaps[-1:]):
            if (step, w) in seen:
                continue
            try:
                print(stats_line(step, w, cp, args.config), flush=True)
                seen.add((step, w))
            except Exception as e:  # noqa: BLE001 - e.g. rotated away while being read
                print(f"step {step}: could not read ({type(e).__name__}: {e}); will retry", flush=True)
        if not args.watch:
            return
        time.sleep(args.watch)


if __name__ == "__main__":
    main()
