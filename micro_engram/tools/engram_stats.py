"""Engram weight statistics of checkpoints on disk (CPU only, so it can run beside a training
job; the reference's engram_stats.py reports the same columns).

    python -m micro_engram.tools.engram_stats OUTPUT_DIR            # newest complete checkpoint
    python -m micro_engram.tools.engram_stats OUTPUT_DIR --all      # every checkpoint on disk
    python -m micro_engram.tools.engram_stats OUTPUT_DIR --watch 120
    python -m micro_engram.tools.engram_stats micro_engram.pt --config micro_engram_config.json

Columns: out|w| (mean |weight| of the output projection, value or ple's up; 0 = untrained),
rms Ng (RMS of the N-gram tables, which start at 0.02), learned Ng (share of rows whose RMS
passed 1.5x the start), scales (gate norm scales, scalar_sqrt). Frozen engrams are skipped.
A checkpoint counts once its trainer_state.json (written last) exists.
"""
import argparse
import glob
import json
import os
import re
import time
from typing import NamedTuple, Optional

from micro_engram.stats import format_stats, weight_stats
from micro_engram.weights import CONFIG_NAME, engram_specs, load_engram_weights, resolve_weights_path

CHECKPOINT = re.compile(r"checkpoint-(\d+)$")
STEP_FILE = re.compile(r"micro_engram-step(\d+)\.pt$")
# where a checkpoint may hold its engram when its config names no weights
FALLBACK_NAMES = ("pytorch_model_fsdp_0", "micro_engram.pt")


class Snapshot(NamedTuple):
    step: Optional[int]
    weights: str
    config: Optional[str]


def _read_json(path):
    if not path or not os.path.isfile(path):
        return {}
    with open(path) as f:
        return json.load(f)


def checkpoint_weights(folder):
    """The engram tensors of one checkpoint folder: its config's weights, a known file name, or
    the folder itself when it holds safetensors; None when none exist."""
    conf_path = os.path.join(folder, CONFIG_NAME)
    named = resolve_weights_path(_read_json(conf_path), conf_path)
    if named and os.path.exists(named):
        return named
    for name in FALLBACK_NAMES:
        if os.path.exists(os.path.join(folder, name)):
            return os.path.join(folder, name)
    return folder if glob.glob(os.path.join(folder, "*.safetensors")) else None


def _complete_checkpoints(run):
    for folder in glob.glob(os.path.join(run, "checkpoint-*")):
        hit = CHECKPOINT.search(folder)
        weights = checkpoint_weights(folder) if hit else None
        if hit and weights and os.path.isfile(os.path.join(folder, "trainer_state.json")):
            yield Snapshot(int(hit.group(1)), weights, os.path.join(folder, CONFIG_NAME))


def find_snapshots(path):
    """[Snapshot] of `path` (a run folder, one checkpoint, or a weights file), oldest first."""
    path = os.path.abspath(path)
    if not os.path.isdir(path):
        return [Snapshot(None, path, None)]
    hit = CHECKPOINT.search(path)
    if hit:
        return [Snapshot(int(hit.group(1)), checkpoint_weights(path), os.path.join(path, CONFIG_NAME))]
    found = list(_complete_checkpoints(path))
    found += [Snapshot(int(STEP_FILE.search(pt).group(1)), pt, os.path.join(path, CONFIG_NAME))
              for pt in glob.glob(os.path.join(path, "micro_engram-step*.pt"))]
    if not found and checkpoint_weights(path):
        found.append(Snapshot(None, checkpoint_weights(path), os.path.join(path, CONFIG_NAME)))
    return sorted(found, key=lambda s: s.step or 0)


def _specs(weights, conf_path, override):
    """(engram specs, whether there are several) for a snapshot."""
    for path in (override, conf_path, os.path.join(os.path.dirname(os.path.dirname(weights)), CONFIG_NAME)):
        conf = _read_json(path)
        if conf:
            specs = engram_specs(conf, path)
            return specs, len(specs) > 1
    return [{"layer": None, "orders": (2, 3), "num_heads": None, "weights": None, "frozen": False}], False


def stats_line(step, weights, conf_path, override=None):
    """The report of one snapshot: one line per trained engram."""
    label = f"step {step:>6}" if step is not None else os.path.basename(weights)
    specs, several = _specs(weights, conf_path, override)
    lines = []
    for spec in (s for s in specs if not s.get("frozen")):
        source = (spec["weights"] or weights) if several else weights
        sd = load_engram_weights(source, layer=spec["layer"] if several else None)
        tag = f"{label} L{spec['layer']}" if several else label
        if any(k.startswith("tables.") for k in sd):
            stats = weight_stats(sd, tuple(spec.get("orders") or (2, 3)), spec.get("num_heads"))
            lines.append(f"{tag}  {format_stats(stats)}")
        else:
            lines.append(f"{tag}: no engram tensors found")
    return "\n".join(lines) if lines else f"{label}: every engram is frozen"


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("path")
    ap.add_argument("--config", default=None, help="the run config, when the weights have none beside them")
    ap.add_argument("--all", action="store_true", help="every checkpoint, not only the newest")
    ap.add_argument("--watch", type=float, default=0, metavar="SECONDS", help="keep reporting new checkpoints")
    args = ap.parse_args(argv)
    reported = set()
    while True:
        snaps = find_snapshots(args.path)
        if not snaps and not args.watch:
            raise SystemExit(f"no complete checkpoint with engram weights under {args.path}")
        for snap in (snaps if (args.all or args.watch) else snaps[-1:]):
            if (snap.step, snap.weights) in reported:
                continue
            try:
                print(stats_line(*snap, args.config), flush=True)
                reported.add((snap.step, snap.weights))
            except Exception as e:  # noqa: BLE001 - a checkpoint rotated away mid-read: try again later
                print(f"step {snap.step}: could not read ({type(e).__name__}: {e}); will retry", flush=True)
        if not args.watch:
            return
        time.sleep(args.watch)


if __name__ == "__main__":
    main()
