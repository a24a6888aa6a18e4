"""Engram weight statistics, for the trainer's periodic log line and for the engram_stats
tool that reads saved checkpoints.

The metric names are the log keys users already chart (Ready-Art/micro_engram_fork,
micro_engram/stats.py:1-84): per n-gram order `engram/table_rms_{n}g` (RMS over every value
of that order's tables) and `engram/rows_learned_{n}g` (share of rows whose own RMS has grown
past LEARNED_FACTOR x the N(0, INIT_STD) init), then `engram/out_abs_mean`,
`engram/key_abs_mean`, `engram/gate_in_abs_mean` and `engram/{q,k}_scale_{mean,dev}`.

Every reduction runs where the tensors live (the GPU during training); the host reads one
small vector at the end, so a stats step costs one synchronisation, not one per table.
"""
import re

import torch

INIT_STD = 0.02
LEARNED_FACTOR = 1.5

TABLE_KEY = re.compile(r"^tables\.(\d+)\.weight$")
# parameter name -> metric (both value.weight and the older up.weight are the output side)
ABS_MEAN_KEYS = {"value.weight": "out_abs_mean", "up.weight": "out_abs_mean", "key.weight": "key_abs_mean",
                 "down.weight": "gate_in_abs_mean"}
SCALE_KEYS = ("q_scale", "k_scale")


def plain(t):
    """A dense tensor without autograd; a DTensor contributes its local shard (a sample of
    rows, which is what a row-sharded rank holds)."""
    t = t.detach()
    return t.to_local() if hasattr(t, "to_local") else t


def _order_of(index, orders, per_order):
    return orders[min(index // per_order, len(orders) - 1)]


def weight_stats(named, orders=(2, 3), num_heads=None):
    """{metric: float} from {parameter name: tensor}; table i belongs to order
    orders[i // num_heads] (the module's order-major layout)."""
    tables = {}
    for key, t in named.items():
        hit = TABLE_KEY.match(key)
        if hit:
            tables[int(hit.group(1))] = plain(t)
    keys, vals = [], []
    if tables:
        per_order = num_heads or max(1, len(tables) // len(orders))
        by_order = {}
        for i in sorted(tables):
            by_order.setdefault(_order_of(i, orders, per_order), []).append(tables[i])
        for n in sorted(by_order):
            ts = [t.float() for t in by_order[n] if t.numel()]
            if ts:
                total_sq = torch.stack([t.square().sum() for t in ts]).sum()
                count = sum(t.numel() for t in ts)
                row_rms = torch.cat([t.square().mean(dim=1).sqrt() for t in ts])
                rms = (total_sq / count).sqrt()
                learned = (row_rms > LEARNED_FACTOR * INIT_STD).float().mean()
            else:
                rms = learned = torch.zeros(())
            keys += [f"engram/table_rms_{n}g", f"engram/rows_learned_{n}g"]
            vals += [rms, learned]
    for param, metric in ABS_MEAN_KEYS.items():
        if param in named:
            keys.append(f"engram/{metric}")
            vals.append(plain(named[param]).float().abs().mean())
    for name in SCALE_KEYS:
        if name in named:
            s = plain(named[name]).float()
            keys += [f"engram/{name}_mean", f"engram/{name}_dev"]
            vals += [s.mean(), (s - 1).abs().mean()]  # the mean hides ups and downs; |s - 1| does not
    if not vals:
        return {}
    dev = vals[0].device
    host = torch.stack([v.reshape(()).to(dev) for v in vals]).tolist()
    return dict(zip(keys, host))


def module_stats(engram):
    """weight_stats of a live MicroEngram: its own table rows when row-sharded, and the scales as
    the saved files store them (1 + the learned delta)."""
    named = dict(engram.named_parameters())
    for k, shard in enumerate(getattr(engram, "row_shards", None) or []):
        named[f"tables.{k}.weight"] = shard
    for name in getattr(engram, "DELTA_SCALES", ()):
        if name in named:
            named[name] = plain(named[name]).float() + 1
    heads = len(engram._table_orders) // len(engram.orders)
    return weight_stats(named, engram.orders, heads)


def _suffix(key):
    return key.rsplit("_", 1)[1]


def format_stats(stats):
    """One compact log line, e.g.
    'out|w| 0.00213  rms 2g 0.0231 3g 0.0225  learned 2g 41% 3g 18%'."""
    out = []
    if "engram/out_abs_mean" in stats:
        out.append(f"out|w| {stats['engram/out_abs_mean']:.5f}")
    for label, prefix, fmt in (("rms", "engram/table_rms_", "{:.4f}"), ("learned", "engram/rows_learned_", "{:.0%}")):
        items = [f"{_suffix(k)} {fmt.format(v)}" for k, v in stats.items() if k.startswith(prefix)]
        if items:
            out.append(label + " " + " ".join(items))
    if "engram/gate_mean" in stats:
        out.append(f"gate {stats['engram/gate_mean']:.3f} (>0.99: {stats['engram/gate_saturated']:.0%})")
    if "engram/q_scale_mean" in stats:
        out.append(f"scales |q-1| {stats['engram/q_scale_dev']:.2e} |k-1| {stats['engram/k_scale_dev']:.2e}")
    return "  ".join(out)
