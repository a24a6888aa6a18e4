"""Check our tokenization of a YAML's datasets against an Axolotl prepared dataset made from the
same YAML (the reference's compare_axolotl_data.py covers the same question).

    python -m micro_engram.tools.compare_axolotl CONFIG.yaml AXOLOTL_PREPARED_DIR [--n 200]

Axolotl drops some samples (too long, nothing trained), so samples are paired by their token
sequence (hash of the bytes) before the trained-token masks are compared. The exit code is 0
only when every compared sample has a partner with the same mask. When differences matter,
train with `axolotl_prepared_dataset: <that folder>`.
"""
import argparse
import hashlib
import sys
from dataclasses import dataclass, field

import numpy as np


def _key(tokens):
    return hashlib.blake2b(np.ascontiguousarray(tokens, dtype=np.int64).tobytes(), digest_size=16).digest()


@dataclass
class Comparison:
    compared: int = 0
    identical: int = 0
    mask_differs: list = field(default_factory=list)  # (our index, their index)
    unmatched: list = field(default_factory=list)     # our indices without a partner

    @property
    def clean(self):
        return not self.mask_differs and not self.unmatched


def compare(ours, theirs, n=0):
    """Pair each of our first `n` samples (0: all) with an Axolotl sample of the same tokens and
    compare the trained masks."""
    partner = {}
    for j in range(len(theirs)):
        partner.setdefault(_key(theirs.get(j)[0]), j)
    res = Comparison(compared=len(ours) if not n else min(n, len(ours)))
    for i in range(res.compared):
        tokens, mask = ours.get(i)
        j = partner.get(_key(tokens))
        if j is None:
            res.unmatched.append(i)
        elif np.array_equal(mask, theirs.get(j)[1]):
            res.identical += 1
        else:
            res.mask_differs.append((i, j))
    return res


def _show_mask_difference(tok, ours, theirs, i, j):
    tokens, mask = ours.get(i)
    other = theirs.get(j)[1]
    where = np.flatnonzero(mask != other)
    lo, hi = max(0, where[0] - 5), min(len(tokens), where[0] + 15)
    marks = [f"{tok.decode([int(tokens[k])])!r}{'+' if mask[k] else ''}{'A' if other[k] else ''}" for k in range(lo, hi)]
    return (f"\n sample {i}: {len(where)} tokens differ, first at {where[0]} (+ = we train, A = Axolotl trains):\n  "
            + " ".join(marks))


def report(res, ours, theirs, tok):
    lines = [f"ours: {len(ours):,} samples, Axolotl: {len(theirs):,}; compared {res.compared:,}",
             f"  identical tokens + mask: {res.identical:,}",
             f"  same tokens, different trained mask: {len(res.mask_differs):,}",
             f"  tokens not found in Axolotl's data: {len(res.unmatched):,}"]
    lines += [_show_mask_difference(tok, ours, theirs, i, j) for i, j in res.mask_differs[:3]]
    for i in res.unmatched[:3]:
        tokens = ours.get(i)[0]
        lines.append(f"\n sample {i} not in Axolotl's data ({len(tokens)} tokens): "
                     f"{tok.decode(tokens[:40].tolist())!r}...")
    return "\n".join(lines)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("config")
    ap.add_argument("axolotl_folder")
    ap.add_argument("--n", type=int, default=0, help="only our first N samples (0: all)")
    args = ap.parse_args(argv)
    from transformers import AutoTokenizer

    from micro_engram.train.config import load_config
    from micro_engram.train.data import read_axolotl_prepared, tokenize_all

    cfg = load_config(args.config)
    tok_path = cfg.tokenizer_config or cfg.base_model
    tok = AutoTokenizer.from_pretrained(tok_path)
    ours, theirs = tokenize_all(cfg, tok, tok_path), read_axolotl_prepared(args.axolotl_folder)
    res = compare(ours, theirs, args.n)
    print(report(res, ours, theirs, tok))
    sys.exit(0 if res.clean else 1)


if __name__ == "__main__":
    main()
