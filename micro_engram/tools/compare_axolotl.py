"""Our tokenization of a YAML's datasets against an Axolotl prepared dataset for the same
YAML (reference: compare_axolotl_data.py:1-75).

    python -m micro_engram.tools.compare_axolotl CONFIG.yaml AXOLOTL_PREPARED_DIR [--n 200]

Samples are matched by their tokens (Axolotl drops some), then the trained-token masks are
compared. Exit code 0 only when every compared sample matches.
"""
import argparse
import sys

import numpy as np


def compare(ours, theirs, n=0):
    """(identical count, [(our idx, their idx) with a different mask], [our idx not found])."""
    by_tokens = {}
    for j in range(len(theirs)):
        t, _ = theirs.get(j)
        by_tokens.setdefault(t.tobytes(), []).append(j)
    n = len(ours) if not n else min(n, len(ours))
    same, diff, missing = 0, [], []
    for i in range(n):
        t, m = ours.get(i)
        hits = by_tokens.get(t.tobytes())
        if not hits:
            missing.append(i)
            continue
        if np.array_equal(m, theirs.get(hits[0])[1]):
            same += 1
        else:
            diff.append((i, hits[0]))
    return same, diff, missing, n


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("config")
    ap.add_argument("axolotl_folder")
    ap.add_argument("--n", type=int, default=0)
    args = ap.parse_args(argv)
    from transformers import AutoTokenizer

    from micro_engram.train.config import load_config
    from micro_engram.train.data import read_axolotl_prepared, tokenize_all

    cfg = load_config(args.config)
    tok_path = cfg.tokenizer_config or cfg.base_model
    tok = AutoTokenizer.from_pretrained(tok_path)
    ours = tokenize_all(cfg, tok, tok_path)
    theirs = read_axolotl_prepared(args.axolotl_folder)
    same, diff, missing, n = compare(ours, theirs, args.n)
    print(f"ours: {len(ours):,} samples, Axolotl: {len(theirs):,}; compared {n:,}")
    print(f"  identical tokens + mask: {same:,}")
    print(f"  same tokens, different trained mask: {len(diff):,}")
    print(f"  tokens not found in Axolotl's data: {len(missing):,}")
    for i, j in diff[:3]:
        t, m = ours.get(i)
        m2 = theirs.get(j)[1]
        d = np.nonzero(m != m2)[0]
        a, b = max(0, d[0] - 5), min(len(t), d[0] + 15)
        print(f"\n sample {i}: {len(d)} tokens differ, first at {d[0]} (+ = we train, A = Axolotl trains):")
        print("  " + " ".join(f"{tok.decode([int(t[k])])!r}{'+' if m[k] else ''}{'A' if m2[k] else ''}"
                              for k in range(a, b)))
    for i in missing[:3]:
        t, _ = ours.get(i)
        print(f"\n sample {i} not in Axolotl's data ({len(t)} tokens): {tok.decode(t[:40].tolist())!r}...")
    sys.exit(0 if not diff and not missing else 1)


if __name__ == "__main__":
    main()
