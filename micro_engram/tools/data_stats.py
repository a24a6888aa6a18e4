"""How much of a prepared dataset would the engram learn from, and how crowded would its
tables be (reference: engram_data_stats.py:25-125).

    python -m micro_engram.tools.data_stats PREPARED_DIR [--max-tokens N] [--orders 2,3,4]
        [--canon canon.pt] [--sizes 1048576,4194304]

Reads an Axolotl-style prepared dataset (input_ids, labels with -100 = masked). Position t
counts as trained when token t+1 is trained (the engram output at t predicts t+1). For each
order: distinct n-grams, those seen >= 3 times ("worth memorizing"), those only in masked
text, and the worth-memorizing load per row for each candidate table size. N-gram keys are
exact for up to 3 ids (base 2^18 digits) and a 64-bit mix (the SplitMix64 finaliser of
Steele, Lea and Flood 2014, applied per id) for longer ones.
"""
import argparse

import numpy as np

V = 1 << 18
ORDERS = (2, 3)
TABLE_SIZES = (65_536, 262_144, 1_048_576)
MIN_REPEATS = 3


def _mix64(x):
    x = x ^ (x >> np.uint64(30))
    x = x * np.uint64(0xBF58476D1CE4E5B9)
    x = x ^ (x >> np.uint64(27))
    x = x * np.uint64(0x94D049BB133111EB)
    return x ^ (x >> np.uint64(31))


def ngram_keys(ids, n):
    """int64 key of every n-gram ending at positions n-1 .. T-1."""
    T = len(ids)
    if n <= 3:
        key = np.zeros(T - n + 1, dtype=np.int64)
        for i in range(n):  # digit i = the token i places back
            key += ids[n - 1 - i:T - i].astype(np.int64) * (V ** i)
        return key
    with np.errstate(over="ignore"):
        h = np.zeros(T - n + 1, dtype=np.uint64)
        for i in range(n):
            h = _mix64(h + ids[n - 1 - i:T - i].astype(np.uint64) + np.uint64(i + 1))
    return h.view(np.int64)


def collect(rows, max_tokens, orders=ORDERS, canon=None):
    """(keys {n: [arrays]}, trained flags {n: [arrays]}, positions, trained positions, rows)."""
    keys = {n: [] for n in orders}
    sup = {n: [] for n in orders}
    total = trained = used = 0
    for ids, labels in rows:
        ids = np.asarray(ids, dtype=np.int64)
        labels = np.asarray(labels, dtype=np.int64)
        if canon is not None:
            ids = canon[np.clip(ids, 0, len(canon) - 1)]
        T = len(ids)
        if T < max(orders) + 1:
            continue
        nxt = np.zeros(T, dtype=bool)
        nxt[:-1] = labels[1:] != -100
        total += T
        trained += int(nxt.sum())
        used += 1
        for n in orders:
            keys[n].append(ngram_keys(ids, n))
            sup[n].append(nxt[n - 1:])
        if total >= max_tokens:
            break
    return keys, sup, total, trained, used


def report(keys, sup, sizes, out=print):
    for n in keys:
        k = np.concatenate(keys[n])
        s = np.concatenate(sup[n])
        uniq, counts = np.unique(k, return_counts=True)
        seen_trained = np.unique(k[s])
        pos = np.clip(np.searchsorted(seen_trained, k), 0, max(len(seen_trained) - 1, 0))
        never = float(np.mean(seen_trained[pos] != k)) if len(seen_trained) else 1.0
        only_masked = len(uniq) - len(seen_trained)
        worth = int((counts >= MIN_REPEATS).sum())
        out(f"--- {n}-grams ---")
        out(f"distinct: {len(uniq):,}")
        out(f"seen at least {MIN_REPEATS}x (worth memorizing): {worth:,}")
        out(f"distinct that only occur in masked text: {only_masked:,} ({only_masked / max(len(uniq), 1):.1%})")
        out(f"positions whose n-gram is never trained directly: {never:.1%}")
        out("worth-memorizing n-grams per table row:")
        for m in sizes:
            out(f"    {m:>9,} rows -> {worth / m:6.2f} per row")
        out("")


def _ints(text):
    return tuple(int(x) for x in text.split(","))


def _load_canon(path):
    if not path:
        return None
    import torch

    return torch.load(path, map_location="cpu").long().numpy()


def _prepared_rows(path):
    """(input_ids, labels) of every sample of a prepared dataset folder (its train split), shuffled."""
    from datasets import DatasetDict, load_from_disk

    ds = load_from_disk(path)
    if isinstance(ds, DatasetDict):
        ds = ds["train" if "train" in ds else next(iter(ds.keys()))]
    missing = {"input_ids", "labels"} - set(ds.column_names)
    if missing:
        raise SystemExit(f"need columns input_ids and labels, found {ds.column_names}")
    ds = ds.select_columns(["input_ids", "labels"]).shuffle(seed=0)
    for batch in ds.iter(batch_size=1000):
        yield from zip(batch["input_ids"], batch["labels"])


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("path")
    ap.add_argument("--max-tokens", type=int, default=50_000_000)
    ap.add_argument("--orders", default="2,3", type=_ints)
    ap.add_argument("--sizes", default=",".join(map(str, TABLE_SIZES)), type=_ints)
    ap.add_argument("--canon", default=None)
    args = ap.parse_args(argv)
    keys, sup, total, trained, used = collect(_prepared_rows(args.path), args.max_tokens, args.orders,
                                              _load_canon(args.canon))
    print(f"\nsampled {used:,} samples, {total:,} tokens")
    print(f"positions with a trained next token: {trained / max(total, 1):.1%}\n")
    report(keys, sup, args.sizes)
    print("Counts come from the sample (a bigger sample finds more distinct n-grams). About 1 per row or fewer "
          "is light sharing, 5+ heavy.")


if __name__ == "__main__":
    main()
