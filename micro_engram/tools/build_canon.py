"""Token-merging map for the engram hash (reference: build_canon.py:46-158).

    python -m micro_engram.tools.build_canon --tokenizer MODEL --out canon.pt [--paper]

A token's merge key is its text, NFKC-normalised and lower-cased, with the leading space
marker kept, so "▁The" and "▁the" share a class but "▁the" and the bare piece "the" do not.
Each option merges more:
  --merge-space       drop the space marker from the key ("▁the" ~ "the")
  --strip-accents     drop combining diacritics U+0300-U+036F ("é" ~ "e")
  --merge-whitespace  every whitespace-only piece shares one class
  --paper             all three
  --protect FILE      names (one per line, # comments) whose own tokens never merge
Special, added and byte tokens (<0xNN>) never merge. The smallest id of a class stands for
it, which makes the map idempotent (canon[canon] == canon). The class count of every option
set is printed for comparison.
"""
import argparse
import random
import re
import unicodedata

import torch

SPACE_MARKS = ("▁", "Ġ")  # SentencePiece and byte-level BPE space markers
_BYTE = re.compile(r"^<0x[0-9A-Fa-f]{2}>$")
_VISIBLE_WS = {"▁": " ", "Ġ": " ", "Ċ": "\n", "ĉ": "\t"}
WHITESPACE_CLASS = "<whitespace>"
_LADDER = (("case only", (False, False, False)), ("+ space", (True, False, False)),
           ("+ accents", (True, True, False)), ("+ whitespace (paper)", (True, True, True)))


def _strip_marks(s):
    return unicodedata.normalize("NFKC", "".join(
        ch for ch in unicodedata.normalize("NFKD", s) if not 0x300 <= ord(ch) <= 0x36F))


def merge_key(piece, merge_space=False, accents=False, whitespace=False):
    """The class key of one tokenizer piece, or None when it has no text to merge on."""
    if whitespace:
        real = "".join(_VISIBLE_WS.get(ch, ch) for ch in piece)
        if real and real.isspace():
            return WHITESPACE_CLASS
    marker = ""
    if piece[:1] in SPACE_MARKS:
        marker, piece = "▁", piece[1:]
    body = unicodedata.normalize("NFKC", piece).lower()
    if accents:
        body = _strip_marks(body)
    if not body:
        return None
    return body if merge_space else marker + body


def read_names(path):
    with open(path, encoding="utf-8") as f:
        return [s.strip() for s in f if s.strip() and not s.lstrip().startswith("#")]


def name_token_ids(names, pieces):
    """(ids of tokens that are exactly a name, bare or space-marked; single-token names;
    names the tokenizer splits, which are left alone)."""
    where = {}
    for i, p in enumerate(pieces):
        if p is not None:
            where.setdefault(p, i)
    ids, single, split = set(), [], []
    for name in names:
        hits = [where[v] for v in [name] + [m + name for m in SPACE_MARKS] if v in where]
        if hits:
            ids.update(hits)
            single.append(name)
        else:
            split.append(name)
    return ids, single, split


def build(pieces, protected, vocab_size, merge_space=False, accents=False, whitespace=False):
    """(canon list of length vocab_size, {key: [ids]})."""
    canon = list(range(vocab_size))
    classes = {}
    for i, p in enumerate(pieces):
        if i in protected or p is None or _BYTE.match(p):
            continue
        key = merge_key(p, merge_space, accents, whitespace)
        if key is not None:
            classes.setdefault(key, []).append(i)
    for ids in classes.values():
        for i in ids:
            canon[i] = ids[0]
    return canon, classes


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--tokenizer", required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--vocab-size", type=int, default=262_144, help="model vocabulary (Gemma 4: 262144)")
    ap.add_argument("--merge-space", action="store_true")
    ap.add_argument("--strip-accents", action="store_true")
    ap.add_argument("--merge-whitespace", action="store_true")
    ap.add_argument("--paper", action="store_true", help="all three merges")
    ap.add_argument("--protect", action="append", default=[], metavar="FILE")
    args = ap.parse_args(argv)
    if args.paper:
        args.merge_space = args.strip_accents = args.merge_whitespace = True
    chosen = (args.merge_space, args.strip_accents, args.merge_whitespace)

    from transformers import AutoTokenizer

    tok = AutoTokenizer.from_pretrained(args.tokenizer)
    n = min(len(tok), args.vocab_size)
    pieces = tok.convert_ids_to_tokens(list(range(n)))
    protected = set(tok.get_added_vocab().values()) | set(tok.all_special_ids)
    print(f"tokenizer pieces: {n:,} | protected (special/added): {len(protected):,}")
    for path in args.protect:
        ids, single, split = name_token_ids(read_names(path), pieces)
        protected |= ids
        print(f"{path}: {len(single)} names kept apart ({len(ids)} tokens)")
        if split:
            print(f"  split by the tokenizer, left alone ({len(split)}): {', '.join(split)}")
    for label, flags in _LADDER:
        canon, _ = build(pieces, protected, args.vocab_size, *flags)
        k = len(set(canon[:n]))
        print(f"{label:22s}: {n:,} tokens -> {k:,} classes ({1 - k / n:.1%} fewer)"
              + ("  <- chosen" if flags == chosen else ""))
    canon, classes = build(pieces, protected, args.vocab_size, *chosen)
    print(f"\nchosen: merge_space={args.merge_space} strip_accents={args.strip_accents} "
          f"merge_whitespace={args.merge_whitespace}")
    if WHITESPACE_CLASS in classes:
        ws = classes[WHITESPACE_CLASS]
        print(f"whitespace class: {len(ws)} pieces, e.g. {[pieces[i] for i in ws[:8]]}")
    big = [ids for key, ids in classes.items() if len(ids) >= 3 and key != WHITESPACE_CLASS]
    print("\nsample of merged classes:")
    for ids in random.Random(0).sample(big, min(12, len(big))):
        print("   ", [pieces[i] for i in ids[:8]])
    t = torch.tensor(canon, dtype=torch.long)
    if not torch.equal(t[t], t):
        raise SystemExit("internal error: the map is not idempotent")
    torch.save(t, args.out)
    print(f"\nsaved {args.out}")


if __name__ == "__main__":
    main()
