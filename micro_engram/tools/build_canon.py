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


def _parser():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--tokenizer", required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--vocab-size", type=int, default=262_144, help="model vocabulary (Gemma 4: 262144)")
    ap.add_argument("--merge-space", action="store_true")
    ap.add_argument("--strip-accents", action="store_true")
    ap.add_argument("--merge-whitespace", action="store_true")
    ap.add_argument("--paper", action="store_true", help="all three merges")
    ap.add_argument("--protect", action="append", default=[], metavar="FILE")
    return ap


def _tokenizer_pieces(path, vocab_size):
    """(pieces of the first min(len, vocab_size) ids, ids of special and added tokens)."""
    from transformers import AutoTokenizer

    tok = AutoTokenizer.from_pretrained(path)
    count = min(len(tok), vocab_size)
    keep = set(tok.all_special_ids).union(tok.get_added_vocab().values())
    return tok.convert_ids_to_tokens(list(range(count))), keep


def _protect_names(files, pieces, protected):
    for path in files:
        hit, kept, split = name_token_ids(read_names(path), pieces)
        protected.update(hit)
        print(f"{path}: {len(kept)} names kept apart ({len(hit)} tokens)")
        if split:
            print(f"  split by the tokenizer, left alone ({len(split)}): {', '.join(split)}")


def _report(pieces, protected, vocab_size, chosen):
    """The class count of every rung of the option ladder, the chosen one marked."""
    n = len(pieces)
    for label, flags in _LADDER:
        classes = len(set(build(pieces, protected, vocab_size, *flags)[0][:n]))
        mark = "  <- chosen" if flags == chosen else ""
        print(f"{label:22s}: {n:,} tokens -> {classes:,} classes ({1 - classes / n:.1%} fewer){mark}")


def _show_classes(pieces, classes):
    ws = classes.get(WHITESPACE_CLASS)
    if ws:
        print(f"whitespace class: {len(ws)} pieces, e.g. {[pieces[i] for i in ws[:8]]}")
    merged = [ids for key, ids in classes.items() if key != WHITESPACE_CLASS and len(ids) >= 3]
    print("\nsample of merged classes:")
    for ids in random.Random(0).sample(merged, min(12, len(merged))):
        print("   ", [pieces[i] for i in ids[:8]])


def main(argv=None):
    args = _parser().parse_args(argv)
    chosen = (True, True, True) if args.paper else (args.merge_space, args.strip_accents, args.merge_whitespace)
    pieces, protected = _tokenizer_pieces(args.tokenizer, args.vocab_size)
    print(f"tokenizer pieces: {len(pieces):,} | protected (special/added): {len(protected):,}")
    _protect_names(args.protect, pieces, protected)
    _report(pieces, protected, args.vocab_size, chosen)
    canon, classes = build(pieces, protected, args.vocab_size, *chosen)
    print(f"\nchosen: merge_space={chosen[0]} strip_accents={chosen[1]} merge_whitespace={chosen[2]}")
    _show_classes(pieces, classes)
    table = torch.tensor(canon, dtype=torch.long)
    if not torch.equal(table[table], table):
        raise SystemExit("internal error: the map is not idempotent")
    torch.save(table, args.out)
    print(f"\nsaved {args.out}")


if __name__ == "__main__":
    main()
