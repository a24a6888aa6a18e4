"""Held-out log-probability of two served configurations (e.g. engram on and off) on the same
texts (the reference's eval_logprob.py answers the same question). Standard library only.

    python -m micro_engram.tools.eval_logprob run --url http://localhost:8000 --data heldout/ --out on.json
    python -m micro_engram.tools.eval_logprob compare on.json off.json

--data: a folder of .txt / .jsonl files, one .txt, or a .jsonl with "text" per line. Texts are
cut at paragraph breaks into pieces of about --max-chars, the same way on every run. A .jsonl
written by render_chat carries "spans": its texts are scored whole and only the tokens inside
the spans count (their positions come from the server's /tokenize). compare reports both
per-token losses, the share of chunks each side wins and a bootstrap 95% interval of the
loss difference.
"""
import argparse
import hashlib
import json
import math
import os
import random
from concurrent.futures import ThreadPoolExecutor

from ._http import Server


# ---------------------------------------------------------------------------- texts
def _files(path):
    if os.path.isdir(path):
        return [os.path.join(path, n) for n in sorted(os.listdir(path)) if n.endswith((".txt", ".jsonl"))]
    return [path]


def read_texts(path):
    """(source id, text) of every text under `path`."""
    for f in _files(path):
        name = os.path.basename(f)
        with open(f, encoding="utf-8") as fh:
            if f.endswith(".jsonl"):
                for i, line in enumerate(fh):
                    if line.strip():
                        yield f"{name}:{i}", json.loads(line)["text"]
            else:
                yield name, fh.read()


def chunk(text, max_chars):
    """Paragraph-aligned pieces of about max_chars characters (a longer paragraph stays whole)."""
    pieces, length = [[]], 0  # paragraphs of the piece being built, and its joined length
    for para in text.split("\n\n"):
        if not length:
            pieces[-1], length = [para], len(para)
        elif length + 2 + len(para) > max_chars:
            pieces.append([para])
            length = len(para)
        else:
            pieces[-1].append(para)
            length += 2 + len(para)
    joined = ["\n\n".join(p) for p in pieces]
    return [p for p in joined if p.strip()]


def load_span_rows(path):
    """render_chat rows with "spans" (those without spans are dropped), or None when `path` is
    not such a file."""
    if not (os.path.isfile(path) and path.endswith(".jsonl")):
        return None
    with open(path, encoding="utf-8") as f:
        rows = [{"id": f"{os.path.basename(path)}:{i}", "text": o["text"], "spans": o.get("spans")}
                for i, o in ((i, json.loads(line)) for i, line in enumerate(f) if line.strip())]
    with_spans = [r for r in rows if r["spans"]]
    if not with_spans:
        return None
    if len(with_spans) < len(rows):
        print(f"note: {len(rows) - len(with_spans)} lines without spans skipped")
    return with_spans


def load_chunks(path, max_chars, min_chars, prefix=""):
    rows = load_span_rows(path)
    if rows is not None:
        return rows
    out = []
    for src, text in read_texts(path):
        body = text.strip()
        if prefix and body.startswith(prefix):
            body = body[len(prefix):]
        out += [{"id": f"{src}#{i}", "text": prefix + piece} for i, piece in enumerate(chunk(body, max_chars))
                if len(piece) >= min_chars]
    return out


# ---------------------------------------------------------------------------- scoring
def _shared_prefix(a, b):
    n = 0
    while n < min(len(a), len(b)) and a[n] == b[n]:
        n += 1
    return n


def span_positions(server, piece, ids):
    """Token positions of `ids` that fall inside the piece's character spans: a boundary's
    position is the token count of the text before it (guarded by the common prefix with the
    whole text's tokens)."""
    text = piece["text"]

    def boundary(char):
        return len(ids) if char >= len(text) else _shared_prefix(server.tokenize(text[:char]), ids)

    positions = set()
    for a, b in piece["spans"]:
        positions.update(range(max(boundary(a), 1), boundary(b)))
    return positions


def score(server, piece):
    got = server.prompt_logprobs(piece["text"], return_ids=True)
    ids, lps = got["prompt_token_ids"], got["prompt_logprobs"]
    positions = sorted(span_positions(server, piece, ids)) if piece.get("spans") else range(1, len(ids))
    fingerprint = hashlib.sha1(json.dumps([ids, piece.get("spans")]).encode()).hexdigest()[:16]
    return {"id": piece["id"], "sum_logprob": sum(lps[j][str(ids[j])]["logprob"] for j in positions),
            "n_tokens": len(positions), "token_hash": fingerprint}


def cmd_run(args):
    server = Server(args.url, args.api_key, args.timeout)
    model = server.model(args.model)
    pieces = load_chunks(args.data, args.max_chars, args.min_chars, args.prefix)
    if not pieces:
        raise SystemExit(f"no text found in {args.data}")
    print(f"scoring {len(pieces)} chunks from {args.data} with '{model}' at {server.base} ...")
    scored = []
    with ThreadPoolExecutor(args.parallel) as pool:
        for r in pool.map(lambda p: score(server, p), pieces):
            scored.append(r)
            if len(scored) % 20 == 0 or len(scored) == len(pieces):
                print(f"  {len(scored)}/{len(pieces)}")
    tokens = sum(r["n_tokens"] for r in scored)
    loss = -sum(r["sum_logprob"] for r in scored) / tokens
    print(f"{model}: {tokens:,} tokens | loss {loss:.4f} | perplexity {math.exp(loss):.3f}")
    with open(args.out, "w") as f:
        json.dump({"model": model, "url": server.base, "data": args.data, "max_chars": args.max_chars,
                   "chunks": scored}, f, indent=1)
    print(f"saved {args.out}")


# ---------------------------------------------------------------------------- comparing
def _per_token_loss(rows):
    return -sum(r["sum_logprob"] for r in rows) / sum(r["n_tokens"] for r in rows)


def _bootstrap_interval(diffs, n_boot, seed):
    """95% interval of the token-weighted mean of per-chunk differences, resampling chunks."""
    rng = random.Random(seed)
    means = []
    for _ in range(n_boot):
        sample = [diffs[rng.randrange(len(diffs))] for _ in diffs]
        means.append(sum(d for d, _ in sample) / sum(n for _, n in sample))
    means.sort()
    return means[int(0.025 * n_boot)], means[int(0.975 * n_boot) - 1]


def compare_runs(a, b, n_boot=2000, seed=0):
    """Summary of two runs over their common, identically tokenized chunks."""
    b_by_id = {r["id"]: r for r in b["chunks"]}
    common = [(r, b_by_id[r["id"]]) for r in a["chunks"] if r["id"] in b_by_id]
    if not common:
        raise SystemExit("no chunks in common: the same --data and --max-chars on both runs?")
    mismatched = [x["id"] for x, y in common if x["token_hash"] != y["token_hash"]]
    pairs = [(x, y) for x, y in common if x["token_hash"] == y["token_hash"]]
    diffs = [(y["sum_logprob"] - x["sum_logprob"], x["n_tokens"]) for x, y in pairs]  # below 0: A better
    return {"pairs": len(pairs), "tokens": sum(x["n_tokens"] for x, _ in pairs),
            "loss_a": _per_token_loss([x for x, _ in pairs]), "loss_b": _per_token_loss([y for _, y in pairs]),
            "wins_a": sum(d < 0 for d, _ in diffs), "ci": _bootstrap_interval(diffs, n_boot, seed),
            "mismatched": mismatched}


def cmd_compare(args):
    runs = []
    for path in (args.a, args.b):
        with open(path) as f:
            runs.append(json.load(f))
    a, b = runs
    s = compare_runs(a, b)
    if s["mismatched"]:
        print(f"WARNING: {len(s['mismatched'])} chunks were tokenized differently, e.g. {s['mismatched'][:3]}; "
              "left out")
    la, lb = s["loss_a"], s["loss_b"]
    lo, hi = s["ci"]
    verdict = ("A is reliably better on this text" if hi < 0 else
               "B is reliably better on this text" if lo > 0 else
               "no reliable difference (more text, or the effect is small)")
    print(f"{s['pairs']} chunks, {s['tokens']:,} tokens\n")
    print(f"  A {a['model']:<32} loss {la:.4f}  perplexity {math.exp(la):.3f}   ({args.a})")
    print(f"  B {b['model']:<32} loss {lb:.4f}  perplexity {math.exp(lb):.3f}   ({args.b})")
    print(f"\n  A - B: loss {la - lb:+.4f} per token, perplexity {math.exp(la) / math.exp(lb) - 1:+.1%}")
    print(f"  A is better on {s['wins_a']}/{s['pairs']} chunks ({s['wins_a'] / s['pairs']:.0%})")
    print(f"  95% interval for the loss difference A - B: [{lo:+.4f}, {hi:+.4f}]\n  -> {verdict}")


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    run = sub.add_parser("run", help="score texts against one server")
    run.add_argument("--url", default="http://localhost:8000")
    run.add_argument("--api-key", default=os.environ.get("VLLM_API_KEY"))
    run.add_argument("--model", default=None)
    run.add_argument("--data", required=True)
    run.add_argument("--out", required=True)
    run.add_argument("--max-chars", type=int, default=6000)
    run.add_argument("--prefix", default="", help="text put before every chunk (e.g. the BOS token)")
    run.add_argument("--min-chars", type=int, default=200)
    run.add_argument("--parallel", type=int, default=8)
    run.add_argument("--timeout", type=float, default=600)
    cmp_ = sub.add_parser("compare", help="compare two saved runs")
    cmp_.add_argument("a")
    cmp_.add_argument("b")
    args = ap.parse_args(argv)
    (cmd_run if args.cmd == "run" else cmd_compare)(args)


if __name__ == "__main__":
    main()
