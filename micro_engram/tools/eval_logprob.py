"""Held-out log-prob of two served configs (e.g. engram on/off) on the same texts
(reference: eval_logprob.py:135-249). Standard library only.

    python -m micro_engram.tools.eval_logprob run --url http://localhost:8000 --data heldout/ --out on.json
    python -m micro_engram.tools.eval_logprob compare on.json off.json

--data: a folder of .txt/.jsonl, one .txt, or a .jsonl with "text" per line. Texts are cut
at paragraph breaks into pieces of about --max-chars, identically on every run. A .jsonl
from render_chat with "spans" is scored whole but only the span tokens count (positions
from the server's /tokenize). compare: per-token loss of both, win rate per chunk and a
bootstrap 95% interval of the loss difference.
"""
import argparse
import hashlib
import json
import math
import os
import random
from concurrent.futures import ThreadPoolExecutor

from ._http import Server


def read_texts(path):
    if os.path.isdir(path):
        for name in sorted(os.listdir(path)):
            if name.endswith((".txt", ".jsonl")):
                yield from read_texts(os.path.join(path, name))
    elif path.endswith(".jsonl"):
        with open(path, encoding="utf-8") as f:
            for i, line in enumerate(f):
                if line.strip():
                    yield f"{os.path.basename(path)}:{i}", json.loads(line)["text"]
    else:
        with open(path, encoding="utf-8") as f:
            yield os.path.basename(path), f.read()


def chunk(text, max_chars):
    """Paragraph-aligned pieces of about max_chars (one longer paragraph stays whole)."""
    pieces, cur = [], ""
    for para in text.split("\n\n"):
        if cur and len(cur) + 2 + len(para) > max_chars:
            pieces.append(cur)
            cur = para
        else:
            cur = cur + "\n\n" + para if cur else para
    if cur.strip():
        pieces.append(cur)
    return [p for p in pieces if p.strip()]


def load_span_rows(path):
    if not (os.path.isfile(path) and path.endswith(".jsonl")):
        return None
    rows = []
    with open(path, encoding="utf-8") as f:
        for i, line in enumerate(f):
            if line.strip():
                o = json.loads(line)
                rows.append({"id": f"{os.path.basename(path)}:{i}", "text": o["text"], "spans": o.get("spans")})
    if not any(r["spans"] for r in rows):
        return None
    kept = [r for r in rows if r["spans"]]
    if len(kept) < len(rows):
        print(f"note: {len(rows) - len(kept)} lines without spans skipped")
    return kept


def load_chunks(path, max_chars, min_chars, prefix=""):
    rows = load_span_rows(path)
    if rows is not None:
        return rows
    out = []
    for src, text in read_texts(path):
        text = text.strip()
        if prefix and text.startswith(prefix):
            text = text[len(prefix):]
        for i, piece in enumerate(chunk(text, max_chars)):
            if len(piece) >= min_chars:
                out.append({"id": f"{src}#{i}", "text": prefix + piece})
    return out


def _common_prefix(a, b):
    n = 0
    for x, y in zip(a, b):
        if x != y:
            break
        n += 1
    return n


def span_positions(server, piece, ids):
    """Token positions of `ids` inside the character spans (token counts of the text up to
    each boundary, guarded by the common prefix with the whole text's tokens)."""
    text, pos = piece["text"], set()
    for a, b in piece["spans"]:
        na = _common_prefix(server.tokenize(text[:a]), ids)
        nb = _common_prefix(server.tokenize(text[:b]), ids)
        if text[:b] == text:
            nb = len(ids)
        pos.update(range(max(na, 1), nb))
    return pos


def score(server, piece):
    ch = server.prompt_logprobs(piece["text"], return_ids=True)
    ids, lps = ch["prompt_token_ids"], ch["prompt_logprobs"]
    positions = sorted(span_positions(server, piece, ids)) if piece.get("spans") else range(1, len(ids))
    total = sum(lps[j][str(ids[j])]["logprob"] for j in positions)
    digest = hashlib.sha1(json.dumps([ids, piece.get("spans")]).encode()).hexdigest()[:16]
    return {"id": piece["id"], "sum_logprob": total, "n_tokens": len(positions), "token_hash": digest}


def cmd_run(args):
    server = Server(args.url, args.api_key, args.timeout)
    model = server.model(args.model)
    pieces = load_chunks(args.data, args.max_chars, args.min_chars, args.prefix)
    if not pieces:
        raise SystemExit(f"no text found in {args.data}")
    print(f"scoring {len(pieces)} chunks from {args.data} with '{model}' at {server.base} ...")
    done = []
    with ThreadPoolExecutor(args.parallel) as pool:
        for i, r in enumerate(pool.map(lambda p: score(server, p), pieces)):
            done.append(r)
            if (i + 1) % 20 == 0 or i + 1 == len(pieces):
                print(f"  {i + 1}/{len(pieces)}")
    n = sum(r["n_tokens"] for r in done)
    nll = -sum(r["sum_logprob"] for r in done) / n
    print(f"{model}: {n:,} tokens | loss {nll:.4f} | perplexity {math.exp(nll):.3f}")
    with open(args.out, "w") as f:
        json.dump({"model": model, "url": server.base, "data": args.data, "max_chars": args.max_chars,
                   "chunks": done}, f, indent=1)
    print(f"saved {args.out}")


def compare_runs(a, b, n_boot=2000, seed=0):
    """Summary dict of two runs' common, identically tokenized chunks."""
    rb = {r["id"]: r for r in b["chunks"]}
    pairs = [(r, rb[r["id"]]) for r in a["chunks"] if r["id"] in rb]
    if not pairs:
        raise SystemExit("no chunks in common: same --data and --max-chars on both runs?")
    bad = [x["id"] for x, y in pairs if x["token_hash"] != y["token_hash"]]
    pairs = [(x, y) for x, y in pairs if x["token_hash"] == y["token_hash"]]

    def loss(rows):
        return -sum(r["sum_logprob"] for r in rows) / sum(r["n_tokens"] for r in rows)

    la, lb = loss([x for x, _ in pairs]), loss([y for _, y in pairs])
    per = [(y["sum_logprob"] - x["sum_logprob"], x["n_tokens"]) for x, y in pairs]  # < 0: A better
    rng = random.Random(seed)
    boots = sorted(sum(d for d, _ in s) / sum(n for _, n in s)
                   for s in ([per[rng.randrange(len(per))] for _ in per] for _ in range(n_boot)))
    return {"pairs": len(pairs), "tokens": sum(x["n_tokens"] for x, _ in pairs), "loss_a": la, "loss_b": lb,
            "wins_a": sum(d < 0 for d, _ in per), "ci": (boots[int(0.025 * n_boot)], boots[int(0.975 * n_boot) - 1]),
            "mismatched": bad}


def cmd_compare(args):
    with open(args.a) as f:
        a = json.load(f)
    with open(args.b) as f:
        b = json.load(f)
    s = compare_runs(a, b)
    if s["mismatched"]:
        print(f"WARNING: {len(s['mismatched'])} chunks were tokenized differently, e.g. {s['mismatched'][:3]}; "
              f"left out")
    la, lb = s["loss_a"], s["loss_b"]
    print(f"{s['pairs']} chunks, {s['tokens']:,} tokens\n")
    print(f"  A {a['model']:<32} loss {la:.4f}  perplexity {math.exp(la):.3f}   ({args.a})")
    print(f"  B {b['model']:<32} loss {lb:.4f}  perplexity {math.exp(lb):.3f}   ({args.b})")
    print(f"\n  A - B: loss {la - lb:+.4f} per token, perplexity {math.exp(la) / math.exp(lb) - 1:+.1%}")
    print(f"  A is better on {s['wins_a']}/{s['pairs']} chunks ({s['wins_a'] / s['pairs']:.0%})")
    lo, hi = s["ci"]
    print(f"  95% interval for the loss difference A - B: [{lo:+.4f}, {hi:+.4f}]")
    print("  -> " + ("A is reliably better on this text" if hi < 0 else "B is reliably better on this text"
                     if lo > 0 else "no reliable difference (more text, or the effect is small)"))


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    r = sub.add_parser("run")
    r.add_argument("--url", default="http://localhost:8000")
    r.add_argument("--api-key", default=os.environ.get("VLLM_API_KEY"))
    r.add_argument("--model", default=None)
    r.add_argument("--data", required=True)
    r.add_argument("--out", required=True)
    r.add_argument("--max-chars", type=int, default=6000)
    r.add_argument("--prefix", default="")
    r.add_argument("--min-chars", type=int, default=200)
    r.add_argument("--parallel", type=int, default=8)
    r.add_argument("--timeout", type=float, default=600)
    c = sub.add_parser("compare")
    c.add_argument("a")
    c.add_argument("b")
    args = ap.parse_args(argv)
    (cmd_run if args.cmd == "run" else cmd_compare)(args)


if __name__ == "__main__":
    main()
