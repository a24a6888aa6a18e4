"""Where does the engram push? Score one reply token by token with the engram on and off
and colour each token by the change (reference: engram_token_diff.py:84-187).

    python -m micro_engram.tools.token_diff run --url URL --messages chat.json --reply reply.txt --out on.json
    (serve the other config)
    python -m micro_engram.tools.token_diff run --url URL --messages chat.json --reply reply.txt --out off.json
    python -m micro_engram.tools.token_diff render on.json off.json --out diff.html

--messages: JSON chat before the reply (the server applies its chat template), or
--context: the raw prompt text. The reply is scored as token ids appended to the context, so
both runs score the same tokens. render prints the largest pushes both ways and writes an
HTML heat map (green: more likely with the engram, red: less; hover for probabilities).
"""
import argparse
import html
import json
import math
import os

from ._http import Server


def _read(path):
    with open(path, encoding="utf-8") as f:
        return f.read()


def cmd_run(args):
    server = Server(args.url, args.api_key, args.timeout)
    model = server.model(args.model)
    if args.messages:
        msgs = json.loads(_read(args.messages))
        if not isinstance(msgs, list) or not all(isinstance(m, dict) and "role" in m for m in msgs):
            raise SystemExit(f"{args.messages}: expected a JSON list of {{'role': ..., 'content': ...}}")
        if msgs and msgs[-1]["role"] == "assistant":
            raise SystemExit(f"{args.messages}: the last message is the assistant's; the reply goes in --reply")
        ctx = server.tokenize(messages=msgs, add_generation_prompt=True)
    else:
        ctx = server.tokenize(prompt=_read(args.context), add_special_tokens=True)
    text = _read(args.reply)
    reply = server.tokenize(prompt=text.strip() if args.strip else text, add_special_tokens=False)
    if not reply:
        raise SystemExit(f"{args.reply} is empty")
    lps = server.prompt_logprobs(ctx + reply)["prompt_logprobs"]
    tokens = []
    for pos, tok in enumerate(reply, start=len(ctx)):
        e = lps[pos][str(tok)]
        tokens.append({"id": tok, "text": e.get("decoded_token") or f"<{tok}>", "logprob": e["logprob"]})
    mean = sum(t["logprob"] for t in tokens) / len(tokens)
    print(f"{model}: {len(tokens)} reply tokens after {len(ctx)} context tokens | mean log-prob {mean:.4f} | "
          f"perplexity {math.exp(-mean):.3f}")
    with open(args.out, "w", encoding="utf-8") as f:
        json.dump({"model": model, "url": server.base, "context_tokens": len(ctx), "context_ids": ctx,
                   "tokens": tokens}, f, ensure_ascii=False, indent=1)
    print(f"saved {args.out}")


def colour(d, scale):
    """Green for d > 0, red for d < 0, transparent near 0; full colour at |d| = scale."""
    a = min(abs(d) / scale, 1.0)
    if a <= 0.02:
        return "transparent"
    return f"rgba(22, 163, 74, {a:.3f})" if d > 0 else f"rgba(220, 38, 38, {a:.3f})"


def _visible(text):
    return text.replace("\n", "↵\n").replace(" ", "·") if not text.strip() else text


def diff_rows(on, off):
    if on["context_ids"] != off["context_ids"] or [t["id"] for t in on["tokens"]] != [t["id"] for t in off["tokens"]]:
        raise SystemExit("the two runs scored different tokens (different text, tokenizer or chat template)")
    return [{"text": a["text"], "on": a["logprob"], "off": b["logprob"], "d": a["logprob"] - b["logprob"]}
            for a, b in zip(on["tokens"], off["tokens"])]


def page(rows, scale):
    n = len(rows)
    lo_on, lo_off = -sum(r["on"] for r in rows) / n, -sum(r["off"] for r in rows) / n
    helped = sum(r["d"] > 0.05 for r in rows)
    hurt = sum(r["d"] < -0.05 for r in rows)
    spans = "".join(
        f'<span style="background:{colour(r["d"], scale)}" title="'
        + html.escape(f"with engram {math.exp(r['on']):.1%} | without {math.exp(r['off']):.1%} | "
                      f"log-prob {r['d']:+.2f}")
        + f'">{html.escape(_visible(r["text"]))}</span>' for r in rows)
    return (
        "<!doctype html><html lang=\"en\"><head><meta charset=\"utf-8\"><title>Engram token diff</title>"
        "<style>body{font:16px/1.7 system-ui,sans-serif;max-width:860px;margin:24px auto;padding:0 16px}"
        ".text{white-space:pre-wrap;word-wrap:break-word;background:#f6f8fa;border-radius:8px;padding:16px}"
        ".text span{border-radius:3px}.meta{color:#59636e;font-size:.9rem}"
        "@media (prefers-color-scheme: dark){body{background:#0d1117;color:#e6edf3}.text{background:#161b22}}"
        "</style></head><body><h1>Where the engram pushes</h1>"
        f"<p class=\"meta\">{n} tokens &middot; loss with engram {lo_on:.4f}, without {lo_off:.4f} &middot; "
        f"more likely with the engram: {helped}, less likely: {hurt} &middot; full colour at &plusmn;{scale:g} "
        f"log-prob</p><p><span style=\"background:{colour(scale, scale)}\">more likely</span> "
        f"<span style=\"background:{colour(-scale, scale)}\">less likely</span></p>"
        f"<div class=\"text\">{spans}</div></body></html>\n")


def cmd_render(args):
    with open(args.on, encoding="utf-8") as f:
        on = json.load(f)
    with open(args.off, encoding="utf-8") as f:
        off = json.load(f)
    rows = diff_rows(on, off)
    n = len(rows)
    lo_on, lo_off = -sum(r["on"] for r in rows) / n, -sum(r["off"] for r in rows) / n
    print(f"{n} tokens | loss with engram {lo_on:.4f}, without {lo_off:.4f} "
          f"(perplexity {math.exp(lo_on):.3f} vs {math.exp(lo_off):.3f})")
    helped = sum(r["d"] > 0.05 for r in rows)
    hurt = sum(r["d"] < -0.05 for r in rows)
    print(f"tokens the engram made clearly more likely: {helped} ({helped / n:.0%}), less likely: {hurt} "
          f"({hurt / n:.0%})")

    def around(i):
        left = "".join(r["text"] for r in rows[max(0, i - 6):i])
        return (left[-40:] + "[" + rows[i]["text"] + "]").replace("\n", " ")

    order = sorted(range(n), key=lambda i: rows[i]["d"])
    k = min(args.top, n)
    print("\nbiggest pushes TOWARD the text (on - off log-prob; prob off -> on):")
    for i in reversed(order[-k:]):
        r = rows[i]
        print(f"  {r['d']:+.2f}  {math.exp(r['off']):6.1%} -> {math.exp(r['on']):6.1%}   {around(i)}")
    print("\nbiggest pushes AWAY from the text:")
    for i in order[:k]:
        r = rows[i]
        print(f"  {r['d']:+.2f}  {math.exp(r['off']):6.1%} -> {math.exp(r['on']):6.1%}   {around(i)}")
    with open(args.out, "w", encoding="utf-8") as f:
        f.write(page(rows, args.scale))
    print(f"\nwrote {args.out}")


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    r = sub.add_parser("run")
    r.add_argument("--url", default="http://localhost:8000")
    r.add_argument("--api-key", default=os.environ.get("VLLM_API_KEY"))
    r.add_argument("--model", default=None)
    src = r.add_mutually_exclusive_group(required=True)
    src.add_argument("--messages")
    src.add_argument("--context")
    r.add_argument("--reply", required=True)
    r.add_argument("--strip", action="store_true")
    r.add_argument("--out", required=True)
    r.add_argument("--timeout", type=float, default=600)
    c = sub.add_parser("render")
    c.add_argument("on")
    c.add_argument("off")
    c.add_argument("--out", default="engram_diff.html")
    c.add_argument("--top", type=int, default=15)
    c.add_argument("--scale", type=float, default=2.0)
    args = ap.parse_args(argv)
    (cmd_run if args.cmd == "run" else cmd_render)(args)


if __name__ == "__main__":
    main()
