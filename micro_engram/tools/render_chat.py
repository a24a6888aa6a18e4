"""Chat samples -> {"text", "spans"} lines for eval_logprob (reference: render_chat.py:49-119).

    python -m micro_engram.tools.render_chat --data convs.jsonl --tokenizer MODEL [--template T.jinja]
        [--kwargs JSON] [--n 80] [--seed 0] [--eot "<turn|>"] [--roles assistant] [--no-spans] --out out.jsonl

Each input line holds "messages" (role/content) or "conversations"/"conversation" (ShareGPT
from/value). --n conversations are drawn with a fixed seed; "spans" are the character spans
of the scored roles' turns (content through the end-of-turn token, not the role header).
"""
import argparse
import json
import random

ROLE = {"human": "user", "user": "user", "gpt": "assistant", "assistant": "assistant", "model": "assistant",
        "system": "system", "tool": "tool"}


def messages_of(obj):
    """[{role, content}] from a messages or ShareGPT record, else None."""
    for key in ("messages", "conversations", "conversation"):
        turns = obj.get(key)
        if isinstance(turns, list) and turns:
            out = []
            for t in turns:
                role, content = t.get("role", t.get("from")), t.get("content", t.get("value"))
                if role is None or content is None:
                    return None
                out.append({"role": ROLE.get(role, role), "content": content})
            return out
    return None


def render_rows(convs, render, roles, eot, no_spans=False):
    """Yield (row dict, had scorable spans)."""
    from micro_engram.train.data import chat_spans

    for msgs in convs:
        if no_spans:
            yield {"text": render(msgs)}, True
            continue
        try:
            text, spans = chat_spans(render, msgs, roles, eot)
        except ValueError:  # template not prefix-stable for this conversation: whole text, no spans
            yield {"text": render(msgs)}, False
            continue
        row = {"text": text}
        if spans:
            row["spans"] = [list(s) for s in spans]
        yield row, bool(spans)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--data", required=True)
    ap.add_argument("--tokenizer", required=True)
    ap.add_argument("--template", default=None)
    ap.add_argument("--kwargs", default="{}")
    ap.add_argument("--n", type=int, default=80)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--out", required=True)
    ap.add_argument("--eot", action="append", default=None)
    ap.add_argument("--roles", default="assistant")
    ap.add_argument("--no-spans", action="store_true")
    args = ap.parse_args(argv)
    from transformers import AutoTokenizer

    tok = AutoTokenizer.from_pretrained(args.tokenizer)
    if args.template:
        with open(args.template, encoding="utf-8") as f:
            tok.chat_template = f.read()
    kw = json.loads(args.kwargs)
    convs, skipped = [], 0
    with open(args.data, encoding="utf-8") as f:
        for line in f:
            if line.strip():
                m = messages_of(json.loads(line))
                if m is None:
                    skipped += 1
                else:
                    convs.append(m)
    if not convs:
        raise SystemExit(f"{args.data}: no conversations (expected 'messages' or 'conversations' per line)")
    picked = random.Random(args.seed).sample(convs, min(args.n, len(convs)))

    def render(m, add_generation_prompt=False):
        return tok.apply_chat_template(m, tokenize=False, add_generation_prompt=add_generation_prompt, **kw)

    roles = {r.strip() for r in args.roles.split(",") if r.strip()}
    chars = no_bos = unscored = 0
    with open(args.out, "w", encoding="utf-8") as g:
        for row, ok in render_rows(picked, render, roles, tuple(args.eot or ()), args.no_spans):
            unscored += not ok
            chars += len(row["text"])
            no_bos += bool(tok.bos_token) and not row["text"].startswith(tok.bos_token)
            g.write(json.dumps(row, ensure_ascii=False) + "\n")
    print(f"{len(picked)} of {len(convs)} conversations rendered to {args.out} (average "
          f"{chars / len(picked):,.0f} characters)" + (f"; {skipped} lines without a conversation skipped"
                                                       if skipped else ""))
    if unscored:
        print(f"note: {unscored} conversations have no scorable {sorted(roles)} turns (or the template is not "
              f"prefix-stable for them); eval_logprob skips them")
    if no_bos:
        print(f"note: {no_bos} texts do not start with {tok.bos_token!r}; pass --prefix \"{tok.bos_token}\" to "
              f"eval_logprob")


if __name__ == "__main__":
    main()
