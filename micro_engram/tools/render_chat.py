"""Render chat samples into {"text", "spans"} lines for eval_logprob (the reference's
render_chat.py produces the same lines).

    python -m micro_engram.tools.render_chat --data convs.jsonl --tokenizer MODEL [--template T.jinja]
        [--kwargs JSON] [--n 80] [--seed 0] [--eot "<turn|>"] [--roles assistant] [--no-spans] --out out.jsonl

Each input line holds "messages" (role/content) or "conversations" / "conversation" (ShareGPT
from/value); the trainer's reader (micro_engram.train.data.messages_of) normalises them. --n
conversations are drawn with a fixed seed. "spans" are the character spans of the scored
roles' turns, located exactly as the trainer locates trained turns (chat_spans): content
through the end-of-turn token, not the role header.
"""
import argparse
import json
import random
import types


def messages_of(obj):
    """[{role, content}] of a messages or ShareGPT record, or None."""
    from micro_engram.train.data import messages_of as normalise

    defaults = types.SimpleNamespace(field_messages=None, message_property_mappings=None, roles=None)
    return normalise(obj, defaults)


def render_rows(convs, render, roles, eot, no_spans=False):
    """Yield (row, whether it has scorable spans) for each conversation."""
    from micro_engram.train.data import chat_spans

    for msgs in convs:
        if no_spans:
            yield {"text": render(msgs)}, True
            continue
        try:
            text, spans = chat_spans(render, msgs, roles, eot)
        except ValueError:  # the template is not prefix-stable for this one: score nothing in it
            yield {"text": render(msgs)}, False
            continue
        yield ({"text": text, "spans": [list(s) for s in spans]} if spans else {"text": text}), bool(spans)


def read_conversations(path):
    """(conversations, lines without one)."""
    with open(path, encoding="utf-8") as f:
        parsed = [messages_of(json.loads(line)) for line in f if line.strip()]
    found = [m for m in parsed if m is not None]
    return found, len(parsed) - len(found)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--data", required=True)
    ap.add_argument("--tokenizer", required=True)
    ap.add_argument("--template", default=None, help="a Jinja chat template file to use instead of the tokenizer's")
    ap.add_argument("--kwargs", default="{}", help="JSON keyword arguments for the chat template")
    ap.add_argument("--n", type=int, default=80, help="conversations to draw")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--out", required=True)
    ap.add_argument("--eot", action="append", default=None, help="end-of-turn marker (repeatable)")
    ap.add_argument("--roles", default="assistant", help="comma-separated roles to score")
    ap.add_argument("--no-spans", action="store_true", help="score the whole text")
    args = ap.parse_args(argv)
    from transformers import AutoTokenizer

    tok = AutoTokenizer.from_pretrained(args.tokenizer)
    if args.template:
        with open(args.template, encoding="utf-8") as f:
            tok.chat_template = f.read()
    template_kwargs = json.loads(args.kwargs)
    convs, skipped = read_conversations(args.data)
    if not convs:
        raise SystemExit(f"{args.data}: no conversations (expected 'messages' or 'conversations' per line)")
    picked = random.Random(args.seed).sample(convs, min(args.n, len(convs)))

    def render(msgs, add_generation_prompt=False):
        return tok.apply_chat_template(msgs, tokenize=False, add_generation_prompt=add_generation_prompt,
                                       **template_kwargs)

    roles = {r.strip() for r in args.roles.split(",") if r.strip()}
    totals = {"chars": 0, "unscored": 0, "no_bos": 0}
    with open(args.out, "w", encoding="utf-8") as out:
        for row, scorable in render_rows(picked, render, roles, tuple(args.eot or ()), args.no_spans):
            totals["chars"] += len(row["text"])
            totals["unscored"] += not scorable
            totals["no_bos"] += bool(tok.bos_token) and not row["text"].startswith(tok.bos_token)
            out.write(json.dumps(row, ensure_ascii=False) + "\n")
    note = f"; {skipped} lines without a conversation skipped" if skipped else ""
    print(f"{len(picked)} of {len(convs)} conversations rendered to {args.out} "
          f"(average {totals['chars'] / len(picked):,.0f} characters){note}")
    if totals["unscored"]:
        print(f"note: {totals['unscored']} conversations have no scorable {sorted(roles)} turns (or the template is "
              "not prefix-stable for them); eval_logprob skips them")
    if totals["no_bos"]:
        print(f"note: {totals['no_bos']} texts do not start with {tok.bos_token!r}; pass --prefix "
              f"\"{tok.bos_token}\" to eval_logprob")


if __name__ == "__main__":
    main()
