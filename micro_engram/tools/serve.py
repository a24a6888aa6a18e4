"""OpenAI-compatible HTTP server for an HF model with trained engram(s)
(reference: serve_engram.py:45-458).

    python -m micro_engram.tools.serve --model MERGED_DIR [--port 8000] [--host 127.0.0.1]
    python -m micro_engram.tools.serve --model BASE_DIR --engram-pt micro_engram.pt

Offers two model names: <name> (engram on) and <name>-noengram (same weights, engram off).
Endpoints: GET /v1/models, /health; POST /v1/chat/completions, /v1/completions (SSE with
"stream": true). One request runs at a time (the engram keeps the generation's history).
Chat replies put the thinking channel (<|channel>thought ... <channel|>) in
reasoning_content; --raw-thinking keeps the markers in content. Thinking defaults on
(enable_thinking + preserve_thinking, as in training); --no-thinking flips the default and a
request may override it in chat_template_kwargs. Stop strings cut the answer, never the
reasoning. A client that disconnects cancels its generation; each request logs prefill and
decode speed.
"""
import argparse
import json
import os
import threading
import time
import uuid
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from types import SimpleNamespace

import torch

THINK_START, THINK_END = "<|channel>thought", "<channel|>"
S = SimpleNamespace(model=None, tok=None, runner=None, name="model", template_kwargs={}, raw_thinking=False)
LOCK = threading.Lock()


# ------------------------------------------------------------------ text stream transforms
def split_reasoning(pieces, specials):
    """Raw text pieces (special tokens kept) -> ("reasoning" | "content", text) pairs.

    Text between THINK_START and THINK_END is reasoning; other special tokens are dropped;
    a newline right after either marker is dropped (the template writes one); text that could
    be the start of a marker is held back until it is decided."""
    drop = [s for s in specials if s and s not in (THINK_START, THINK_END, "<|channel>")]
    hold = max([len(THINK_START), len(THINK_END)] + [len(s) for s in drop]) - 1
    mode, buf, eat_newline = "content", "", False

    def clean(t):
        for s in drop:
            t = t.replace(s, "")
        return t

    try:
        for p in pieces:
            buf += p
            while True:
                if eat_newline and buf:
                    if buf.startswith("\n"):
                        buf = buf[1:]
                    eat_newline = False
                marker = THINK_START if mode == "content" else THINK_END
                at = buf.find(marker)
                if at < 0:
                    buf = clean(buf)
                    if len(buf) > hold:
                        yield mode, buf[:-hold] if hold else buf
                        buf = buf[-hold:] if hold else ""
                    break
                head = clean(buf[:at])
                if head:
                    yield mode, head
                buf = buf[at + len(marker):]
                mode = "reasoning" if mode == "content" else "content"
                eat_newline = True
        buf = clean(buf)
        if buf:
            yield mode, buf
    finally:
        if hasattr(pieces, "close"):
            pieces.close()


def keep_markers(tagged):
    """--raw-thinking: the thinking goes back into content with its markers."""
    inside = False
    for kind, text in tagged:
        if kind == "reasoning" and not inside:
            yield "content", THINK_START + "\n"
            inside = True
        elif kind == "content" and inside:
            yield "content", THINK_END
            inside = False
        yield "content", text
    if inside:
        yield "content", THINK_END


def with_stops(tagged, stops, cancel):
    """Cut the answer at the first stop string (reasoning is never cut); holds back answer
    text that could start a stop string."""
    if not stops:
        yield from tagged
        return
    hold = max(len(s) for s in stops) - 1
    buf = ""
    try:
        for kind, p in tagged:
            if kind != "content":
                yield kind, p
                continue
            buf += p
            cut = min((buf.find(s) for s in stops if s in buf), default=-1)
            if cut >= 0:
                yield "content", buf[:cut]
                cancel.cancelled = True
                return
            if len(buf) > hold:
                yield "content", buf[:len(buf) - hold]
                buf = buf[len(buf) - hold:]
        yield "content", buf
    finally:
        if hasattr(tagged, "close"):
            tagged.close()


def parse_stops(body):
    stop = body.get("stop")
    if not stop:
        return []
    return [stop] if isinstance(stop, str) else [s for s in stop if s]


def flat_content(c):
    if c is None:
        return ""
    if isinstance(c, str):
        return c
    if isinstance(c, list):  # OpenAI content parts
        return "".join(p.get("text", "") for p in c if isinstance(p, dict) and p.get("type") == "text")
    return str(c)


# ------------------------------------------------------------------ generation
class Cancel:
    """A stopping criterion that can be raised from outside; also times the tokens."""

    def __init__(self):
        self.cancelled = False
        self.steps = 0
        self.t_first = self.t_last = None

    def __call__(self, input_ids, scores, **kw):
        now = time.time()
        self.t_first = self.t_first or now
        self.t_last = now
        self.steps += 1
        return torch.full((input_ids.shape[0],), self.cancelled, dtype=torch.bool, device=input_ids.device)


def encode_chat(messages, template_kwargs):
    msgs = []
    for m in messages:
        msg = {"role": m.get("role", "user"), "content": flat_content(m.get("content"))}
        thought = m.get("reasoning_content") or m.get("reasoning")
        if thought:
            msg["reasoning_content"] = thought
        msgs.append(msg)
    text = S.tok.apply_chat_template(msgs, add_generation_prompt=True, tokenize=False, **template_kwargs)
    return S.tok(text, add_special_tokens=False, return_tensors="pt").input_ids  # the template has <bos>


def encode_text(prompt):
    bos = S.tok.bos_token or ""
    return S.tok(prompt, add_special_tokens=not (bos and prompt.startswith(bos)), return_tensors="pt").input_ids


def raw_pieces(body, input_ids, engram_on, cancel, max_new, skip_special=True):
    """Decoded text pieces of model.generate running in a worker thread (caller holds LOCK)."""
    from transformers import StoppingCriteriaList, TextIteratorStreamer

    S.runner.enabled = engram_on
    S.runner.reset()
    temp = 0.8 if body.get("temperature") is None else float(body["temperature"])
    kw = {"input_ids": input_ids, "attention_mask": torch.ones_like(input_ids), "max_new_tokens": max_new,
          "do_sample": temp > 0, "use_cache": True, "stopping_criteria": StoppingCriteriaList([cancel])}
    if temp > 0:
        kw["temperature"] = temp
        kw["top_p"] = float(body["top_p"]) if body.get("top_p") is not None else 1.0
        if body.get("top_k"):
            kw["top_k"] = int(body["top_k"])
        if body.get("min_p"):
            kw["min_p"] = float(body["min_p"])
    if body.get("repetition_penalty"):
        kw["repetition_penalty"] = float(body["repetition_penalty"])
    if body.get("seed") is not None:
        torch.manual_seed(int(body["seed"]))
    streamer = TextIteratorStreamer(S.tok, skip_prompt=True, skip_special_tokens=skip_special)
    kw["streamer"] = streamer
    failed = []

    def work():
        try:
            with torch.no_grad():
                S.model.generate(**kw)
        except Exception as e:  # noqa: BLE001 - surfaced to the request below
            failed.append(e)
            streamer.on_finalized_text("", stream_end=True)

    th = threading.Thread(target=work, daemon=True)
    th.start()
    try:
        yield from streamer
    finally:
        cancel.cancelled = True
        th.join()
    if failed:
        raise failed[0]


# ------------------------------------------------------------------ HTTP
class Handler(BaseHTTPRequestHandler):
    server_version = "engram-server"

    def log_message(self, fmt, *a):
        pass

    def _cors(self):
        self.send_header("Access-Control-Allow-Origin", "*")
        self.send_header("Access-Control-Allow-Headers", "*")
        self.send_header("Access-Control-Allow-Methods", "GET, POST, OPTIONS")

    def _json(self, obj, code=200):
        data = json.dumps(obj).encode()
        self.send_response(code)
        self.send_header("Content-Type", "application/json")
        self.send_header("Content-Length", str(len(data)))
        self._cors()
        self.end_headers()
        self.wfile.write(data)

    def do_OPTIONS(self):
        self.send_response(204)
        self._cors()
        self.end_headers()

    def do_GET(self):
        path = self.path.rstrip("/")
        if path in ("/v1/models", "/models"):
            now = int(time.time())
            self._json({"object": "list", "data": [{"id": n, "object": "model", "created": now, "owned_by": "local"}
                                                   for n in (S.name, S.name + "-noengram")]})
        elif path in ("/health", ""):
            self._json({"status": "ok"})
        else:
            self._json({"error": "not found"}, 404)

    def do_POST(self):
        path = self.path.rstrip("/")
        if path not in ("/v1/chat/completions", "/v1/completions"):
            return self._json({"error": "not found"}, 404)
        chat = path.endswith("chat/completions")
        try:
            body = json.loads(self.rfile.read(int(self.headers.get("Content-Length", 0))) or b"{}")
            if chat:
                tmpl = dict(S.template_kwargs, **(body.get("chat_template_kwargs") or {}))
                input_ids = encode_chat(body.get("messages", []), tmpl)
            else:
                p = body.get("prompt", "")
                input_ids = encode_text(p if isinstance(p, str) else "".join(p))
        except Exception as e:  # noqa: BLE001
            return self._json({"error": f"bad request: {e}"}, 400)
        name = body.get("model") or S.name
        engram_on = not name.endswith("-noengram")
        max_new = int(body.get("max_tokens") or body.get("max_completion_tokens") or 512)
        stream = bool(body.get("stream"))
        input_ids = input_ids.to(next(S.model.parameters()).device)
        rid = ("chatcmpl-" if chat else "cmpl-") + uuid.uuid4().hex[:24]
        created = int(time.time())

        def event(text, finish=None, first=False, kind="content"):
            if chat:
                delta = {"role": "assistant"} if first else {}
                if text:
                    delta["reasoning_content" if kind == "reasoning" else "content"] = text
                return {"id": rid, "object": "chat.completion.chunk", "created": created, "model": name,
                        "choices": [{"index": 0, "delta": delta, "finish_reason": finish}]}
            return {"id": rid, "object": "text_completion", "created": created, "model": name,
                    "choices": [{"index": 0, "text": text, "finish_reason": finish}]}

        t0 = time.time()
        answer, thought = "", ""
        with LOCK:
            cancel = Cancel()
            if chat:
                raw = raw_pieces(body, input_ids, engram_on, cancel, max_new, skip_special=False)
                tagged = split_reasoning(raw, S.tok.all_special_tokens + list(S.tok.get_added_vocab()))
                if S.raw_thinking:
                    tagged = keep_markers(tagged)
            else:
                tagged = (("content", p) for p in raw_pieces(body, input_ids, engram_on, cancel, max_new))
            gen = with_stops(tagged, parse_stops(body), cancel)
            try:
                if stream:
                    self.send_response(200)
                    self.send_header("Content-Type", "text/event-stream")
                    self.send_header("Cache-Control", "no-cache")
                    self._cors()
                    self.end_headers()
                    if chat:
                        self.wfile.write(f"data: {json.dumps(event('', first=True))}\n\n".encode())
                for kind, piece in gen:
                    if not piece:
                        continue
                    if kind == "reasoning":
                        thought += piece
                    else:
                        answer += piece
                    if stream:
                        self.wfile.write(f"data: {json.dumps(event(piece, kind=kind))}\n\n".encode())
                        self.wfile.flush()
            except (BrokenPipeError, ConnectionResetError):
                cancel.cancelled = True
                print("[server] client disconnected, generation cancelled")
            except Exception as e:  # noqa: BLE001
                cancel.cancelled = True
                print(f"[server] generation error: {e!r}")
                if not stream:
                    return self._json({"error": str(e)}, 500)
            finally:
                gen.close()
        both = thought + answer
        n_new = len(S.tok(both, add_special_tokens=False).input_ids) if both else 0
        finish = "length" if n_new >= max_new else "stop"
        n_prompt = int(input_ids.shape[1])
        if cancel.t_first is not None:
            prefill = cancel.t_first - t0
            dec = cancel.t_last - cancel.t_first
            speed = f"{(cancel.steps - 1) / dec:.1f} tok/s" if cancel.steps > 1 and dec > 0 else "n/a"
            timing = (f"prompt {prefill:.1f}s ({n_prompt / max(prefill, 1e-6):.0f} tok/s) | generation {speed} | "
                      f"{cancel.steps} new tok")
        else:
            timing = f"~{n_new} new tok"
        print(f"[server] {'ENGRAM' if engram_on else 'no-engram'} | prompt {n_prompt} tok | {timing} | {finish}")
        if stream:
            try:
                self.wfile.write(f"data: {json.dumps(event('', finish=finish))}\n\n".encode())
                self.wfile.write(b"data: [DONE]\n\n")
                self.wfile.flush()
            except (BrokenPipeError, ConnectionResetError):
                pass
            return
        usage = {"prompt_tokens": n_prompt, "completion_tokens": n_new, "total_tokens": n_prompt + n_new}
        if chat:
            msg = {"role": "assistant", "content": answer, "reasoning_content": thought or None}
            self._json({"id": rid, "object": "chat.completion", "created": created, "model": name,
                        "choices": [{"index": 0, "message": msg, "finish_reason": finish}], "usage": usage})
        else:
            self._json({"id": rid, "object": "text_completion", "created": created, "model": name,
                        "choices": [{"index": 0, "text": answer, "finish_reason": finish}], "usage": usage})


def main(argv=None):
    from .infer import add_engram_args, load_model

    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    add_engram_args(ap)
    ap.add_argument("--name", default=None)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--raw-thinking", action="store_true")
    ap.add_argument("--no-thinking", action="store_true")
    args = ap.parse_args(argv)
    S.template_kwargs = {"enable_thinking": not args.no_thinking, "preserve_thinking": True}
    S.raw_thinking = args.raw_thinking
    S.name = args.name or os.path.basename(os.path.normpath(args.model))
    S.model, S.tok, S.runner = load_model(args)
    print(f"\n[server] ready: http://{args.host}:{args.port}/v1")
    print(f"[server] models: '{S.name}' (engram on) | '{S.name}-noengram' (engram off)")
    ThreadingHTTPServer((args.host, args.port), Handler).serve_forever()


if __name__ == "__main__":
    main()
