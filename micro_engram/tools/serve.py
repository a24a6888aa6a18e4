"""OpenAI-compatible HTTP server for an HF model with trained engram(s) (the reference's
serve_engram.py offers the same endpoints and model names).

    python -m micro_engram.tools.serve --model MERGED_DIR [--port 8000] [--host 127.0.0.1]
    python -m micro_engram.tools.serve --model BASE_DIR --engram-pt micro_engram.pt

Two model names are offered: <name> (engram on) and <name>-noengram (same weights, engram off).
Endpoints: GET /v1/models, /health; POST /v1/chat/completions and /v1/completions (server-sent
events with "stream": true). One request runs at a time, because the engram keeps the
generation's token history. Chat replies put the thinking channel (<|channel>thought ...
<channel|>) in reasoning_content; --raw-thinking leaves the markers in content. Thinking is on
by default (enable_thinking + preserve_thinking, as in training); --no-thinking flips the
default and a request may override it through chat_template_kwargs. Stop strings cut the
answer, never the reasoning. A client that disconnects cancels its generation; every request
logs its prefill and decode speed.
"""
import argparse
import json
import os
import threading
import time
import uuid
from dataclasses import dataclass, field
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

import torch

THINK_START, THINK_END = "<|channel>thought", "<channel|>"


# ============================================================================ stream transforms
class ReasoningSplitter:
    """Feeds raw decoded text (special tokens kept) and emits ("reasoning" | "content", text):
    text between THINK_START and THINK_END is reasoning, other special tokens are removed, the
    newline the template writes after either marker is dropped, and text that might be the
    beginning of a marker is held back until it is decided."""

    def __init__(self, specials):
        self.remove = [s for s in specials if s and s not in (THINK_START, THINK_END, "<|channel>")]
        self.keep_back = max([len(THINK_START), len(THINK_END)] + [len(s) for s in self.remove]) - 1
        self.mode, self.pending, self.skip_newline = "content", "", False

    def _strip(self, text):
        for s in self.remove:
            text = text.replace(s, "")
        return text

    def feed(self, piece):
        self.pending += piece
        out = []
        while True:
            if self.skip_newline and self.pending:
                if self.pending[0] == "\n":
                    self.pending = self.pending[1:]
                self.skip_newline = False
            marker = THINK_START if self.mode == "content" else THINK_END
            at = self.pending.find(marker)
            if at < 0:
                self.pending = self._strip(self.pending)
                if len(self.pending) > self.keep_back:
                    cut = len(self.pending) - self.keep_back
                    out.append((self.mode, self.pending[:cut]))
                    self.pending = self.pending[cut:]
                return out
            before = self._strip(self.pending[:at])
            if before:
                out.append((self.mode, before))
            self.pending = self.pending[at + len(marker):]
            self.mode = "reasoning" if self.mode == "content" else "content"
            self.skip_newline = True

    def finish(self):
        rest = self._strip(self.pending)
        self.pending = ""
        return [(self.mode, rest)] if rest else []


def split_reasoning(pieces, specials):
    splitter = ReasoningSplitter(specials)
    try:
        for piece in pieces:
            yield from splitter.feed(piece)
        yield from splitter.finish()
    finally:
        if hasattr(pieces, "close"):
            pieces.close()


def keep_markers(tagged):
    """--raw-thinking: the reasoning goes back into content between its markers."""
    thinking = False
    for kind, text in tagged:
        if (kind == "reasoning") != thinking:
            yield "content", (THINK_START + "\n") if not thinking else THINK_END
            thinking = not thinking
        yield "content", text
    if thinking:
        yield "content", THINK_END


def with_stops(tagged, stops, cancel):
    """Cut the answer at the first stop string (reasoning passes untouched); answer text that
    could begin a stop string is held back until it is decided."""
    if not stops:
        yield from tagged
        return
    keep_back = max(len(s) for s in stops) - 1
    answer = ""
    try:
        for kind, piece in tagged:
            if kind != "content":
                yield kind, piece
                continue
            answer += piece
            hits = [answer.find(s) for s in stops if s in answer]
            if hits:
                yield "content", answer[:min(hits)]
                cancel.cancelled = True
                return
            if len(answer) > keep_back:
                yield "content", answer[:len(answer) - keep_back]
                answer = answer[len(answer) - keep_back:]
        yield "content", answer
    finally:
        if hasattr(tagged, "close"):
            tagged.close()


def parse_stops(body):
    """The request's stop strings as a list: OpenAI accepts one string or a list (empty entries
    mean nothing)."""
    stop = body.get("stop") or []
    return list(filter(None, [stop] if isinstance(stop, str) else stop))


def flat_content(content):
    """A message's text: a string, or the text parts of OpenAI content parts."""
    if content is None:
        return ""
    if isinstance(content, list):
        return "".join(p.get("text", "") for p in content if isinstance(p, dict) and p.get("type") == "text")
    return content if isinstance(content, str) else str(content)


# ============================================================================ generation
class Cancel:
    """A stopping criterion that the request side can raise; it also times the tokens."""

    def __init__(self):
        self.cancelled = False
        self.steps = 0
        self.t_first = self.t_last = None

    def __call__(self, input_ids, scores, **kw):
        self.t_last = time.time()
        if self.t_first is None:
            self.t_first = self.t_last
        self.steps += 1
        return torch.full((input_ids.shape[0],), self.cancelled, dtype=torch.bool, device=input_ids.device)


def sampling_kwargs(body):
    """model.generate keyword arguments for an OpenAI-style request body."""
    temperature = 0.8 if body.get("temperature") is None else float(body["temperature"])
    kw = {"do_sample": temperature > 0}
    if temperature > 0:
        kw["temperature"] = temperature
        kw["top_p"] = 1.0 if body.get("top_p") is None else float(body["top_p"])
        for key, cast in (("top_k", int), ("min_p", float)):
            if body.get(key):
                kw[key] = cast(body[key])
    if body.get("repetition_penalty"):
        kw["repetition_penalty"] = float(body["repetition_penalty"])
    return kw


@dataclass
class Server:
    model: object = None
    tok: object = None
    runner: object = None
    name: str = "model"
    template_kwargs: dict = field(default_factory=dict)
    raw_thinking: bool = False
    lock: threading.Lock = field(default_factory=threading.Lock)

    def encode_chat(self, messages, template_kwargs):
        msgs = []
        for m in messages:
            msg = {"role": m.get("role", "user"), "content": flat_content(m.get("content"))}
            thought = m.get("reasoning_content") or m.get("reasoning")
            if thought:
                msg["reasoning_content"] = thought
            msgs.append(msg)
        text = self.tok.apply_chat_template(msgs, add_generation_prompt=True, tokenize=False, **template_kwargs)
        return self.tok(text, add_special_tokens=False, return_tensors="pt").input_ids  # the template has <bos>

    def encode_text(self, prompt):
        bos = self.tok.bos_token or ""
        return self.tok(prompt, add_special_tokens=not (bos and prompt.startswith(bos)), return_tensors="pt").input_ids

    def generate(self, body, input_ids, engram_on, cancel, max_new, skip_special=True):
        """Decoded text pieces of model.generate running in a worker thread (the caller holds
        the lock)."""
        from transformers import StoppingCriteriaList, TextIteratorStreamer

        self.runner.enabled = engram_on
        self.runner.new_sequence()
        if body.get("seed") is not None:
            torch.manual_seed(int(body["seed"]))
        streamer = TextIteratorStreamer(self.tok, skip_prompt=True, skip_special_tokens=skip_special)
        kw = dict(sampling_kwargs(body), input_ids=input_ids, attention_mask=torch.ones_like(input_ids),
                  max_new_tokens=max_new, use_cache=True, stopping_criteria=StoppingCriteriaList([cancel]),
                  streamer=streamer)
        error = []

        def work():
            try:
                with torch.no_grad():
                    self.model.generate(**kw)
            except Exception as e:  # noqa: BLE001 - reraised on the request's thread
                error.append(e)
                streamer.on_finalized_text("", stream_end=True)

        worker = threading.Thread(target=work, daemon=True)
        worker.start()
        try:
            yield from streamer
        finally:
            cancel.cancelled = True
            worker.join()
        if error:
            raise error[0]

    def stream(self, body, input_ids, engram_on, cancel, max_new, chat):
        """(kind, text) of one request: reasoning split off for chat, stops applied."""
        if chat:
            raw = self.generate(body, input_ids, engram_on, cancel, max_new, skip_special=False)
            tagged = split_reasoning(raw, self.tok.all_special_tokens + list(self.tok.get_added_vocab()))
            if self.raw_thinking:
                tagged = keep_markers(tagged)
        else:
            tagged = (("content", p) for p in self.generate(body, input_ids, engram_on, cancel, max_new))
        return with_stops(tagged, parse_stops(body), cancel)


SERVER = Server()


# ============================================================================ HTTP
@dataclass
class Reply:
    """One response under construction: ids, the chunk format, the accumulated text."""
    chat: bool
    model: str
    rid: str = ""
    created: int = 0
    answer: str = ""
    thought: str = ""

    def __post_init__(self):
        self.rid = ("chatcmpl-" if self.chat else "cmpl-") + uuid.uuid4().hex[:24]
        self.created = int(time.time())

    def chunk(self, text, finish=None, first=False, kind="content"):
        if not self.chat:
            return {"id": self.rid, "object": "text_completion", "created": self.created, "model": self.model,
                    "choices": [{"index": 0, "text": text, "finish_reason": finish}]}
        delta = {"role": "assistant"} if first else {}
        if text:
            delta["reasoning_content" if kind == "reasoning" else "content"] = text
        return {"id": self.rid, "object": "chat.completion.chunk", "created": self.created, "model": self.model,
                "choices": [{"index": 0, "delta": delta, "finish_reason": finish}]}

    def final(self, finish, usage):
        if self.chat:
            msg = {"role": "assistant", "content": self.answer, "reasoning_content": self.thought or None}
            return {"id": self.rid, "object": "chat.completion", "created": self.created, "model": self.model,
                    "choices": [{"index": 0, "message": msg, "finish_reason": finish}], "usage": usage}
        return {"id": self.rid, "object": "text_completion", "created": self.created, "model": self.model,
                "choices": [{"index": 0, "text": self.answer, "finish_reason": finish}], "usage": usage}


def _timing_line(cancel, t0, n_prompt, n_new):
    if cancel.t_first is None:
        return f"~{n_new} new tok"
    prefill = cancel.t_first - t0
    decode = cancel.t_last - cancel.t_first
    speed = f"{(cancel.steps - 1) / decode:.1f} tok/s" if cancel.steps > 1 and decode > 0 else "n/a"
    return (f"prompt {prefill:.1f}s ({n_prompt / max(prefill, 1e-6):.0f} tok/s) | generation {speed} | "
            f"{cancel.steps} new tok")


class Handler(BaseHTTPRequestHandler):
    server_version = "engram-server"

    def log_message(self, fmt, *a):
        pass

    _CORS = (("Access-Control-Allow-Origin", "*"), ("Access-Control-Allow-Headers", "*"),
             ("Access-Control-Allow-Methods", "GET, POST, OPTIONS"))

    def _head(self, code, headers=()):
        """Status line, the given headers and the CORS headers, then the blank line."""
        self.send_response(code)
        for key, value in (*headers, *self._CORS):
            self.send_header(key, value)
        self.end_headers()

    def _json(self, obj, code=200):
        body = json.dumps(obj).encode()
        self._head(code, (("Content-Type", "application/json"), ("Content-Length", str(len(body)))))
        self.wfile.write(body)

    def _event(self, obj):
        self.wfile.write(f"data: {json.dumps(obj)}\n\n".encode())
        self.wfile.flush()

    def do_OPTIONS(self):
        self._head(204)

    def do_GET(self):
        path = self.path.rstrip("/")
        if path in ("/v1/models", "/models"):
            now = int(time.time())
            self._json({"object": "list", "data": [{"id": n, "object": "model", "created": now, "owned_by": "local"}
                                                   for n in (SERVER.name, SERVER.name + "-noengram")]})
        elif path in ("/health", ""):
            self._json({"status": "ok"})
        else:
            self._json({"error": "not found"}, 404)

    def _read_request(self, chat):
        body = json.loads(self.rfile.read(int(self.headers.get("Content-Length", 0))) or b"{}")
        if chat:
            kwargs = dict(SERVER.template_kwargs, **(body.get("chat_template_kwargs") or {}))
            return body, SERVER.encode_chat(body.get("messages", []), kwargs)
        prompt = body.get("prompt", "")
        return body, SERVER.encode_text(prompt if isinstance(prompt, str) else "".join(prompt))

    def do_POST(self):
        path = self.path.rstrip("/")
        if path not in ("/v1/chat/completions", "/v1/completions"):
            return self._json({"error": "not found"}, 404)
        chat = path.endswith("chat/completions")
        try:
            body, input_ids = self._read_request(chat)
        except Exception as e:  # noqa: BLE001
            return self._json({"error": f"bad request: {e}"}, 400)
        reply = Reply(chat, body.get("model") or SERVER.name)
        engram_on = not reply.model.endswith("-noengram")
        max_new = int(body.get("max_tokens") or body.get("max_completion_tokens") or 512)
        streaming = bool(body.get("stream"))
        input_ids = input_ids.to(next(SERVER.model.parameters()).device)
        t0 = time.time()
        with SERVER.lock:
            cancel = Cancel()
            pieces = SERVER.stream(body, input_ids, engram_on, cancel, max_new, chat)
            try:
                if streaming:
                    self._head(200, (("Content-Type", "text/event-stream"), ("Cache-Control", "no-cache")))
                    if chat:
                        self._event(reply.chunk("", first=True))
                for kind, text in pieces:
                    if not text:
                        continue
                    if kind == "reasoning":
                        reply.thought += text
                    else:
                        reply.answer += text
                    if streaming:
                        self._event(reply.chunk(text, kind=kind))
            except (BrokenPipeError, ConnectionResetError):
                cancel.cancelled = True
                print("[server] client disconnected, generation cancelled")
            except Exception as e:  # noqa: BLE001
                cancel.cancelled = True
                print(f"[server] generation error: {e!r}")
                if not streaming:
                    return self._json({"error": str(e)}, 500)
            finally:
                pieces.close()
        generated = reply.thought + reply.answer
        n_new = len(SERVER.tok(generated, add_special_tokens=False).input_ids) if generated else 0
        n_prompt = int(input_ids.shape[1])
        finish = "length" if n_new >= max_new else "stop"
        print(f"[server] {'ENGRAM' if engram_on else 'no-engram'} | prompt {n_prompt} tok | "
              f"{_timing_line(cancel, t0, n_prompt, n_new)} | {finish}")
        if streaming:
            try:
                self._event(reply.chunk("", finish=finish))
                self.wfile.write(b"data: [DONE]\n\n")
                self.wfile.flush()
            except (BrokenPipeError, ConnectionResetError):
                pass
            return
        self._json(reply.final(finish, {"prompt_tokens": n_prompt, "completion_tokens": n_new,
                                        "total_tokens": n_prompt + n_new}))


def main(argv=None):
    from .infer import add_engram_args, load_model

    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    add_engram_args(ap)
    ap.add_argument("--name", default=None, help="model name (default: the model folder's name)")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--raw-thinking", action="store_true", help="keep the thinking markers in content")
    ap.add_argument("--no-thinking", action="store_true", help="thinking off unless a request asks for it")
    args = ap.parse_args(argv)
    SERVER.template_kwargs = {"enable_thinking": not args.no_thinking, "preserve_thinking": True}
    SERVER.raw_thinking = args.raw_thinking
    SERVER.name = args.name or os.path.basename(os.path.normpath(args.model))
    SERVER.model, SERVER.tok, SERVER.runner = load_model(args)
    print(f"\n[server] ready: http://{args.host}:{args.port}/v1")
    print(f"[server] models: '{SERVER.name}' (engram on) | '{SERVER.name}-noengram' (engram off)")
    ThreadingHTTPServer((args.host, args.port), Handler).serve_forever()


if __name__ == "__main__":
    main()
