"""The command-line tools (micro_engram.tools): token merging, assembly/extraction, checkpoint
stats, order zeroing, data statistics, chat rendering, held-out scoring and the token diff
against a fake OpenAI-style server, and the HF server's text-stream transforms. Reference
counterparts: test_canon.py, test_zero_order.py, test_render_chat.py, test_eval_spans.py,
test_token_diff.py."""
import json
import math
import os
import re
import threading
from http.server import BaseHTTPRequestHandler, HTTPServer

import numpy as np
import pytest
import torch

from micro_engram.module import MicroEngram


# ------------------------------------------------------------------ build_canon
def test_canon_merge_rules():
    from micro_engram.tools.build_canon import WHITESPACE_CLASS, build, merge_key, name_token_ids

    assert merge_key("▁The") == merge_key("▁the") == "▁the"
    assert merge_key("the") != merge_key("▁the")
    assert merge_key("the", merge_space=True) == merge_key("▁the", merge_space=True)
    assert merge_key("é", accents=True) == "e" and merge_key("é") == "é"
    assert merge_key("Ċ", whitespace=True) == merge_key("▁▁", whitespace=True) == WHITESPACE_CLASS
    assert merge_key("▁") is None
    pieces = ["<pad>", "▁the", "▁The", "the", "THE", "<0x41>", "▁é", "▁e", "Ċ", "▁▁", "▁Peril", "▁peril"]
    protected = {0}
    canon, _ = build(pieces, protected, 16)
    assert canon[2] == 1 and canon[4] == 3 and canon[3] == 3  # case merges, space marker kept apart
    assert canon[5] == 5  # byte token never merges
    assert canon[12:] == [12, 13, 14, 15]  # beyond the tokenizer: identity
    canon_p, _ = build(pieces, protected, 16, True, True, True)
    assert canon_p[3] == 1 and canon_p[6] == 6 and canon_p[7] == 6 and canon_p[9] == 8
    ids, single, split = name_token_ids(["Peril", "Nobody"], pieces)
    canon_n, _ = build(pieces, protected | ids, 16)
    assert single == ["Peril"] and split == ["Nobody"] and canon_n[10] == 10 and canon_n[11] == 11
    t = torch.tensor(canon_p)
    assert torch.equal(t[t], t)  # idempotent; smallest id stands for its class


def test_canon_hashing_in_module():
    V = 1000
    canon = torch.arange(V)
    canon[11], canon[501] = 10, 500
    eng = MicroEngram(model_dim=16, table_size=257, engram_dim=4, num_heads=2, vocab_size=V, canon=canon)
    a = torch.tensor([[3, 10, 7, 500, 9, 10, 4]])
    b = torch.tensor([[3, 11, 7, 501, 9, 11, 4]])
    c = torch.tensor([[3, 12, 7, 500, 9, 10, 4]])
    same = lambda x, y: all(torch.equal(p, q) for p, q in zip(eng.hash_ids(x), eng.hash_ids(y)))  # noqa: E731
    assert same(a, b) and not same(a, c)
    fresh = MicroEngram(model_dim=16, table_size=257, engram_dim=4, num_heads=2, vocab_size=V)
    old = {k: v for k, v in fresh.state_dict().items() if k != "canon"}
    res = MicroEngram(model_dim=16, table_size=257, engram_dim=4, num_heads=2, vocab_size=V).load_state_dict(
        old, strict=False)
    assert list(res.missing_keys) == ["canon"] and not res.unexpected_keys
    e2 = MicroEngram(model_dim=16, table_size=257, engram_dim=4, num_heads=2, vocab_size=V)
    e2.load_state_dict(eng.state_dict())
    assert torch.equal(e2.canon, canon)


# ------------------------------------------------------------------ zero_order
def _engram_folder(tmp, layers=(2,), orders=(2, 3, 4)):
    conf = {"table_size": 31, "engram_dim": 4, "num_heads": 2, "orders": list(orders), "gate": "scalar",
            "engrams": [{"layer": L, "seed": 10007 * L, "weights": "w.pt"} for L in layers]}
    sd = {}
    for L in layers:
        torch.manual_seed(L)
        e = MicroEngram(model_dim=8, table_size=31, engram_dim=4, num_heads=2, vocab_size=50, orders=orders,
                        seed=10007 * L)
        with torch.no_grad():
            e.value.weight.normal_()
        sd.update({f"model.layers.{L}.micro_engram.{k}": v for k, v in e.state_dict().items()})
    torch.save(sd, os.path.join(tmp, "w.pt"))
    with open(os.path.join(tmp, "micro_engram_config.json"), "w") as f:
        json.dump(conf, f)
    return sd


def test_zero_order(tmp_path):
    from micro_engram.tools import zero_order

    src, out = tmp_path / "src", tmp_path / "out"
    src.mkdir()
    sd = _engram_folder(str(src), layers=(2, 5))
    zero_order.main([str(src), "--order", "4", "--layer-scale", "5=0.5", "--out", str(out)])
    got = torch.load(out / "consolidated.pth")
    conf = json.load(open(out / "micro_engram_config.json"))
    for L, scale in ((2, 1.0), (5, 0.5)):
        pre = f"model.language_model.layers.{L}.micro_engram."
        for k in range(6):  # tables ordered order-major: 2,2,3,3,4,4
            t = got[pre + f"tables.{k}.weight"]
            want = sd[f"model.layers.{L}.micro_engram.tables.{k}.weight"]
            assert torch.equal(t, torch.zeros_like(t)) if k >= 4 else torch.equal(t, want)
        torch.testing.assert_close(got[pre + "value.weight"], sd[f"model.layers.{L}.micro_engram.value.weight"] * scale)
    assert conf["zeroed_orders"] == [4] and conf["injection_scale"] == {"2": 1.0, "5": 0.5}
    assert all(e["weights"] == "consolidated.pth" for e in conf["engrams"])
    with pytest.raises(SystemExit):
        zero_order.main([str(src), "--out", str(tmp_path / "x")])  # nothing to do
    with pytest.raises(SystemExit):
        zero_order.main([str(src), "--order", "4", "--out", str(out)])  # exists, no --force


# ------------------------------------------------------------------ assemble / extract / stats
def test_assemble_extract_and_stats(tmp_path):
    from safetensors.torch import save_file

    from micro_engram.tools import assemble, engram_stats, extract

    base = tmp_path / "base"
    base.mkdir()
    save_file({"model.language_model.layers.0.mlp.weight": torch.ones(2, 2),
               "model.language_model.layers.1.mlp.weight": torch.ones(2, 2),
               "model.vision_tower.layers.0.w": torch.ones(1)}, str(base / "model.safetensors"))
    (base / "config.json").write_text("{}")
    eng = tmp_path / "ckpt"
    eng.mkdir()
    e = MicroEngram(model_dim=8, table_size=31, engram_dim=4, num_heads=2, vocab_size=50)
    with torch.no_grad():
        e.value.weight.normal_()
    torch.save(e.state_dict(), eng / "micro_engram.pt")
    (eng / "micro_engram_config.json").write_text(json.dumps({"layer": 1, "table_size": 31, "engram_dim": 4,
                                                              "num_heads": 2, "weights": "micro_engram.pt"}))
    out = tmp_path / "out"
    assemble.main(["--base", str(base), "--engram", str(eng / "micro_engram.pt"), "--out", str(out)])
    assert os.path.islink(out / "config.json") and os.path.islink(out / "model.safetensors")
    idx = json.load(open(out / "model.safetensors.index.json"))
    key = "model.language_model.layers.1.micro_engram.tables.0.weight"
    assert idx["weight_map"][key] == "micro_engram.safetensors"
    assert "weights" not in json.load(open(out / "micro_engram_config.json"))
    back = extract.extract(str(out))
    assert set(back) == set(e.state_dict()) and torch.equal(back["tables.0.weight"], e.tables[0].weight)
    # stats over an output_dir with one complete and one incomplete checkpoint
    run = tmp_path / "run"
    for step, complete in ((100, True), (200, False)):
        c = run / f"checkpoint-{step}"
        c.mkdir(parents=True)
        torch.save(e.state_dict(), c / "micro_engram.pt")
        (c / "micro_engram_config.json").write_text(json.dumps({"layer": 1, "table_size": 31, "engram_dim": 4,
                                                                "num_heads": 2}))
        if complete:
            (c / "trainer_state.json").write_text("{}")
    snaps = engram_stats.find_snapshots(str(run))
    assert [s[0] for s in snaps] == [100]
    line = engram_stats.stats_line(*snaps[0])
    assert line.startswith("step    100") and "rms" in line


# ------------------------------------------------------------------ data stats
def test_data_stats_keys_and_counts():
    from micro_engram.tools.data_stats import collect, ngram_keys

    ids = np.array([5, 6, 7, 5, 6, 7, 5, 6])
    k2 = ngram_keys(ids, 2)
    assert len(k2) == 7 and k2[0] == k2[3] and k2[0] != k2[1]
    assert k2[0] == 6 + 5 * (1 << 18)  # exact: last token + previous * V
    k4 = ngram_keys(ids, 4)
    assert k4[0] == k4[3] and len(set(k4.tolist())) == 3
    labels = np.array([-100, -100, 1, 1, 1, 1, 1, 1])
    keys, sup, total, trained, used = collect([(ids, labels)], 10 ** 9, orders=(2, 3))
    assert total == 8 and trained == 6 and used == 1 and sup[2][0].sum() == 6


# ------------------------------------------------------------------ render_chat
def test_render_rows_spans():
    from micro_engram.tools.render_chat import messages_of, render_rows

    def render(msgs, add_generation_prompt=False):
        s = "<bos>" + "".join(f"<{m['role']}>{m['content']}<end>\n" for m in msgs)
        return s + ("<assistant>" if add_generation_prompt else "")

    conv = messages_of({"conversations": [{"from": "human", "value": "hi"}, {"from": "gpt", "value": "yo there"}]})
    assert conv == [{"role": "user", "content": "hi"}, {"role": "assistant", "content": "yo there"}]
    (row, ok), = list(render_rows([conv], render, {"assistant"}, ("<end>",)))
    a, b = row["spans"][0]
    assert ok and row["text"][a:b] == "yo there<end>"
    (row2, _), = list(render_rows([conv], render, {"assistant"}, (), no_spans=True))
    assert "spans" not in row2
    assert messages_of({"messages": [{"role": "user"}]}) is None


# ------------------------------------------------------------------ fake OpenAI-style server
_VOCAB = {}


def _tok(text):
    return [_VOCAB.setdefault(t, len(_VOCAB) + 10) for t in re.findall(r"<bos>|<end>|<user>|<assistant>|\s|[^\s<]+",
                                                                        text)]


def _word(i):
    return next(k for k, v in _VOCAB.items() if v == i)


def _prompt_logprobs(ids, boost):
    """vLLM-style prompt_logprobs: assistant-ish words ("aa...", "<end>") get probability `boost`,
    every other word 0.1; the first position has none."""
    def entry(i):
        word = _word(i)
        p = boost if word.startswith("aa") or word == "<end>" else 0.1
        return {str(i): {"logprob": math.log(p), "rank": 1, "decoded_token": word}}

    return [None] + [entry(i) for i in ids[1:]]


class _Fake(BaseHTTPRequestHandler):
    """A stand-in vLLM server: /tokenize and /v1/completions with prompt log-probs."""

    boost = 0.9

    def log_message(self, *a):
        pass

    def _reply(self, payload):
        body = json.dumps(payload).encode()
        self.send_response(200)
        for key, value in (("Content-Type", "application/json"), ("Content-Length", str(len(body)))):
            self.send_header(key, value)
        self.end_headers()
        self.wfile.write(body)

    def do_GET(self):
        self._reply({"data": [{"id": "fake"}]})

    def do_POST(self):
        size = int(self.headers["Content-Length"])
        req = json.loads(self.rfile.read(size))
        if self.path == "/tokenize":
            text = req.get("prompt")
            if text is None:  # chat: a simple role-tagged rendering
                text = "".join(f"<{m['role']}>{m['content']}<end>" for m in req["messages"]) + "<assistant>"
            self._reply({"tokens": _tok(text)})
            return
        ids = req["prompt"] if isinstance(req["prompt"], list) else _tok(req["prompt"])
        choice = {"text": "", "prompt_token_ids": ids, "prompt_logprobs": _prompt_logprobs(ids, type(self).boost)}
        self._reply({"choices": [choice]})


@pytest.fixture
def fake_server():
    srv = HTTPServer(("127.0.0.1", 0), _Fake)
    th = threading.Thread(target=srv.serve_forever, daemon=True)
    th.start()
    yield f"http://127.0.0.1:{srv.server_address[1]}"
    srv.shutdown()


def test_eval_logprob_spans_and_compare(tmp_path, fake_server):
    from micro_engram.tools import eval_logprob

    rows = []
    for k in range(4):
        text, spans = "<bos>", []
        for t in range(3):
            text += f"<user>uu{k} said something here\n<assistant>"
            a = len(text)
            text += f"aa{k} aa{t} aaa<end>"
            spans.append([a, len(text)])
            text += "\n"
        rows.append({"text": text, "spans": spans})
    with_spans, no_spans = tmp_path / "s.jsonl", tmp_path / "n.jsonl"
    with_spans.write_text("".join(json.dumps(r) + "\n" for r in rows))
    no_spans.write_text("".join(json.dumps({"text": r["text"]}) + "\n" for r in rows))
    common = ["--url", fake_server, "--parallel", "1", "--min-chars", "1"]
    eval_logprob.main(["run", "--data", str(with_spans), "--out", str(tmp_path / "a.json")] + common)
    a = json.load(open(tmp_path / "a.json"))
    n = sum(c["n_tokens"] for c in a["chunks"])
    loss = -sum(c["sum_logprob"] for c in a["chunks"]) / n
    per_turn = [0.9, 0.1, 0.9, 0.1, 0.9, 0.9]  # aaK, " ", aaT, " ", aaa, <end>
    assert n == 4 * 3 * 6 and abs(loss - (-sum(map(math.log, per_turn)) / 6)) < 1e-9
    eval_logprob.main(["run", "--data", str(no_spans), "--out", str(tmp_path / "b.json")] + common)
    b = json.load(open(tmp_path / "b.json"))
    assert sum(c["n_tokens"] for c in b["chunks"]) > n
    s = eval_logprob.compare_runs(a, a)
    assert s["pairs"] == 4 and s["loss_a"] == s["loss_b"] and s["wins_a"] == 0 and s["ci"] == (0.0, 0.0)
    assert eval_logprob.chunk("a\n\nb\n\nc", 4) == ["a\n\nb", "c"] and eval_logprob.chunk("a\n\nb", 3) == ["a", "b"]


def test_token_diff_run_and_render(tmp_path, fake_server):
    from micro_engram.tools import token_diff

    (tmp_path / "chat.json").write_text(json.dumps([{"role": "user", "content": "hello"}]))
    (tmp_path / "reply.txt").write_text("aa1 bb aa2")
    base = ["run", "--url", fake_server, "--messages", str(tmp_path / "chat.json"), "--reply",
            str(tmp_path / "reply.txt")]
    _Fake.boost = 0.9
    token_diff.main(base + ["--out", str(tmp_path / "on.json")])
    _Fake.boost = 0.5
    token_diff.main(base + ["--out", str(tmp_path / "off.json")])
    _Fake.boost = 0.9
    on, off = json.load(open(tmp_path / "on.json")), json.load(open(tmp_path / "off.json"))
    rows = token_diff.diff_rows(on, off)
    assert [round(r["d"], 6) for r in rows] == [round(math.log(0.9 / 0.5), 6), 0.0, 0.0, 0.0,
                                                round(math.log(0.9 / 0.5), 6)]
    token_diff.main(["render", str(tmp_path / "on.json"), str(tmp_path / "off.json"), "--out",
                     str(tmp_path / "d.html")])
    html_text = (tmp_path / "d.html").read_text()
    assert html_text.count("<span style=") == 5 + 2 and "rgba(22, 163, 74" in html_text
    assert token_diff.colour(0.0, 2.0) == "transparent"


# ------------------------------------------------------------------ HF server stream transforms
def test_server_stream_transforms():
    from micro_engram.tools.serve import THINK_END, THINK_START, keep_markers, parse_stops, split_reasoning, with_stops

    text = f"<bos>{THINK_START}\nlet me think<channel|>\nThe answer is 42.<turn|>"
    for cut in (1, 3, 7):  # any split of the stream gives the same result
        pieces = [text[i:i + cut] for i in range(0, len(text), cut)]
        out = list(split_reasoning(iter(pieces), ["<bos>", "<turn|>", THINK_START, THINK_END]))
        reasoning = "".join(t for k, t in out if k == "reasoning")
        content = "".join(t for k, t in out if k == "content")
        assert reasoning == "let me think" and content == "The answer is 42.", (cut, out)
    tagged = [("reasoning", "hm"), ("content", "ok")]
    assert "".join(t for _, t in keep_markers(tagged)) == f"{THINK_START}\nhm{THINK_END}ok"

    class C:
        cancelled = False

    c = C()
    out = list(with_stops(iter([("reasoning", "STOP inside"), ("content", "abc ST"), ("content", "OP tail")]),
                          ["STOP"], c))
    assert "".join(t for k, t in out if k == "content") == "abc " and c.cancelled
    assert ("reasoning", "STOP inside") in out
    assert parse_stops({"stop": "x"}) == ["x"] and parse_stops({"stop": ["a", ""]}) == ["a"]


def test_infer_settings_layering(tmp_path, capsys):
    """Each setting comes from the first source that gives it: flag, engram config, the saved
    tensors, the defaults; an explicit --table-size drops per-order sizes."""
    import json
    import types

    import torch

    from micro_engram.tools import infer

    sd = {f"tables.{k}.weight": torch.zeros(rows, 16) for k, rows in enumerate([100, 100, 300, 300])}
    sd["q_scale"] = torch.zeros(8)
    sd["value.weight"] = torch.zeros(8, 32)

    def args(**kw):
        base = {"model": str(tmp_path), "engram_config": None, "layer": None, "table_size": None, "dim": None,
                "heads": None, "gate": None}
        return types.SimpleNamespace(**{**base, **kw})

    s = infer.resolve_settings(args(), sd, 5)  # no config: the tensors, then the defaults
    assert (s["layer"], s["table_size"], s["engram_dim"], s["num_heads"], s["gate"]) == (5, 100, 16, 2, "scalar_sqrt")
    assert s["table_sizes"] == {2: 100, 3: 300} and s["seed"] == 0 and s["orders"] == (2, 3)
    conf = {"layer": 7, "engram_dim": 16, "gate": "scalar", "seed": 70049, "orders": [2, 3], "table_sizes": {"2": 9}}
    path = tmp_path / "micro_engram_config.json"
    path.write_text(json.dumps(conf))
    s = infer.resolve_settings(args(heads=4), sd, 5)  # config over tensors, flags over both
    assert (s["layer"], s["gate"], s["seed"], s["num_heads"], s["table_sizes"]) == (7, "scalar", 70049, 4, {"2": 9})
    s = infer.resolve_settings(args(table_size=64, layer=1), sd, 5)
    assert (s["table_size"], s["table_sizes"], s["layer"]) == (64, None, 1)
    assert infer.shape_settings({}, (2, 3)) == {"table_size": None, "table_sizes": None, "engram_dim": None,
                                                "num_heads": None, "gate": None}
    assert "settings:" in capsys.readouterr().out


def test_base_fingerprint_and_mismatch(tmp_path):
    """The base fingerprint names a folder's text weights (embedding and the first, middle and
    last layers' projections): the same weights give the same fingerprint, changed weights or
    an engram config recorded on another base give a warning, no record gives none."""
    import torch
    from safetensors.torch import save_file

    from micro_engram.weights import base_fingerprint, base_mismatch

    def folder(name, scale, engram_scale=1.0):
        d = tmp_path / name
        d.mkdir()
        g = torch.Generator().manual_seed(1)
        ts = {"model.embed_tokens.weight": torch.randn(32, 8, generator=g) * scale}
        for i in range(3):
            for proj in ("self_attn.q_proj", "mlp.down_proj"):
                ts[f"model.layers.{i}.{proj}.weight"] = torch.randn(8, 8, generator=g)
        ts["model.layers.1.micro_engram.tables.0.weight"] = torch.randn(4, 8, generator=g) * engram_scale
        save_file(ts, str(d / "model.safetensors"))
        return str(d)

    a, same, other = folder("a", 1.0), folder("same", 1.0, engram_scale=3.0), folder("other", 2.0)
    fa = base_fingerprint(a)
    assert fa is not None and len(fa) == 16 and base_fingerprint(other) != fa
    assert base_fingerprint(same) == fa  # an assembled engram inside the folder is not part of the base
    assert base_fingerprint(str(tmp_path / "missing")) is None
    assert base_mismatch({"base_fingerprint": fa}, same) is None
    assert "other base weights" in base_mismatch({"base_fingerprint": fa, "base_model": "a"}, other)
    assert base_mismatch({}, other) is None
