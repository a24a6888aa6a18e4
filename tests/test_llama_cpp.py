"""llama.cpp with the engram bridge against HF Gemma 4 + MicroEngram, on CPU.

Runs where LLAMA_CPP_DIR names a llama.cpp checkout with engram_runtime/llama_cpp/apply.py
applied and libllama built (the CI job `llama-cpp`); skipped everywhere else. A tiny random
Gemma 4 is converted with llama.cpp's own convert_hf_to_gguf.py, a random scalar_sqrt engram is
added with micro_engram.gguf_export, and llama.cpp's logits (engram_runtime/llama_cpp/
llama_logits.cpp: one batch, then ubatches of 5) must match the HF model with the engram
attached by micro_engram.module.attach_engram. Negative control: the HF model without the engram
must differ by far more than the tolerance."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

LLAMA = os.environ.get("LLAMA_CPP_DIR", "")
HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

pytestmark = pytest.mark.skipif(
    not (LLAMA and os.path.isfile(os.path.join(LLAMA, "build", "bin", "libllama.so"))),
    reason="needs LLAMA_CPP_DIR: a llama.cpp checkout with the bridge applied and libllama built")

V, D, LAYERS, ENGRAM_LAYER, T = 384, 64, 6, 2, 40


def _hf_model(folder):
    from transformers import Gemma4ForCausalLM
    from transformers.models.gemma4.configuration_gemma4 import Gemma4TextConfig

    types = ["sliding_attention"] * (LAYERS - 1) + ["full_attention"]
    cfg = Gemma4TextConfig(vocab_size=V, hidden_size=D, intermediate_size=160, num_hidden_layers=LAYERS,
                           num_attention_heads=4, num_key_value_heads=2, head_dim=16, global_head_dim=32,
                           layer_types=types, sliding_window=16, hidden_size_per_layer_input=0,
                           vocab_size_per_layer_input=V, max_position_embeddings=512, final_logit_softcapping=30.0)
    cfg.architectures = ["Gemma4ForCausalLM"]
    torch.manual_seed(3)
    model = Gemma4ForCausalLM(cfg).float().eval()
    with torch.no_grad():  # norm weights away from their init so the norms matter
        for p in model.parameters():
            if p.dim() == 1:
                p.add_(0.15 * torch.randn_like(p))
    model.save_pretrained(folder, safe_serialization=True)
    with open(os.path.join(folder, "tokenizer.json"), "w") as f:  # the converter only counts the vocab
        json.dump({"model": {"vocab": {f"tok{i}": i for i in range(V)}}, "added_tokens": []}, f)
    return model


def _engram():
    from micro_engram.module import MicroEngram

    torch.manual_seed(11)
    e = MicroEngram(model_dim=D, table_size=131, engram_dim=8, num_heads=2, vocab_size=V, gate="scalar_sqrt",
                    orders=(2, 3), seed=ENGRAM_LAYER * 10007)
    with torch.no_grad():
        for t in e.tables:
            t.weight.normal_()
        e.value.weight.normal_(std=0.3)
        e.q_scale.normal_(std=0.2)
        e.k_scale.normal_(std=0.2)
    return e.eval()


def _engram_gguf(tmp, base, e):
    folder = os.path.join(tmp, "engram")
    os.makedirs(folder)
    torch.save({f"model.layers.{ENGRAM_LAYER}.micro_engram.{k}": v for k, v in e.state_dict().items()},
               os.path.join(folder, "w.pt"))
    conf = {"layer": ENGRAM_LAYER, "table_size": e.table_size, "engram_dim": 8, "num_heads": 2, "orders": [2, 3],
            "gate": e.gate, "seed": ENGRAM_LAYER * 10007, "pad_id": 0, "vocab_size": V, "weights": "w.pt"}
    with open(os.path.join(folder, "micro_engram_config.json"), "w") as f:
        json.dump(conf, f)
    from micro_engram.gguf_export import add_engrams

    out = os.path.join(tmp, "model.gguf")
    add_engrams(base, folder, out, dtype="f32", force=True)
    return out


def _driver(tmp):
    exe = os.path.join(tmp, "llama_logits")
    inc = [f"-I{LLAMA}/include", f"-I{LLAMA}/ggml/include"]
    lib = os.path.join(LLAMA, "build", "bin")
    subprocess.run(["g++", "-O2", "-std=c++17", *inc, os.path.join(ROOT, "engram_runtime", "llama_cpp",
                                                                   "llama_logits.cpp"),
                    f"-L{lib}", "-lllama", "-lggml", "-lggml-base", f"-Wl,-rpath,{lib}", "-o", exe], check=True)
    return exe


def test_llama_cpp_bridge_matches_hf(tmp_path):
    from micro_engram.module import attach_engram

    tmp = str(tmp_path)
    hf_dir = os.path.join(tmp, "hf")
    model = _hf_model(hf_dir)
    base = os.path.join(tmp, "base.gguf")
    subprocess.run([sys.executable, os.path.join(LLAMA, "convert_hf_to_gguf.py"), hf_dir, "--outfile", base,
                    "--outtype", "f32"], check=True)
    e = _engram()
    gguf_path = _engram_gguf(tmp, base, e)
    exe = _driver(tmp)
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(1, V, (T,), generator=g)
    ids[10:14] = ids[2:6]  # a repeated n-gram
    tok_file = os.path.join(tmp, "tokens.i32")
    ids.to(torch.int32).numpy().tofile(tok_file)
    with torch.no_grad():
        plain = model(input_ids=ids[None]).logits[0].double()
        attach_engram(model, e, ENGRAM_LAYER, dtype=torch.float32)
        want = model(input_ids=ids[None], position_ids=torch.arange(T)[None]).logits[0].double()
    gap = (want - plain).abs().max().item()
    for ub in (T, 5):
        out = os.path.join(tmp, f"logits_{ub}.f32")
        subprocess.run([exe, gguf_path, tok_file, str(T), out, str(ub)], check=True)
        got = torch.from_numpy(np.fromfile(out, dtype=np.float32).reshape(T, V)).double()
        err = (got - want).abs().max().item()
        assert err < 5e-2, f"ubatch {ub}: llama.cpp differs from HF + engram by {err}"
        assert gap > 20 * err, f"negative control too close: engram effect {gap}, error {err}"
