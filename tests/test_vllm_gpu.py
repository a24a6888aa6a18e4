"""End to end through real vLLM on one GPU: a small random Gemma 4 checkpoint plus an engram
config, served by vLLM with this repository's plugin (fused serve_inject op, history fill
kernel, V2 runner), must give the prompt log-probs and the greedy continuation of the HF
transformers model with the same engram attached (micro_engram.module.attach_engram).

The vLLM engine runs in a child process (in-process engine core, so the plugin registered
there is the one the model runner sees). With tensor parallelism 2 the table rows are split
over the two GPUs' row stores and the fused op reads the other GPU's rows over NVLink; the
TP worker processes find the plugin through the `vllm.general_plugins` entry point of the
in-tree egg-info (`setup.py egg_info`), as an installed package would provide it."""
import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

LAYER, V, D = 1, 512, 256


def _build(folder):
    from transformers import Gemma4ForCausalLM
    from transformers.models.gemma4.configuration_gemma4 import Gemma4TextConfig

    from micro_engram.module import MicroEngram

    cfg = Gemma4TextConfig(vocab_size=V, hidden_size=D, intermediate_size=512, num_hidden_layers=4,
                           num_attention_heads=4, num_key_value_heads=2, head_dim=64, global_head_dim=128,
                           num_global_key_value_heads=1, attention_k_eq_v=True, hidden_size_per_layer_input=0,
                           layer_types=["sliding_attention", "sliding_attention", "sliding_attention",
                                        "full_attention"], sliding_window=16, final_logit_softcapping=30.0,
                           max_position_embeddings=512, tie_word_embeddings=True)
    torch.manual_seed(0)
    hf = Gemma4ForCausalLM(cfg).to(torch.bfloat16)
    hf.save_pretrained(folder)
    eng = MicroEngram(model_dim=D, table_size=1021, engram_dim=32, num_heads=2, vocab_size=V, gate="scalar_sqrt",
                      seed=LAYER * 10007)
    with torch.no_grad():
        for t in eng.tables:
            t.weight.normal_(std=1.0)
        eng.value.weight.normal_(std=0.2)
        eng.q_scale.normal_(std=0.1)
        eng.k_scale.normal_(std=0.1)
    sd = {f"model.layers.{LAYER}.micro_engram.{k}": v for k, v in eng.state_dict().items()}
    torch.save(sd, os.path.join(folder, "engram.pt"))
    conf = {"layer": LAYER, "table_size": 1021, "engram_dim": 32, "num_heads": 2, "gate": "scalar_sqrt",
            "seed": LAYER * 10007, "orders": [2, 3], "pad_id": 0, "weights": "engram.pt"}
    with open(os.path.join(folder, "engram_config.json"), "w") as f:
        json.dump(conf, f)
    return hf, eng


def _hf_logprobs(hf, eng, ids):
    """log-softmax over `ids` of the HF model without, then with the engram attached."""
    from micro_engram.module import attach_engram

    dev = torch.device("cuda", 0)
    model = hf.to(dev)
    x = torch.tensor([ids], device=dev)
    with torch.no_grad():
        plain = torch.log_softmax(model(input_ids=x).logits[0].float(), -1).cpu()
        attach_engram(model, eng.to(dev).to(torch.bfloat16), LAYER)
        withe = torch.log_softmax(model(input_ids=x).logits[0].float(), -1).cpu()
    return plain, withe


def _serve(folder, prompt, n_new, tp=1, fused=False):
    os.environ["VLLM_ENABLE_V1_MULTIPROCESSING"] = "0"
    os.environ["VLLM_USE_V2_MODEL_RUNNER"] = "1"
    if tp > 1:
        os.environ["VLLM_WORKER_MULTIPROC_METHOD"] = "fork"
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import micro_engram_vllm
    from vllm import LLM, SamplingParams

    micro_engram_vllm.register()
    extra = {"tensor_parallel_size": tp, "distributed_executor_backend": "mp"} if tp > 1 else {}
    llm = LLM(model=folder, skip_tokenizer_init=True, dtype="bfloat16", enforce_eager=True, max_model_len=256,
              gpu_memory_utilization=0.2, max_num_seqs=4,
              additional_config={"micro_engram": os.path.join(folder, "engram_config.json"),
                                 "micro_engram_fused_tp": fused}, **extra)
    sp = SamplingParams(max_tokens=n_new, temperature=0.0, prompt_logprobs=0, logprobs=0, detokenize=False)
    out = llm.generate([{"prompt_token_ids": prompt}], sp)[0]
    prompt_lp = [None] + [next(iter(d.values())).logprob for d in out.prompt_logprobs[1:]]
    gen = list(out.outputs[0].token_ids)
    gen_lp = [next(iter(d.values())).logprob for d in out.outputs[0].logprobs]
    return prompt_lp, gen, gen_lp


def _main(folder, tp, fused):
    torch.manual_seed(3)
    prompt = torch.randint(3, V, (40,)).tolist()
    prompt_lp, gen, gen_lp = _serve(folder, prompt, 8, tp, fused)
    with open(os.path.join(folder, "served.json"), "w") as f:
        json.dump({"prompt": prompt, "prompt_lp": prompt_lp, "gen": gen, "gen_lp": gen_lp}, f)


@pytest.mark.parametrize("tp,fused", [(1, False), (2, False), (2, True)])
def test_vllm_serves_engram_like_hf(tmp_path, tp, fused):
    """fused: the row-parallel linears' GEMM + all-reduce replaced by the fused peer-memory op."""
    pytest.importorskip("vllm")
    if torch.cuda.device_count() < tp:
        pytest.skip(f"needs {tp} GPUs")
    folder = str(tmp_path)
    if tp > 1:  # TP workers load plugins through entry points: an in-tree egg-info declares ours
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        subprocess.run([sys.executable, "setup.py", "-q", "egg_info"], cwd=root, check=True, capture_output=True)
    hf, eng = _build(folder)
    env = dict(os.environ, PYTHONPATH=os.pathsep.join([os.path.dirname(os.path.dirname(__file__)),
                                                       os.environ.get("PYTHONPATH", "")]))
    r = subprocess.run([sys.executable, __file__, folder, str(tp), str(int(fused))], env=env, capture_output=True,
                       text=True, timeout=900)
    if fused:
        assert "row-parallel linears fused" in r.stdout + r.stderr, "the fused op was not switched on"
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-6000:]
    with open(os.path.join(folder, "served.json")) as f:
        s = json.load(f)
    seq = s["prompt"] + s["gen"]
    plain, ref = _hf_logprobs(hf, eng, seq)
    want_prompt = [float(ref[t - 1, seq[t]]) for t in range(1, len(s["prompt"]))]
    got_prompt = s["prompt_lp"][1:]
    err = max(abs(a - b) for a, b in zip(got_prompt, want_prompt))
    assert err < 0.15, f"prompt log-probs differ from HF + engram by {err}"
    n = len(s["prompt"])
    want_gen = [float(ref[n - 1 + i, seq[n + i]]) for i in range(len(s["gen"]))]
    err_g = max(abs(a - b) for a, b in zip(s["gen_lp"], want_gen))
    assert err_g < 0.15, f"decode log-probs differ from HF + engram by {err_g}"
    # the greedy token at every decode step is HF's argmax (or within bf16 noise of it)
    for i, tok in enumerate(s["gen"]):
        row = ref[n - 1 + i]
        assert float(row.max() - row[tok]) < 0.15, f"decode step {i}: token {tok} is not HF's greedy choice"
    # the engram matters: without it the prompt log-probs move by far more than the tolerance
    moved = max(abs(float(plain[t - 1, seq[t]]) - w) for t, w in zip(range(1, n), want_prompt))
    assert moved > 4 * max(err, 0.02), f"the engram moves the log-probs by only {moved}; the check shows nothing"


if __name__ == "__main__":
    _main(sys.argv[1], int(sys.argv[2]) if len(sys.argv) > 2 else 1, len(sys.argv) > 3 and sys.argv[3] == "1")
