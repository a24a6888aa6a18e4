"""vLLM serving benchmark of the engram plugin: prefill time to first token
and decode tokens/s of the 31B-class bf16 Gemma-style decoder with two engrams, tensor
parallel over N GPUs of one node.

    python -m micro_engram_fork_b200.utils.serve_bench --tp 2 [--impl ours|reference]
        [--requests 64 --prompt 2048 --gen 256]

Model: the training benchmark's 31B-class config (60 layers, d 5376, 32 q heads, sliding hd256
/ global hd512 5:1, vocab 262144, softcap 30) with random weights (vLLM load_format="dummy")
and two engrams at layers 0 and 29, tables {2: 1572864, 3: 4194304, 4: 4194304} rows x 8 heads
x dim 64, scalar_sqrt gate, rows split over the TP ranks. The engram config sits beside the
model (an assembled model folder), so no weight file is read.

ours       this repository's plugin (micro_engram_vllm): one fused custom op per engram layer
           reads each row from the TP rank that owns it over NVLink (no all-reduce), projects it
           on the tcgen05 GEMM and applies the gate; with --fused-tp the base model's o_proj and
           down_proj also run as the fused GEMM -> reduce-scatter -> all-gather op
           (parallel/tp_linear.py) instead of a library GEMM and vLLM's all-reduce
reference  the reference's plugin from baseline/_ref (masked local lookup + all-reduce)

Workload: `requests` prompts of `prompt` Zipf(1.1) token ids, `gen` greedy tokens each
(ignore_eos). Two timed generate() calls after one warm-up: max_tokens=1 gives the prefill
time to first token of the whole batch (TTFT), max_tokens=gen the full time; decode tokens/s
= requests x (gen - 1) / (full - TTFT). Both are wall-clock around generate() with the GPUs
synchronised (an end-to-end serving number: scheduling, sampling and detokenisation-free
output included). Eager mode (no CUDA graphs) in both arms.
"""
import argparse
import json
import os
import sys
import tempfile
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.abspath(os.path.join(HERE, "..", ".."))
TABLES = {2: 1572864, 3: 4194304, 4: 4194304}
LAYERS = (0, 29)


def _model_folder(tmp):
    sys.path.insert(0, ROOT)
    import bench
    from transformers.models.gemma4.configuration_gemma4 import Gemma4TextConfig

    base = bench.base_config_31b()
    cfg = Gemma4TextConfig(**{k: v for k, v in base.items() if k not in ("architectures", "model_type")})
    cfg.architectures = ["Gemma4ForCausalLM"]
    cfg.max_position_embeddings = 8192
    cfg.save_pretrained(tmp)
    engrams = [{"layer": layer, "table_size": 2097152, "table_sizes": {str(k): v for k, v in TABLES.items()},
                "engram_dim": 64, "num_heads": 8, "orders": [2, 3, 4], "gate": "scalar_sqrt", "seed": layer * 10007,
                "pad_id": 0} for layer in LAYERS]
    conf = dict(engrams[0], engrams=engrams, vocab_size=base["vocab_size"])
    with open(os.path.join(tmp, "micro_engram_config.json"), "w") as f:
        json.dump(conf, f)
    return tmp


def _prompts(n, length, vocab=262144, seed=0):
    import numpy as np

    rng = np.random.default_rng(seed)
    p = np.arange(1, vocab + 1, dtype=np.float64) ** -1.1
    cdf = np.cumsum(p / p.sum())
    return [np.searchsorted(cdf, rng.random(length)).astype(np.int64).tolist() for _ in range(n)]


def _plugin_root(impl):
    return os.path.join(ROOT, "baseline", "_ref") if impl == "reference" else ROOT


def run(args):
    """Build the model folder, then serve it in a child process whose import path holds only the
    chosen plugin (vLLM's worker processes find plugins through their import path, so the two
    arms must never share one)."""
    import subprocess

    plugin = _plugin_root(args.impl)
    if not os.path.isfile(os.path.join(plugin, "micro_engram_vllm", "__init__.py")):
        print(json.dumps({"impl": args.impl, "unavailable": "baseline/_ref is not installed"}))
        return
    if args.impl == "ours":  # the vllm.general_plugins entry point of this repository (in-tree metadata)
        subprocess.run([sys.executable, "setup.py", "-q", "egg_info"], cwd=ROOT, check=True, capture_output=True)
    folder = _model_folder(tempfile.mkdtemp(prefix="me_serve_"))
    env = dict(os.environ, PYTHONPATH=plugin, VLLM_USE_V2_MODEL_RUNNER="1")
    if args.fused_tp and args.impl == "ours":
        env["MICRO_ENGRAM_FUSED_TP"] = "1"
    env.setdefault("VLLM_WORKER_MULTIPROC_METHOD", "fork")
    child = [sys.executable, os.path.abspath(__file__), "--child", folder, "--impl", args.impl, "--tp", str(args.tp),
             "--requests", str(args.requests), "--prompt", str(args.prompt), "--gen", str(args.gen)]
    if args.fused_tp and args.impl == "ours":
        child.append("--fused-tp")
    subprocess.run(child, env=env, cwd=tempfile.gettempdir(), check=True)


def serve(args):
    """The timed serving run (child process: only the arm's plugin is importable)."""
    plugin = _plugin_root(args.impl)
    import micro_engram_vllm
    import torch

    try:
        from vllm import LLM, SamplingParams
    except ImportError as exc:
        print(json.dumps({"impl": args.impl, "unavailable": f"vllm is not importable ({exc})"}))
        return

    where = os.path.abspath(micro_engram_vllm.__file__)
    if not where.startswith(os.path.abspath(plugin) + os.sep) or (args.impl == "reference" and where.startswith(
            os.path.join(ROOT, "micro_engram_vllm"))):
        raise SystemExit(f"serve_bench: the {args.impl} arm imported the plugin from {where}")
    micro_engram_vllm.register()
    llm = LLM(model=args.child, skip_tokenizer_init=True, dtype="bfloat16", load_format="dummy", enforce_eager=True,
              tensor_parallel_size=args.tp, distributed_executor_backend="mp" if args.tp > 1 else None,
              max_model_len=args.prompt + args.gen + 16, max_num_seqs=args.requests,
              max_num_batched_tokens=max(8192, args.prompt), gpu_memory_utilization=0.85)
    prompts = [{"prompt_token_ids": p} for p in _prompts(args.requests, args.prompt)]
    first = SamplingParams(max_tokens=1, temperature=0.0, ignore_eos=True, detokenize=False)
    full = SamplingParams(max_tokens=args.gen, temperature=0.0, ignore_eos=True, detokenize=False)
    llm.generate(prompts[: min(8, len(prompts))], full)  # warm-up
    times = {}
    for name, sp in (("ttft", first), ("full", full)):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        outs = llm.generate(prompts, sp)
        torch.cuda.synchronize()
        times[name] = time.perf_counter() - t0
        n_out = sum(len(o.outputs[0].token_ids) for o in outs)
        assert n_out == len(prompts) * sp.max_tokens, (n_out, sp.max_tokens)
    decode_tps = args.requests * (args.gen - 1) / max(times["full"] - times["ttft"], 1e-9)
    print(json.dumps({
        "impl": args.impl, "metric": "vLLM TP decode tok/s (config 5)", "value": round(decode_tps, 1),
        "unit": "tokens/s", "tp": args.tp, "prefill_ttft_s": round(times["ttft"], 3),
        "full_s": round(times["full"], 3), "higher_is_better": True, "dtype": "bf16",
        "fused_tp_linears": bool(args.fused_tp and args.impl == "ours"),
        "data": "synthetic Zipf(1.1) prompts, random (dummy) weights", "plugin": where,
        "config": {"model": "31B-class Gemma-style hybrid decoder + engrams at layers 0 and 29",
                   "requests": args.requests, "prompt_tokens": args.prompt, "gen_tokens": args.gen,
                   "tables": TABLES, "cuda_graphs": False,
                   "timing": "wall clock around generate(), GPUs synchronised; decode = (full - ttft)"}}), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--requests", type=int, default=64)
    ap.add_argument("--prompt", type=int, default=2048)
    ap.add_argument("--gen", type=int, default=256)
    ap.add_argument("--fused-tp", action="store_true",
                    help="ours: o_proj / down_proj GEMM + all-reduce as the fused peer-memory op")
    ap.add_argument("--child", default="", help=argparse.SUPPRESS)  # internal: serve this model folder
    args = ap.parse_args()
    if args.child:
        serve(args)
    else:
        run(args)


if __name__ == "__main__":
    main()
