"""Headline benchmark: stage-1 engram training throughput of the 31B-class Gemma-style hybrid
decoder at seq 8192, on N GPUs of one node.

  python bench.py --gpus N --steps K --warmup W          (N=1)
  torchrun --nproc-per-node N bench.py --gpus N ...       (N>1, one rank per GPU)
  python bench.py --impl reference ...                    (the unmodified reference)
  python bench.py --config 4 ...                          (NF4 base, engrams at
                                                           layers 0 and 29, synthetic 10% canon)

Config: 60 layers, d 5376, FFN 21504, 32 q heads, sliding-1024 layers (16 KV heads, head_dim
256) interleaved 5:1 with global layers (4 KV heads, head_dim 512, v = k), vocab 262144 tied
with final softcap 30; frozen random-init bf16 base; one engram at layer 0 with 2/3/4-gram
tables {1572864, 4194304, 4194304} x 8 heads x dim 64 (scalar_sqrt gate, rowwise_adam, bf16 +
stochastic rounding); seq 8192, micro-batch 1, grad accumulation 3, per-layer activation
checkpointing + activation offloading; synthetic packed Zipf(1.1) token documents of uniform
length 256-4096 (weak scaling: every GPU trains its own micro-batches).

Timing: W untimed warm-up steps, then K steps bracketed by a barrier + synchronize, timed with
CUDA events on the launching stream, max over ranks. Each step streams the ~61 GB base through
the GPU several times, far more than the 126 MB L2, so no flush is needed between steps.
`value` is the device-timed step (inputs staged on the device beforehand); `e2e` repeats the
K steps through the public `Trainer.train_step` API, which collates each step's micro-batches
on the host, copies them from pinned memory and reads the loss back.
"""
import argparse
import json
import os
import re
import subprocess
import sys
import tempfile

METRIC = "train tokens/s (31B-class, seq 8192)"
MODEL = "31B-class Gemma-style hybrid decoder (60L, d5376, FFN 21504, 32q heads, sliding hd256x16kv / global hd512x4kv 5:1, V=262144), stage-1 engram"
SEQ, MBS, GA = 8192, 1, 3
TABLES = {2: 1572864, 3: 4194304, 4: 4194304}
BASELINE_VALUE = None  # the reference publishes no tokens/s figure, so vs_baseline is null


def base_config_31b():
    return {
        "architectures": ["Gemma4ForCausalLM"], "model_type": "gemma4_text",
        "vocab_size": 262144, "hidden_size": 5376, "intermediate_size": 21504, "num_hidden_layers": 60,
        "num_attention_heads": 32, "num_key_value_heads": 16, "head_dim": 256, "global_head_dim": 512,
        "num_global_key_value_heads": 4, "attention_k_eq_v": True, "sliding_window": 1024,
        "final_logit_softcapping": 30.0, "rms_norm_eps": 1e-6, "pad_token_id": 0, "eos_token_id": 1,
        "bos_token_id": 2, "tie_word_embeddings": True, "hidden_size_per_layer_input": 0,
        "layer_types": ["sliding_attention" if (i + 1) % 6 else "full_attention" for i in range(60)],
        "rope_parameters": {"sliding_attention": {"rope_type": "default", "rope_theta": 10000.0},
                            "full_attention": {"rope_type": "proportional", "partial_rotary_factor": 0.25,
                                               "rope_theta": 1000000.0}},
    }


def synthetic_samples(n_bins, vocab, seed=1234, min_len=256, max_len=4096, seq=SEQ):
    """Zipf(1.1) token documents of uniform length min_len-max_len, enough for n_bins bins of seq."""
    import numpy as np

    from micro_engram.train.data import Samples

    rng = np.random.default_rng(seed)
    ranks = np.arange(1, vocab + 1, dtype=np.float64)
    p = ranks ** -1.1
    cdf = np.cumsum(p / p.sum())
    items, total = [], 0
    need = n_bins * seq * 1.15
    while total < need:
        n = int(rng.integers(min_len, max_len + 1))
        ids = np.searchsorted(cdf, rng.random(n)).astype(np.int32)
        items.append((ids, None))
        total += n
    return Samples.from_list(items)


METRIC4 = "train tokens/s (31B-class NF4, 2 engrams, seq 8192)"
MODEL4 = MODEL.replace("stage-1 engram", "NF4 frozen base (block 64, fp32 absmax), engrams at layers 0 and 29")


def synthetic_canon(path, vocab=262144, share=0.10, seed=1):
    """Config 4's canon map: a random `share` of the vocabulary ids (seed 1) is paired up, and
    each pair shares one canonical id (the smaller of the two). Idempotent."""
    import numpy as np
    import torch

    rng = np.random.default_rng(seed)
    n = int(share * vocab) // 2 * 2
    pairs = rng.choice(vocab, size=n, replace=False).reshape(-1, 2)
    canon = np.arange(vocab, dtype=np.int64)
    canon[pairs.max(1)] = pairs.min(1)
    torch.save(torch.from_numpy(canon), path)
    return path


def bench_config(tmp, steps, config=3):
    base = os.path.join(tmp, "base")
    os.makedirs(base, exist_ok=True)
    with open(os.path.join(base, "config.json"), "w") as f:
        json.dump(base_config_31b(), f)
    if config == 4:  # NF4 base, a second engram at layer 29, a synthetic 10% canon
        c = bench_config(tmp, steps)
        c.update({"load_in_4bit": True, "base_placement": "replicated",
                  "micro_engram_extra": [{"layer": 29}],
                  "micro_engram_canon_path": synthetic_canon(os.path.join(tmp, "canon.pt"))})
        return c
    return {
        "base_model": base, "base_init": "random",
        "datasets": [{"path": os.path.join(tmp, "unused.jsonl"), "type": "completion"}],
        "output_dir": os.path.join(tmp, "out"), "sequence_len": SEQ,
        "micro_batch_size": MBS, "gradient_accumulation_steps": GA, "max_steps": steps,
        "micro_engram_layer": 0, "micro_engram_table_size": 2097152, "micro_engram_table_sizes": TABLES,
        "micro_engram_dim": 64, "micro_engram_heads": 8, "micro_engram_gate": "scalar_sqrt",
        "micro_engram_dtype": "bf16", "micro_engram_optimizer": "rowwise_adam",
        "learning_rate": 5e-3, "micro_engram_dense_lr": 1e-3, "max_grad_norm": 2.0, "warmup_steps": 0,
        "gradient_checkpointing": True, "activation_offloading": True, "micro_engram_stats_steps": 0,
        "gradient_checkpointing_policy": os.environ.get("ME_BENCH_AC", "auto"),
        "gradient_checkpointing_reserve_gib": float(os.environ.get("ME_BENCH_AC_RESERVE", "23")),
        # config 3 is FSDP2: the frozen base row-sharded over the GPUs (ME_BENCH_PLACEMENT=replicated
        # runs the replicated-base variant instead)
        "base_placement": os.environ.get("ME_BENCH_PLACEMENT", "sharded"),
        "seed": 42,
    }


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx = float(parts[2])
                except ValueError:
                    continue
                for name, val in zip(names, parts[5:9]):
                    if val.lower() == "active":
                        reasons.add(name)
        os.unlink(self.path)
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def count_launches(trainer, micro):
    """Kernels of our extension launched by one step (profiled outside the timed region)."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    ours = ("hash_kernel", "hash_prev_kernel", "gather_kernel", "scatter_grad_kernel", "touched_sqnorm_kernel",
            "clip_coef_kernel", "adam_touched_kernel", "adam_dense_kernel", "gate_fwd_kernel", "gate_bwd_kernel",
            "gate_fwd_vec_kernel", "gate_bwd_vec_kernel", "fill_ids_kernel", "rmsnorm_fwd_kernel",
            "rmsnorm_bwd_kernel", "post_norm_add_kernel", "post_norm_add_bwd_kernel", "qkv_norm_rope_kernel",
            "qkv_norm_rope_bwd_kernel", "geglu_fwd_kernel", "geglu_bwd_kernel", "ce_fwd_kernel", "ce_bwd_kernel",
            "attn_fwd_kernel", "attn_fwd_tc_kernel", "attn_bwd_pre_kernel", "attn_bwd_dkdv_kernel",
            "attn_bwd_dq_kernel", "attn_bwd_tc_kernel", "attn_delta_kernel", "doc_end_from_start_kernel",
            "attn_tiles_kernel", "attn_bwd_sdp_kernel", "attn_bwd_acc_kernel",
            "gemm_pair_kernel", "nf4_dequant_kernel", "nf4_quantize_kernel", "p2p_allreduce_mean_kernel",
            "layer_gather_kernel", "p2p_gather_kernel", "p2p_sum_slots_kernel", "row_push_kernel",
            "row_accumulate_kernel", "rows_serve_kernel", "rows_collect_kernel", "adam_rows_kernel")
    pat = re.compile(r"\b(" + "|".join(ours) + r")\b")
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        trainer.train_step(micro)
        torch.cuda.synchronize()
    dump = os.environ.get("ME_BENCH_KERNEL_TABLE")
    if dump:  # per-kernel device time of this one (untimed) step, for finding the next target
        with open(dump, "w") as f:
            f.write(prof.key_averages().table(sort_by="device_time_total", row_limit=60, max_name_column_width=90))
    n_ours, n_all = 0, 0
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA:
            n_all += 1
            if pat.search(ev.name):
                n_ours += 1
    return n_ours, n_all


def phase_breakdown(trainer, micro, world):
    """Device time per phase of one untimed step (CUDA events around embed / forward / loss /
    backward / reduce / optimizer), max over ranks, plus the spread of the whole step over ranks."""
    import torch
    import torch.distributed as dist

    from micro_engram_fork_b200.utils.timers import PhaseTimers

    timers, trainer.timers = trainer.timers, PhaseTimers(enabled=True, device=trainer.device)
    try:
        trainer.train_step(micro)
        ms = trainer.timers.report()
    finally:
        trainer.timers = timers
    names = sorted(ms)
    vals = torch.tensor([ms[n] for n in names] + [sum(ms.values())], dtype=torch.float64, device=trainer.device)
    lo = vals.clone()
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
        dist.all_reduce(lo, op=dist.ReduceOp.MIN)
    out = {n: round(v, 2) for n, v in zip(names, vals.tolist())}
    out["step_max_over_ranks"] = round(vals[-1].item(), 2)
    out["step_min_over_ranks"] = round(lo[-1].item(), 2)
    return out


def run_ours(args):
    import torch
    import torch.distributed as dist

    from micro_engram.train.config import load_config
    from micro_engram.train.data import collate
    from micro_engram.train.loop import Trainer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    steps_total = args.warmup + 2 * args.steps + 1
    tmp = tempfile.mkdtemp(prefix="me_bench_")
    cfg = load_config(bench_config(tmp, steps_total, args.config))
    trainer = Trainer(cfg)
    rank, device = trainer.rank, trainer.device
    n_bins = steps_total * GA * MBS * world + 8
    samples = synthetic_samples(n_bins, 262144)
    trainer.build(samples=samples, tokenizer=None)
    plan = trainer.plan

    def sync():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    step_idx = 0

    def next_micro():
        nonlocal step_idx
        m = plan.micro_batches(0, step_idx, rank)
        step_idx += 1
        return m

    for _ in range(args.warmup):
        trainer.train_step(next_micro())
    n_ours, n_all = count_launches(trainer, next_micro())
    phases = phase_breakdown(trainer, next_micro(), world)

    # device-timed: inputs staged on the GPU before the timed region
    staged = []
    for _ in range(args.steps):
        micro = next_micro()
        staged.append((micro, [{k: v.to(device) for k, v in collate(trainer.samples, b, SEQ, trainer.pad_id).items()}
                               for b in micro]))
    clocks = Clocks(int(os.environ.get("LOCAL_RANK", 0)))
    sync()
    clocks.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    tokens = 0
    t0.record()
    for micro, batches in staged:
        trainer.train_step(micro, batches=batches, sync=False)  # no host read: the device-timed loop
        tokens += SEQ * MBS * GA
    t1.record()
    sync()
    clk = clocks.stop()
    dev_ms = t0.elapsed_time(t1)

    # end to end through the public API: host collate + pinned H2D + loss readback each step
    sync()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        trainer.train_step(next_micro())
    e1.record()
    sync()
    e2e_ms = e0.elapsed_time(e1)
    # a kernel-side error (row-store bounds/capacity, a bounded peer wait that ran out) fails the run
    for slot in trainer.slots:
        store = slot.engram.__dict__.get("row_store")
        if store is not None:
            store.check_status()
    if getattr(trainer, "_p2p_ar", None) is not None:
        trainer._p2p_ar.check_status()

    vals = torch.tensor([dev_ms, e2e_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    dev_ms, e2e_ms = vals.tolist()
    ms_step = dev_ms / args.steps
    value = tokens * world / (dev_ms / 1e3)
    e2e_value = tokens * world / (e2e_ms / 1e3)
    if rank == 0:
        parallelism = (f"fsdp{world} (row-sharded frozen base, layer all-gathers carried by the tcgen05 GEMMs; "
                       "row-sharded engram; vocab-parallel head)" if trainer.placement == "sharded" else
                       f"dp{world} (replicated frozen base, row-sharded engram, vocab-parallel head)")
        engram = ("layer 0, tables {2:1572864,3:4194304,4:4194304} x8 heads x dim 64, scalar_sqrt, "
                  "rowwise_adam bf16+SR")
        if args.config == 4:
            engram = "layers 0 and 29 (same tables each), synthetic canon pairing 10% of the vocabulary; " + engram
        line = {
            "metric": METRIC if args.config == 3 else METRIC4, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 2),
            "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None if not BASELINE_VALUE else round(value / BASELINE_VALUE, 4),
            "dtype": "bf16", "data": "synthetic (Zipf(1.1) packed docs 256-4096, random-init weights)",
            "config": {"model": MODEL if args.config == 3 else MODEL4, "global_batch": MBS * GA * world,
                       "seq_len": SEQ, "baseline_config": args.config, "parallelism": parallelism, "engram": engram,
                       "activation_checkpointing": f"per-layer, policy {trainer.cfg.gradient_checkpointing_policy}"
                                                   " (HBM-budgeted: selective = q/k/v projection, attention output"
                                                   " and o-proj kept on the GPU, norms/RoPE/MLP recomputed; none ="
                                                   " nothing recomputed)",
                       "activation_checkpointing_plan": getattr(trainer, "ckpt_plan", None),
                       "table_moments_on_host": getattr(trainer, "table_moments_on_host", None),
                       "peak_hbm_reserved_gib": round(torch.cuda.max_memory_reserved() / 2 ** 30, 1),
                       "activation_offloading": "layer inputs to pinned host memory, prefetched in the backward",
                       "l2": "inputs larger than L2 (61 GB base streamed per step), no flush"},
            "clocks": clk,
            "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": GA * 3 * SEQ * MBS * 8, "d2h_bytes_per_step": 16},
            "gpu_launches": n_ours * args.steps,
            "gpu_launches_all_per_step": n_all,
            "phase_ms_one_step": phases,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _purge_micro_engram():
    for k in list(sys.modules):
        if k == "micro_engram" or k.startswith("micro_engram.") or k.startswith("micro_engram_vllm"):
            del sys.modules[k]


def run_reference(args):
    """The unmodified reference (baseline/_ref) through its own Trainer: build() and
    train_step() run stock. Two setup inputs are replaced because the benchmark prescribes
    synthetic ones and the stock loaders cannot provide them here: the base model is a
    random-init HF Gemma4ForCausalLM of the 31B config built on the GPU (the stock
    load_base calls from_pretrained(device_map=...), which needs `accelerate`, not installed
    offline), and the samples are the same synthetic token documents as our arm (the stock
    prepare() tokenizes JSONL text). Everything timed is the reference's own code."""
    here = os.path.dirname(os.path.abspath(__file__))
    ref_root = os.path.join(here, "baseline", "_ref")
    if not os.path.isfile(os.path.join(ref_root, "micro_engram", "train", "loop.py")):
        print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref is not installed"}))
        return
    import numpy as np  # noqa: F401
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world == 1 and "MASTER_ADDR" not in os.environ:  # single process without a launcher
        import socket

        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            os.environ["MASTER_PORT"] = str(s.getsockname()[1])
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ.setdefault("RANK", "0")
        os.environ.setdefault("LOCAL_RANK", "0")
    samples_ours = synthetic_samples(
        (args.warmup + 2 * args.steps + 2) * GA * MBS * world + 8, 262144)  # generated with our helper
    toks, offs = samples_ours.tokens, samples_ours.offsets
    _purge_micro_engram()
    sys.path.insert(0, ref_root)
    try:
        import micro_engram.train.loop as L
        import micro_engram.train.model as RM
        from micro_engram.train.config import load_config
        from micro_engram.train.data import Samples
    finally:
        sys.path.pop(0)
    assert os.path.abspath(L.__file__).startswith(ref_root), L.__file__
    from transformers import Gemma4ForCausalLM, PreTrainedTokenizerFast
    from transformers.models.gemma4.configuration_gemma4 import Gemma4TextConfig

    tmp = tempfile.mkdtemp(prefix="me_ref_")
    c = bench_config(tmp, args.warmup + 2 * args.steps + 2, 3)
    for k in ("base_init", "gradient_checkpointing_policy", "gradient_checkpointing_reserve_gib",
              "base_placement"):  # not reference keys
        c.pop(k)
    # the reference's recommended B200-runnable kernel settings (README example config)
    # (fused_attn_kernel off: that patch's shared-KV side channel is None under the installed
    # transformers and the stock layer then fails; its unfused path is the reference's own option)
    c.update({"gemma4_hybrid_attn_impl": True, "large_head_attention": "auto", "liger_rms_norm": True,
              "liger_glu_activation": True, "attn_implementation": "sdpa", "fused_attn_kernel": False})
    try:
        import flash_attn  # noqa: F401
        from flash_attn import flash_attn_func

        q = torch.randn(1, 64, 2, 64, device="cuda", dtype=torch.bfloat16)
        flash_attn_func(q, q, q, causal=True)
        torch.cuda.synchronize()
        c["attn_implementation"] = "flash_attention_2"
    except Exception:  # noqa: BLE001 - FA2 without sm_100 kernels: the stock sdpa path
        pass
    # a minimal tokenizer folder: the reference reads only pad_token_id from it
    from tokenizers import Tokenizer, models

    tk = Tokenizer(models.WordLevel({"<pad>": 0, "<eos>": 1, "<bos>": 2, "<unk>": 3}, unk_token="<unk>"))
    PreTrainedTokenizerFast(tokenizer_object=tk, pad_token="<pad>", eos_token="<eos>",
                            bos_token="<bos>").save_pretrained(c["base_model"])
    cfg = load_config(c)
    hf_conf = Gemma4TextConfig(**{k: v for k, v in base_config_31b().items()
                                  if k not in ("architectures", "model_type")})

    def random_base(cfg_, rank, local_rank, device):
        torch.manual_seed(cfg_.seed)
        with torch.device(device):
            model = Gemma4ForCausalLM._from_config(hf_conf, dtype=torch.bfloat16,
                                                   attn_implementation=cfg_.attn_implementation)
        for p in model.parameters():
            p.requires_grad_(False)
        return model, False

    RM.load_base = random_base
    L.prepare = lambda *a, **k: Samples(toks, np.ones_like(toks, dtype=bool), offs)
    trainer = L.Trainer(cfg)
    trainer.build()
    rank, device = trainer.rank, trainer.device
    plan = trainer.plan

    def sync():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for i in range(args.warmup):
        trainer.train_step(plan.micro_batches(0, i, rank))
    sync()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(args.steps):
        trainer.train_step(plan.micro_batches(0, args.warmup + i, rank))
    t1.record()
    sync()
    ms = torch.tensor([t0.elapsed_time(t1)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms)
    value = SEQ * MBS * GA * args.steps * world / (ms / 1e3)
    if rank == 0:
        # the stock train_step collates each step on the host, copies it to the GPU and reads the
        # loss back, so this timed loop is already end to end through the reference's public API
        e2e = {"value": round(value, 1), "unit": "tokens/s", "h2d_bytes_per_step": GA * 3 * SEQ * MBS * 8,
               "d2h_bytes_per_step": 8, "note": "the timed loop itself (stock Trainer.train_step)"}
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (same token documents as our arm), random-init weights",
            "config": {"model": MODEL, "global_batch": MBS * GA * world, "seq_len": SEQ,
                       "parallelism": f"fsdp2 dp{world} (reference)", "attn_implementation": cfg.attn_implementation,
                       "e2e_note": "reference Trainer.train_step: host collate + H2D + loss readback each step"},
            "e2e": e2e,
        }), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, choices=[3, 4], default=3,
                    help="BASELINE config: 3 = bf16 base, one engram (headline); 4 = NF4 base, two engrams")
    args = ap.parse_args()
    if args.warmup < 3:
        print("bench: at least 3 warm-up steps", file=sys.stderr)
        args.warmup = 3
    if args.impl == "reference" and args.config == 4:
        print(json.dumps({"impl": "reference", "metric": METRIC4, "unavailable":
                          "the reference's NF4 base needs bitsandbytes and accelerate, neither installed offline"}))
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    main()
