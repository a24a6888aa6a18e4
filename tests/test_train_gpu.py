"""Trainer on the GPU: one optimizer step of a small Gemma-4-style model with an engram, for
every activation-checkpointing policy, with and without activation offloading (layer inputs
above the 1 MiB threshold go to pinned host memory and are prefetched in the backward).
Checkpointing and offloading only move work and memory around: the loss and both gradient
norms must not change."""
import json
import os
import tempfile

import pytest
import torch

pytestmark = pytest.mark.gpu


def _step(tmp, policy, offload, gc=True):
    import bench
    from micro_engram.train.config import load_config
    from micro_engram.train.loop import Trainer
    from micro_engram_fork_b200.models.gemma import tiny_config

    base = os.path.join(tmp, f"base_{policy}_{offload}_{gc}")
    os.makedirs(base)
    json.dump(tiny_config(hidden_size=1024, intermediate_size=2048).to_dict(), open(os.path.join(base, "config.json"), "w"))
    cfg = load_config({
        "base_model": base, "base_init": "random", "datasets": [{"path": "unused.jsonl", "type": "completion"}],
        "output_dir": os.path.join(base, "out"), "sequence_len": 1024, "gradient_accumulation_steps": 2, "max_steps": 2,
        "micro_engram_table_sizes": {2: 4096, 3: 8192, 4: 8192}, "micro_engram_dim": 64, "micro_engram_heads": 2,
        "micro_engram_gate": "scalar_sqrt", "micro_engram_dtype": "bf16", "micro_engram_optimizer": "rowwise_adam",
        "micro_engram_stats_steps": 0, "gradient_checkpointing": gc, "gradient_checkpointing_policy": policy,
        "activation_offloading": offload, "seed": 7,
    })
    t = Trainer(cfg)
    t.build(samples=bench.synthetic_samples(6, 4096, min_len=64, max_len=700, seq=1024), tokenizer=None)
    with torch.no_grad():  # a non-zero output projection, so the tables get gradients at step 0
        for s in t.slots:
            s.engram.value.weight.normal_(std=0.02)
    logs = t.train_step(t.plan.micro_batches(0, 0, 0))
    for s in t.slots:
        s.engram.row_store.check_status()
    return logs


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_checkpoint_policies_and_offload_agree(dist_env):
    tmp = tempfile.mkdtemp()
    runs = {
        "none": _step(tmp, "full", False, gc=False),
        "full": _step(tmp, "full", False),
        "full+offload": _step(tmp, "full", True),
        "selective+offload": _step(tmp, "selective", True),
        "auto+offload": _step(tmp, "auto", True),
    }
    ref = runs["none"]
    assert ref["table_grad_norm"] > 0 and ref["grad_norm"] > 0
    for name, logs in runs.items():
        assert abs(logs["loss"] - ref["loss"]) <= 1e-6 * abs(ref["loss"]), (name, logs["loss"], ref["loss"])
        for key in ("grad_norm", "table_grad_norm"):
            assert abs(logs[key] - ref[key]) <= 1e-3 * ref[key], (name, key, logs[key], ref[key])
