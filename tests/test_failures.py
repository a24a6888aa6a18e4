"""Failure detection, recovery and determinism of micro_engram.train on CPU (gloo ranks).

Faults are made on the host only (MICRO_ENGRAM_FAULT, micro_engram/train/faults.py): a rank
raises between steps, with none of its collectives in flight. The survivors learn of it in
their next collective (gloo sees the connection close) and fail fast, so the whole job ends
instead of hanging; the run then resumes from its last complete checkpoint on FEWER ranks
(3 -> 2: the row-sharded tables reshard on load) and finishes. A step rerun from the same
state gives bitwise the same loss and the same table rows."""
import json
import os
import subprocess
import sys
import time

import pytest
import torch
import yaml

from helpers import run_dist
from test_train_cpu import base_cfg, make_assets

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_fault_spec():
    from micro_engram.train.faults import FaultHook, FaultInjected, parse_fault

    assert parse_fault(None) is None and parse_fault("") is None
    assert parse_fault("2:5") == (2, 5, "raise") and parse_fault("0:1:exit") == (0, 1, "exit")
    for bad in ("1", "a:b", "1:2:explode", "1:2:3:4"):
        with pytest.raises(ValueError):
            parse_fault(bad)
    hook = FaultHook(rank=1, spec="1:3")
    hook.before_step(2)
    FaultHook(rank=0, spec="1:3").before_step(3)  # another rank's fault
    with pytest.raises(FaultInjected):
        hook.before_step(3)


@pytest.fixture(scope="module")
def assets(tmp_path_factory):
    root = str(tmp_path_factory.mktemp("failures"))
    model_dir, data = make_assets(root)
    return root, model_dir, data


def _launch(world, cfg_path, port, extra_env):
    procs = []
    for rank in range(world):
        env = dict(os.environ, RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(port), MICRO_ENGRAM_CPU="1", PYTHONPATH=ROOT, **extra_env)
        procs.append(subprocess.Popen([sys.executable, "-m", "micro_engram.train", cfg_path], env=env, cwd=ROOT,
                                      stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True))
    return procs


def _wait(procs, limit_s):
    """(exit codes, outputs, seconds) once every process has ended; kills what is still
    running at the limit (exit code None)."""
    t0 = time.time()
    codes = [None] * len(procs)
    while time.time() - t0 < limit_s and any(c is None for c in codes):
        codes = [p.poll() for p in procs]
        time.sleep(0.5)
    outs = []
    for p, c in zip(procs, codes):
        if c is None:
            p.kill()
        outs.append(p.communicate()[0])
    return codes, outs, time.time() - t0


def test_survivors_fail_fast_then_resume_on_fewer_ranks(assets):
    from conftest import free_port

    root, model_dir, data = assets
    out = os.path.join(root, "run")
    cfg = base_cfg(root, model_dir, data, out, save_steps=1, max_steps=4, micro_engram_extra=None,
                   micro_engram_stats_steps=0)
    cfg_path = os.path.join(root, "cfg.yaml")
    with open(cfg_path, "w") as f:
        yaml.safe_dump(cfg, f)
    # rank 1 fails before step 3; ranks 0 and 2 are in (or entering) step 3's collectives
    procs = _launch(3, cfg_path, free_port(), {"MICRO_ENGRAM_FAULT": "1:3", "MICRO_ENGRAM_PG_TIMEOUT_S": "60"})
    codes, outs, took = _wait(procs, 300)
    assert all(c is not None for c in codes), f"ranks still running after {took:.0f} s: {codes}\n" + outs[0][-3000:]
    assert all(c != 0 for c in codes), codes
    assert "injected fault on rank 1 before step 3" in outs[1], outs[1][-3000:]
    done = sorted(d for d in os.listdir(out) if d.startswith("checkpoint-")
                  and os.path.isfile(os.path.join(out, d, "trainer_state.json")))
    assert done == ["checkpoint-1", "checkpoint-2"], done
    # the same run on 2 ranks resumes from checkpoint-2 and finishes
    codes, outs, took = _wait(_launch(2, cfg_path, free_port(), {}), 300)
    assert codes == [0, 0], (codes, outs[0][-3000:])
    assert "resumed from" in outs[0] and "checkpoint-2" in outs[0], outs[0][-3000:]
    with open(os.path.join(out, "checkpoint-4", "trainer_state.json")) as f:
        assert json.load(f)["global_step"] == 4
    with open(os.path.join(out, "train_log.jsonl")) as f:
        steps = [json.loads(x)["step"] for x in f]
    assert steps[-2:] == [3, 4], steps


def _rerun(rank, world, root, model_dir, data):
    from micro_engram.train.config import load_config
    from micro_engram.train.loop import Trainer

    results = []
    for attempt in range(2):
        cfg = base_cfg(root, model_dir, data, os.path.join(root, f"det{attempt}"))
        t = Trainer(load_config(cfg))
        t.build()
        with torch.no_grad():  # a trained-looking output projection: the rows get real gradients
            for s in t.slots:
                s.engram.value.weight.copy_(torch.randn(s.engram.value.weight.shape,
                                                        generator=torch.Generator().manual_seed(3)))
        logs = t.train_step(t.plan.micro_batches(0, 0, rank))
        rows = torch.cat([p.detach().reshape(-1) for s in t.slots for p in s.engram.row_shards])
        results.append((logs["loss"], logs["table_grad_norm"], rows))
    (l0, n0, r0), (l1, n1, r1) = results
    return {"same_loss": l0 == l1, "same_norm": n0 == n1, "same_rows": torch.equal(r0, r1)}


def test_step_is_deterministic(assets):
    root, model_dir, data = assets
    for rank, res in run_dist(_rerun, 2, root, model_dir, data, timeout=900).items():
        assert all(res.values()), (rank, res)
