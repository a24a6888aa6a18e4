"""Several engrams, init_from and frozen, through the trainer on CPU (one gloo process).

Run A trains one engram at layer 1 and saves a checkpoint. Run B loads it FROZEN (init_from run
A's output_dir: the newest complete checkpoint) and adds a new engram at layer 3. Then: the
frozen engram equals run A's and never moves, the new one trains and starts as a no-op, the
run's config lists both (the frozen one pointing at run A's weights), the inference loader
rebuilds both exactly as trained (full sequence and prefill + decode), assemble_engram_model
puts both into one folder, and the
request rules (two engrams in one layer, frozen without init_from, per-order sizes inherited by
extra engrams, orders dropped with 0) hold. Reference counterpart: test_multi.py."""
import json
import os

import pytest
import torch

from helpers import run_dist
from test_train_cpu import V, base_cfg, make_assets


def _trainer(cfg):
    from micro_engram.train.config import load_config
    from micro_engram.train.loop import Trainer

    t = Trainer(load_config(cfg))
    t.build()
    return t


def _run(rank, world, root, model_dir, data):
    res = {}
    a_out = os.path.join(root, "run_a")
    ca = base_cfg(root, model_dir, data, a_out, micro_engram_extra=None, max_steps=3, save_steps=3,
                  micro_engram_canon_path=None, num_epochs=1)
    ta = _trainer(ca)
    ta.train()
    a_state = {n: p.detach().clone() for n, p in ta.slots[0].engram.named_parameters()}
    a_rows = [p.detach().clone() for p in ta.slots[0].engram.row_shards]
    del ta
    b_out = os.path.join(root, "run_b")
    cb = base_cfg(root, model_dir, data, b_out, micro_engram_init_from=a_out, micro_engram_frozen=True,
                  micro_engram_extra=[{"layer": 3}], max_steps=2, save_steps=2, micro_engram_canon_path=None)
    tb = _trainer(cb)
    s_frozen, s_new = tb.slots[0], tb.slots[1]
    res["layers"] = [s.layer for s in tb.slots]
    # (norm scales are stored as 1 + delta and read back as delta: equal up to fp32 rounding)
    res["frozen_equal"] = {n: bool(torch.allclose(p, a_state[n], atol=1e-6, rtol=0))
                           for n, p in s_frozen.engram.named_parameters()}
    res["frozen_equal"]["rows"] = all(torch.equal(p, r) for p, r in zip(s_frozen.engram.row_shards, a_rows))
    loaded = {n: p.detach().clone() for n, p in s_frozen.engram.named_parameters()}
    loaded_rows = [p.detach().clone() for p in s_frozen.engram.row_shards]
    res["new_noop"] = float(s_new.engram.value.weight.detach().abs().sum()) == 0.0
    res["new_seed"] = s_new.engram.seed
    before = {n: p.detach().clone() for n, p in s_new.engram.named_parameters()}
    tb.train()
    res["frozen_still"] = all(torch.equal(p, loaded[n]) for n, p in s_frozen.engram.named_parameters()) and \
        all(torch.equal(p, r) for p, r in zip(s_frozen.engram.row_shards, loaded_rows)) and \
        not any(p.requires_grad for p in s_frozen.engram.parameters())
    res["new_moved"] = any(not torch.equal(p, before[n]) for n, p in s_new.engram.named_parameters())
    # the trained engrams as a server would see them: module state + the (unsharded) rows
    res["engrams"] = {s.layer: ({k: v.detach().float().clone() for k, v in s.engram.state_dict().items()},
                                [p.detach().float().clone() for p in s.engram.row_shards]) for s in tb.slots}
    return res


@pytest.fixture(scope="module")
def multi(tmp_path_factory):
    root = str(tmp_path_factory.mktemp("multi"))
    model_dir, data = make_assets(root)
    res = run_dist(_run, 1, root, model_dir, data, timeout=900)[0]
    return root, model_dir, res


def test_frozen_and_new_engram(multi):
    root, _, res = multi
    assert res["layers"] == [1, 3]
    assert all(res["frozen_equal"].values()), res["frozen_equal"]
    assert res["frozen_still"]
    assert res["new_noop"] and res["new_moved"] and res["new_seed"] == 3 * 10007
    conf_path = os.path.join(root, "run_b", "micro_engram_config.json")
    from micro_engram.weights import engram_specs

    with open(conf_path) as f:
        specs = engram_specs(json.load(f), conf_path)
    assert [s["layer"] for s in specs] == [1, 3]
    assert os.path.realpath(specs[0]["weights"]).startswith(os.path.realpath(os.path.join(root, "run_a")))
    assert os.path.realpath(specs[1]["weights"]).startswith(os.path.realpath(os.path.join(root, "run_b")))


def test_inference_loads_the_trained_engrams(multi):
    """infer_engram's plan (config -> weights, by layer) rebuilds both engrams exactly as trained:
    same tables and parameters, same injection on the same tokens, full sequence and prefill +
    one-token decode steps with the history kept."""
    from micro_engram.module import engram_from_spec
    from micro_engram.tools import infer

    root, model_dir, res = multi
    args = type("A", (), {"model": model_dir, "engram_pt": None,
                          "engram_config": os.path.join(root, "run_b", "micro_engram_config.json"),
                          "layer": None, "table_size": None, "dim": None, "heads": None, "gate": None})()
    plans = infer.plan_engrams(args)
    assert [p[0]["layer"] for p in plans] == [1, 3]
    torch.manual_seed(0)
    ids = torch.randint(0, V, (1, 40))
    h = torch.randn(1, 40, 64) * 3
    for spec, sd in plans:
        served = engram_from_spec(spec, 64, V, 0)
        served.load_state_dict({k: v.float() for k, v in sd.items()})
        trained_sd, rows = res["engrams"][spec["layer"]]
        for k, t in enumerate(served.tables):
            assert torch.allclose(t.weight, rows[k], atol=1e-6)
        trained = engram_from_spec(spec, 64, V, 0)
        trained.load_state_dict({**trained_sd, **{f"tables.{k}.weight": r for k, r in enumerate(rows)}})
        want = trained(h, ids)
        torch.testing.assert_close(served(h, ids), want, atol=1e-5, rtol=0)
        # prefill 25 tokens, then decode one at a time through the runner's history rule
        session = infer.EngramSession.__new__(infer.EngramSession)
        session.history, session.enabled = None, True
        outs = []
        for a, b in [(0, 25)] + [(t, t + 1) for t in range(25, 40)]:
            session._see_inputs(None, (), {"input_ids": ids[:, a:b]})
            outs.append(session.with_memory(served, h[:, a:b]))
        torch.testing.assert_close(torch.cat(outs, 1), want, atol=1e-5, rtol=0)


def test_assemble_writes_both(multi, tmp_path):
    from safetensors import safe_open

    from micro_engram.tools import assemble

    root, model_dir, _ = multi
    out = tmp_path / "assembled"
    assemble.main(["--base", model_dir, "--engram", os.path.join(root, "run_b"), "--out", str(out),
                   "--config", os.path.join(root, "run_b", "micro_engram_config.json")])
    with safe_open(str(out / "micro_engram.safetensors"), "pt") as f:
        keys = list(f.keys())
    assert any(".layers.1.micro_engram.tables.0.weight" in k for k in keys)
    assert any(".layers.3.micro_engram.tables.0.weight" in k for k in keys)


def test_request_rules():
    from micro_engram.runconfig import engram_requests
    from micro_engram.train.config import load_config

    base = {"base_model": "/nonexistent", "datasets": [{"path": "x.jsonl", "type": "completion"}],
            "sequence_len": 32, "output_dir": "/tmp/x", "micro_engram_layer": 1, "micro_engram_table_size": 97,
            "micro_engram_table_sizes": {2: 97, 3: 131, 4: 0}}
    reqs = engram_requests(load_config({**base, "micro_engram_extra": [{"layer": 3}]}))
    sizes = [r.spec.get("table_sizes") for r in reqs]
    assert sizes[0] == sizes[1] and 4 not in (sizes[0] or {}) or not (sizes[0] or {}).get(4)
    with pytest.raises(ValueError):
        engram_requests(load_config({**base, "micro_engram_extra": [{"layer": 1}]}))
    with pytest.raises(ValueError):
        engram_requests(load_config({**base, "micro_engram_frozen": True}))
    from micro_engram.module import resolve_order_sizes

    assert resolve_order_sizes(97, (2, 3, 4), {"2": 101, "3": 0, "4": None}) == {2: 101}
    assert V > 0
