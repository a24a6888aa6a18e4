"""Gate modes of MicroEngram on CPU: exact no-op start, gradient flow, parameter names and
checkpoint compatibility, sqrt-gate saturation, gate statistics, keep mask, delta-stored
norm scales, weight stats, and a code guard on reading the delta parameters."""
import pathlib
import re

import pytest
import torch
import torch.nn.functional as F

from micro_engram.module import MicroEngram
from micro_engram.stats import format_stats, module_stats, weight_stats

V, D = 1000, 32


def make(gate, **kw):
    return MicroEngram(model_dim=D, table_size=257, engram_dim=4, num_heads=2, vocab_size=V, gate=gate, **kw)


@pytest.fixture
def data():
    torch.manual_seed(0)
    return torch.randint(5, V, (2, 12)), torch.randn(2, 12, D) * 50


@pytest.mark.parametrize("gate", MicroEngram.GATES)
def test_noop_start_and_grad_flow(gate, data):
    ids, hidden = data
    eng = make(gate)
    assert torch.equal(eng(hidden, ids), hidden)
    h = hidden.clone().requires_grad_(True)
    eng(h, ids).pow(2).sum().backward()
    out_layer = eng.up if gate == "ple" else eng.value
    assert out_layer.weight.grad is not None and out_layer.weight.grad.abs().sum() > 0
    eng.zero_grad()
    with torch.no_grad():
        out_layer.weight.normal_(std=0.02)
    eng(hidden, ids).pow(2).sum().backward()
    assert eng.tables[0].weight.grad.abs().sum() > 0
    assert not torch.equal(eng(hidden, ids), hidden)
    ob = make(gate).to(torch.bfloat16)(hidden.to(torch.bfloat16), ids)
    assert ob.dtype == torch.bfloat16 and ob.shape == hidden.shape


def test_names_and_compat():
    s, p, q = make("scalar"), make("ple"), make("scalar_sqrt")
    assert {"key.weight", "value.weight"} <= set(s.state_dict())
    assert {"down.weight", "up.weight"} <= set(p.state_dict()) and "key.weight" not in p.state_dict()
    assert sum(x.numel() for x in s.parameters()) == sum(x.numel() for x in p.parameters())
    assert not make("scalar").load_state_dict(s.state_dict(), strict=True).missing_keys
    sd = q.state_dict()
    assert torch.equal(q.q_scale, torch.zeros(D)) and q.q_scale.requires_grad
    assert torch.equal(sd["q_scale"], torch.ones(D))
    missing = set(make("scalar_sqrt").load_state_dict(s.state_dict(), strict=False).missing_keys)
    assert missing == {"q_scale", "k_scale"}
    with pytest.raises(ValueError):
        make("bogus")


def _gate_of(eng, h, ids):
    eng.train()
    eng._gate_stats = None
    eng(h, ids)
    return eng.pop_gate_stats()


def test_sqrt_gate_saturates_less_and_stats(data):
    ids, hidden = data
    torch.manual_seed(1)
    sq, sc = make("scalar_sqrt"), make("scalar")
    with torch.no_grad():
        sc.key.weight.copy_(sq.key.weight)
        sc.tables.load_state_dict(sq.tables.state_dict())
        for e in (sq, sc):
            e.value.weight.normal_(std=0.02)
    idx = sq.hash_ids(ids)
    mem = torch.cat([t(i) for t, i in zip(sq.tables, idx)], dim=-1)
    h_al = sq.key(mem).detach() * 30
    g_sq, sat_sq = _gate_of(sq, h_al, ids)
    g_sc, sat_sc = _gate_of(sc, h_al, ids)
    assert g_sc > g_sq > 0.5 and sat_sc >= sat_sq
    sq.eval()
    sq(h_al, ids)
    assert sq.pop_gate_stats() is None
    sq.train()
    sq.zero_grad()
    sq(h_al + torch.randn_like(h_al), ids).pow(2).sum().backward()
    assert sq.q_scale.grad.abs().sum() > 0 and sq.k_scale.grad.abs().sum() > 0


def test_weight_stats():
    big = MicroEngram(model_dim=D, table_size=4096, engram_dim=64, num_heads=2, vocab_size=V, gate="scalar_sqrt")
    st = module_stats(big)
    assert abs(st["engram/table_rms_2g"] - 0.02) < 0.002 and st["engram/rows_learned_3g"] < 0.001
    assert st["engram/out_abs_mean"] == 0 and abs(st["engram/q_scale_mean"] - 1) < 1e-6
    with torch.no_grad():
        big.tables[2].weight[:1024] *= 3
    st2 = module_stats(big)
    assert 0.10 < st2["engram/rows_learned_3g"] < 0.15 and st2["engram/rows_learned_2g"] < 0.001
    assert weight_stats(big.state_dict(), big.orders, 2) == st2
    assert "learned" in format_stats({**st2, "engram/gate_mean": 0.42, "engram/gate_saturated": 0.03})


def test_keep_mask(data):
    ids, hidden = data
    eng = make("ple")
    with torch.no_grad():
        eng.up.weight.normal_(std=0.05)
    idx = eng.hash_ids(ids)
    keep = torch.tensor([[True] * 6 + [False] * 6] * 2)
    masked, full = eng.inject(hidden, idx, keep), eng.inject(hidden, idx)
    assert torch.equal(masked[:, 6:], hidden[:, 6:]) and torch.equal(masked[:, :6], full[:, :6])


def test_delta_scales(data):
    ids, hidden = data
    torch.manual_seed(3)
    old = make("scalar_sqrt").state_dict()
    old["q_scale"] = 1 + 0.3 * torch.rand(D)
    old["k_scale"] = 1 - 0.2 * torch.rand(D)
    old["value.weight"] = torch.randn_like(old["value.weight"]) * 0.05
    new = make("scalar_sqrt")
    new.load_state_dict(old)
    assert torch.allclose(new.q_scale, old["q_scale"] - 1) and torch.allclose(new.k_scale, old["k_scale"] - 1)
    assert torch.allclose(new.state_dict()["q_scale"], old["q_scale"])
    idx = new.hash_ids(ids)
    mem = torch.cat([t(i) for t, i in zip(new.tables, idx)], dim=-1)
    h = F.rms_norm(hidden.float(), (D,), weight=old["q_scale"])
    k = F.rms_norm(new.key(mem).float(), (D,), weight=old["k_scale"])
    s = (h * k).sum(-1, keepdim=True) / D ** 0.5
    want = hidden + torch.sigmoid(s.sign() * s.abs().clamp_min(1e-6).sqrt()) * new.value(mem)
    assert torch.allclose(new.inject(hidden, idx), want, atol=1e-5)
    st = module_stats(new)
    assert abs(st["engram/q_scale_mean"] - float(old["q_scale"].mean())) < 1e-5
    rt = make("scalar_sqrt").to(torch.bfloat16)
    with torch.no_grad():
        rt.q_scale.copy_(torch.linspace(-0.01, 0.01, D))
    saved = rt.state_dict()
    back = make("scalar_sqrt").to(torch.bfloat16)
    back.load_state_dict(saved)
    assert torch.equal(back.q_scale, rt.q_scale) and saved["q_scale"].dtype == torch.float32
    ns = make("scalar_sqrt").to(torch.bfloat16)
    with torch.no_grad():
        ns.q_scale.fill_(0.003)
    qs, ks = ns.norm_scales()
    assert qs.dtype == torch.float32 and abs(float(qs[0]) - 1.003) < 1e-4 and float(ks[0]) == 1.0


def test_bf16_scales_learn(data):
    ids, hidden = data
    bf = make("scalar_sqrt").to(torch.bfloat16)
    with torch.no_grad():
        bf.value.weight.normal_(std=0.05)
    opt = torch.optim.AdamW(bf.parameters(), lr=1e-3, weight_decay=0.0)
    hb = hidden.to(torch.bfloat16)
    for _ in range(50):
        opt.zero_grad()
        bf(hb, ids).float().pow(2).mean().backward()
        opt.step()
    moved = (bf.state_dict()["q_scale"].float() - 1).abs()
    assert (moved > 0).float().mean() > 0.5


def test_code_guard_delta_parameters():
    """Only module.py reads .q_scale/.k_scale (they hold scale - 1)."""
    root = pathlib.Path(__file__).resolve().parent.parent
    bad = []
    for f in root.rglob("*.py"):
        rel = f.relative_to(root).as_posix()
        if rel == "micro_engram/module.py" or rel.startswith(("tests/", "_work/", "baseline/", "build/")):
            continue
        for i, line in enumerate(f.read_text(encoding="utf-8", errors="replace").splitlines(), 1):
            if re.search(r"\.(q|k)_scale\b", line):
                bad.append(f"{rel}:{i}")
    assert not bad, bad
