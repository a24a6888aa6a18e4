"""The three gates of MicroEngram on CPU (scalar, scalar_sqrt, ple).

Checked: an untrained engram is an exact no-op and still passes gradients to its output
projection; once that projection is non-zero the tables get gradients too; parameter names
and checkpoint compatibility between gates; the signed-sqrt gate saturates less than the plain
scalar gate; gate statistics are collected in training mode only; the keep mask; the norm
scales stored as deltas (loaded from and saved as the scale itself); weight statistics; and a
guard that only module.py reads the delta parameters directly."""
import pathlib
import re

import pytest
import torch
import torch.nn.functional as F

from micro_engram.module import MicroEngram
from micro_engram.stats import format_stats, module_stats, weight_stats

VOCAB, DIM = 1000, 32


def engram(gate, **kw):
    return MicroEngram(model_dim=DIM, table_size=257, engram_dim=4, num_heads=2, vocab_size=VOCAB, gate=gate, **kw)


def output_projection(e):
    return e.up if e.gate == "ple" else e.value


def memory(e, ids):
    """The concatenated table rows the engram reads for `ids`."""
    return torch.cat([table(i) for table, i in zip(e.tables, e.hash_ids(ids))], dim=-1)


@pytest.fixture
def batch():
    g = torch.Generator().manual_seed(0)
    return torch.randint(5, VOCAB, (2, 12), generator=g), torch.randn(2, 12, DIM, generator=g) * 50


@pytest.mark.parametrize("gate", MicroEngram.GATES)
def test_untrained_engram_is_a_noop_that_learns(gate, batch):
    ids, hidden = batch
    e = engram(gate)
    assert torch.equal(e(hidden, ids), hidden)
    h = hidden.clone().requires_grad_()
    e(h, ids).square().sum().backward()
    assert output_projection(e).weight.grad.abs().sum() > 0  # the zero projection still learns
    e.zero_grad()
    with torch.no_grad():
        output_projection(e).weight.normal_(std=0.02)
    e(hidden, ids).square().sum().backward()
    assert e.tables[0].weight.grad.abs().sum() > 0
    assert not torch.equal(e(hidden, ids), hidden)
    half = engram(gate).to(torch.bfloat16)(hidden.to(torch.bfloat16), ids)
    assert half.dtype == torch.bfloat16 and half.shape == hidden.shape


def test_parameter_names_across_gates():
    scalar, ple, sqrt = engram("scalar"), engram("ple"), engram("scalar_sqrt")
    assert {"key.weight", "value.weight"} <= set(scalar.state_dict())
    assert {"down.weight", "up.weight"} <= set(ple.state_dict()) and "key.weight" not in ple.state_dict()
    assert sum(p.numel() for p in scalar.parameters()) == sum(p.numel() for p in ple.parameters())
    assert not engram("scalar").load_state_dict(scalar.state_dict(), strict=True).missing_keys
    # scalar_sqrt stores its norm scales as deltas from 1 and saves the scales themselves
    assert torch.equal(sqrt.q_scale, torch.zeros(DIM)) and sqrt.q_scale.requires_grad
    assert torch.equal(sqrt.state_dict()["q_scale"], torch.ones(DIM))
    result = engram("scalar_sqrt").load_state_dict(scalar.state_dict(), strict=False)
    assert set(result.missing_keys) == {"q_scale", "k_scale"}
    with pytest.raises(ValueError):
        engram("no_such_gate")


def _gate_stats(e, hidden, ids):
    e.train()
    e._gate_stats = None
    e(hidden, ids)
    return e.pop_gate_stats()


def test_sqrt_gate_saturates_less(batch):
    ids, hidden = batch
    torch.manual_seed(1)
    sqrt, plain = engram("scalar_sqrt"), engram("scalar")
    with torch.no_grad():
        plain.key.weight.copy_(sqrt.key.weight)
        plain.tables.load_state_dict(sqrt.tables.state_dict())
        for e in (sqrt, plain):
            e.value.weight.normal_(std=0.02)
    aligned = sqrt.key(memory(sqrt, ids)).detach() * 30  # hidden states pointing along the keys
    mean_sqrt, sat_sqrt = _gate_stats(sqrt, aligned, ids)
    mean_plain, sat_plain = _gate_stats(plain, aligned, ids)
    assert mean_plain > mean_sqrt > 0.5 and sat_plain >= sat_sqrt
    sqrt.eval()
    sqrt(aligned, ids)
    assert sqrt.pop_gate_stats() is None  # no statistics outside training mode
    sqrt.train()
    sqrt.zero_grad()
    sqrt(aligned + torch.randn_like(aligned), ids).square().sum().backward()
    assert sqrt.q_scale.grad.abs().sum() > 0 and sqrt.k_scale.grad.abs().sum() > 0


def test_weight_stats_of_tables():
    e = MicroEngram(model_dim=DIM, table_size=4096, engram_dim=64, num_heads=2, vocab_size=VOCAB, gate="scalar_sqrt")
    fresh = module_stats(e)
    assert abs(fresh["engram/table_rms_2g"] - 0.02) < 0.002 and fresh["engram/rows_learned_3g"] < 0.001
    assert fresh["engram/out_abs_mean"] == 0 and abs(fresh["engram/q_scale_mean"] - 1) < 1e-6
    with torch.no_grad():
        e.tables[2].weight[:1024] *= 3  # a quarter of one 3-gram table "learned"
    grown = module_stats(e)
    assert 0.10 < grown["engram/rows_learned_3g"] < 0.15 and grown["engram/rows_learned_2g"] < 0.001
    assert weight_stats(e.state_dict(), e.orders, 2) == grown
    assert "learned" in format_stats({**grown, "engram/gate_mean": 0.42, "engram/gate_saturated": 0.03})


def test_keep_mask_leaves_tokens_untouched(batch):
    ids, hidden = batch
    e = engram("ple")
    with torch.no_grad():
        e.up.weight.normal_(std=0.05)
    idx = e.hash_ids(ids)
    keep = torch.zeros(2, 12, dtype=torch.bool)
    keep[:, :6] = True
    masked, unmasked = e.inject(hidden, idx, keep), e.inject(hidden, idx)
    assert torch.equal(masked[:, 6:], hidden[:, 6:]) and torch.equal(masked[:, :6], unmasked[:, :6])


def test_norm_scales_stored_as_deltas(batch):
    ids, hidden = batch
    torch.manual_seed(3)
    saved = engram("scalar_sqrt").state_dict()
    saved["q_scale"] = 1 + 0.3 * torch.rand(DIM)
    saved["k_scale"] = 1 - 0.2 * torch.rand(DIM)
    saved["value.weight"] = torch.randn_like(saved["value.weight"]) * 0.05
    e = engram("scalar_sqrt")
    e.load_state_dict(saved)
    assert torch.allclose(e.q_scale, saved["q_scale"] - 1) and torch.allclose(e.k_scale, saved["k_scale"] - 1)
    assert torch.allclose(e.state_dict()["q_scale"], saved["q_scale"])
    # the gate computed by hand from the saved scales
    mem = memory(e, ids)
    q = F.rms_norm(hidden.float(), (DIM,), weight=saved["q_scale"])
    k = F.rms_norm(e.key(mem).float(), (DIM,), weight=saved["k_scale"])
    score = (q * k).sum(-1, keepdim=True) / DIM ** 0.5
    gate = torch.sigmoid(torch.sign(score) * score.abs().clamp_min(1e-6).sqrt())
    assert torch.allclose(e.inject(hidden, e.hash_ids(ids)), hidden + gate * e.value(mem), atol=1e-5)
    assert abs(module_stats(e)["engram/q_scale_mean"] - float(saved["q_scale"].mean())) < 1e-5
    # bf16 module: deltas keep full precision in the saved fp32 scale and round-trip exactly
    bf = engram("scalar_sqrt").to(torch.bfloat16)
    with torch.no_grad():
        bf.q_scale.copy_(torch.linspace(-0.01, 0.01, DIM))
    sd = bf.state_dict()
    again = engram("scalar_sqrt").to(torch.bfloat16)
    again.load_state_dict(sd)
    assert torch.equal(again.q_scale, bf.q_scale) and sd["q_scale"].dtype == torch.float32
    small = engram("scalar_sqrt").to(torch.bfloat16)
    with torch.no_grad():
        small.q_scale.fill_(0.003)
    qs, ks = small.norm_scales()
    assert qs.dtype == torch.float32 and abs(float(qs[0]) - 1.003) < 1e-4 and float(ks[0]) == 1.0


def test_bf16_norm_scales_train(batch):
    ids, hidden = batch
    e = engram("scalar_sqrt").to(torch.bfloat16)
    with torch.no_grad():
        e.value.weight.normal_(std=0.05)
    opt = torch.optim.AdamW(e.parameters(), lr=1e-3, weight_decay=0.0)
    for _ in range(50):
        opt.zero_grad()
        e(hidden.to(torch.bfloat16), ids).float().square().mean().backward()
        opt.step()
    moved = (e.state_dict()["q_scale"].float() - 1).abs() > 0
    assert moved.float().mean() > 0.5  # a bf16 scale near 1 would round most updates away


def test_only_module_reads_delta_parameters():
    """.q_scale / .k_scale hold scale - 1; outside module.py code must use norm_scales()."""
    root = pathlib.Path(__file__).resolve().parent.parent
    pattern = re.compile(r"\.(q|k)_scale\b")
    offenders = []
    for path in root.rglob("*.py"):
        rel = path.relative_to(root).as_posix()
        if rel == "micro_engram/module.py" or rel.startswith(("tests/", "_work/", "baseline/", "build/")):
            continue
        text = path.read_text(encoding="utf-8", errors="replace")
        offenders += [f"{rel}:{n}" for n, line in enumerate(text.splitlines(), 1) if pattern.search(line)]
    assert not offenders, offenders
