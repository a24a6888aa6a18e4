"""Token merging (canon map) and LazyAdamW / rowwise Adam / stochastic rounding on CPU.

Oracles: an independently written hash, torch.optim.AdamW, and analytic properties
(untouched rows bit-identical, bias-corrected second moment = 1 under a constant gradient,
unbiased stochastic rounding)."""
import os

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from micro_engram.module import _PRIME, MicroEngram, check_loaded
from micro_engram.optim import LazyAdamW, stochastic_bf16

V = 1000


def make(canon=None):
    return MicroEngram(model_dim=16, table_size=257, engram_dim=4, num_heads=2, vocab_size=V, canon=canon)


def independent_hash(eng, ids):
    ids = ids.long()
    T = ids.shape[-1]
    n_max = max(eng.orders)
    padded = F.pad(ids, (n_max - 1, 0), value=eng.pad_id)
    out = []
    for k, n in enumerate(eng._table_orders):
        x = torch.zeros_like(ids)
        for i in range(n):
            x = x + padded[:, n_max - 1 - i: n_max - 1 - i + T] * eng.mults[k, i]
        out.append((x % _PRIME) % eng.table_rows[k])
    return out


def same(a, b):
    return all(torch.equal(x, y) for x, y in zip(a, b))


def test_canon_hashing_and_state():
    torch.manual_seed(0)
    ids = torch.randint(5, V, (3, 20))
    eng = make()
    assert same(eng.hash_ids(ids), independent_hash(eng, ids))
    canon = torch.arange(V)
    canon[11], canon[501] = 10, 500
    eng = make(canon)
    a = torch.tensor([[3, 10, 7, 500, 9, 10, 4]])
    b = torch.tensor([[3, 11, 7, 501, 9, 11, 4]])
    c = torch.tensor([[3, 12, 7, 500, 9, 10, 4]])
    assert same(eng.hash_ids(a), eng.hash_ids(b))
    assert not same(eng.hash_ids(a), eng.hash_ids(c))
    assert "canon" in eng.state_dict()
    old = {k: v for k, v in make().state_dict().items() if k != "canon"}
    res = make().load_state_dict(old, strict=False)
    assert list(res.missing_keys) == ["canon"] and not res.unexpected_keys
    e2 = make()
    e2.load_state_dict(eng.state_dict())
    assert torch.equal(e2.canon, canon)


def test_mults_seed_and_check_loaded():
    a, b = make(), make()
    assert torch.equal(a.mults, b.mults) and (a.mults % 2 == 1).all()
    sd = a.state_dict()
    sd["mults"] = sd["mults"] + 2
    with pytest.raises(ValueError, match="seed does not belong"):
        check_loaded(make(), sd, "x")


def test_position_ids_stop_ngrams():
    eng = make()
    ids = torch.tensor([[5, 6, 7, 8, 9, 10]])
    pos = torch.tensor([[0, 1, 2, 0, 1, 2]])
    h_split = eng.hash_ids(ids, pos)
    h_doc2 = eng.hash_ids(ids[:, 3:])
    assert same([h[:, 3:] for h in h_split], h_doc2)


def _run(opt_cls, grads, init, lazy=True, wd=0.0, dtype=torch.float32, **kw):
    p = nn.Parameter(init.clone().to(dtype))
    if opt_cls is LazyAdamW:
        kw["lazy"] = lazy
    kw.setdefault("lr", 1e-2)
    opt = opt_cls([p], betas=(0.9, 0.999), eps=1e-8, weight_decay=wd, **kw)
    for g in grads:
        opt.zero_grad()
        p.grad = g.clone().to(dtype)
        opt.step()
    return p.detach().float(), opt


R, C = 16, 8


@pytest.fixture
def grads():
    torch.manual_seed(0)
    init = torch.randn(R, C)
    dense = [torch.randn(R, C) for _ in range(5)]
    sparse = []
    for i in range(5):
        g = torch.randn(R, C)
        g[4:] = 0
        if i > 0:
            g[0] = 0
        sparse.append(g)
    return init, dense, sparse


def test_lazy_adam_vs_adamw(grads):
    init, dense, sparse = grads
    for wd in (0.0, 0.1):
        a, _ = _run(torch.optim.AdamW, dense, init, wd=wd, foreach=False)
        b, _ = _run(LazyAdamW, dense, init, wd=wd, lazy=True)
        assert torch.allclose(a, b, atol=1e-6)
    a, _ = _run(torch.optim.AdamW, sparse, init, foreach=False)
    b, _ = _run(LazyAdamW, sparse, init, lazy=False)
    assert torch.allclose(a, b, atol=1e-6)
    c, opt = _run(LazyAdamW, sparse, init, lazy=True)
    after1, _ = _run(LazyAdamW, sparse[:1], init, lazy=True)
    assert torch.equal(c[4:], init[4:])
    assert torch.equal(c[0], after1[0]) and not torch.allclose(a[0], after1[0])
    assert torch.allclose(c[1:4], a[1:4], atol=1e-6)
    st = opt.state[opt.param_groups[0]["params"][0]]
    assert set(st) == {"step", "exp_avg", "exp_avg_sq"}
    assert torch.equal(st["exp_avg"][4:], torch.zeros(R - 4, C))
    d, optb = _run(LazyAdamW, sparse, init, lazy=True, dtype=torch.bfloat16)
    stb = optb.state[optb.param_groups[0]["params"][0]]
    assert torch.equal(d[4:], init[4:].bfloat16().float()) and stb["exp_avg"].dtype == torch.bfloat16


def test_rowwise(grads):
    init, _, sparse = grads
    row_scale = torch.rand(R, 1) + 0.5
    uniform = [row_scale * torch.sign(torch.randn(R, C)) * (i + 1) for i in range(5)]
    a, _ = _run(torch.optim.AdamW, uniform, init, wd=0.1, foreach=False)
    b, opt = _run(LazyAdamW, uniform, init, wd=0.1, lazy=False, rowwise=True)
    assert torch.allclose(a, b, atol=1e-6)
    st = opt.state[opt.param_groups[0]["params"][0]]
    assert st["exp_avg_sq"].shape == (R,) and st["exp_avg_sq"].dtype == torch.float32
    c, optl = _run(LazyAdamW, sparse, init, lazy=True, rowwise=True)
    stl = optl.state[optl.param_groups[0]["params"][0]]
    assert torch.equal(c[4:], init[4:]) and torch.equal(stl["exp_avg_sq"][4:], torch.zeros(R - 4))


def test_bf16_second_moment_freeze(grads):
    init, _, _ = grads
    pb, ps, pr = (nn.Parameter(init.clone().bfloat16()) for _ in range(3))
    ob = LazyAdamW([pb], lr=0.0, stochastic_rounding=False)
    osr = LazyAdamW([ps], lr=0.0)
    orw = LazyAdamW([pr], lr=0.0, rowwise=True)
    for _ in range(1500):
        for p_, o_ in ((pb, ob), (ps, osr), (pr, orw)):
            p_.grad = torch.ones_like(p_)
            o_.step()
    bc2 = 1 - 0.999 ** 1500
    v_bf = float(ob.state[pb]["exp_avg_sq"].float().mean()) / bc2
    v_sr = float(osr.state[ps]["exp_avg_sq"].float().mean()) / bc2
    v_rw = float(orw.state[pr]["exp_avg_sq"].mean()) / bc2
    assert v_bf < 0.5 and abs(v_sr - 1) < 0.02 and abs(v_rw - 1) < 1e-4


def test_stochastic_rounding():
    x = torch.full((100_000,), 1.00149)
    assert abs(float(stochastic_bf16(x).float().mean()) - 1.00149) < 2e-5
    assert abs(float(stochastic_bf16(-x).float().mean()) + 1.00149) < 2e-5
    assert torch.isinf(stochastic_bf16(torch.tensor([float("inf")]))).all()
    for lr in (2.5e-5, 6.25e-5):
        moved = {}
        for name, dtype, sr in (("fp32", torch.float32, True), ("plain", torch.bfloat16, False),
                                ("sr", torch.bfloat16, True)):
            torch.manual_seed(5)
            w = nn.Parameter(torch.full((2000, 8), 0.03, dtype=dtype))
            opt = LazyAdamW([{"params": [w], "lazy": True, "rowwise": True}], lr=lr, stochastic_rounding=sr)
            for _ in range(300):
                w.grad = torch.ones_like(w)
                opt.step()
            moved[name] = float((0.03 - w.float()).mean())
        assert abs(moved["plain"] / moved["fp32"] - 1) > 0.2
        assert abs(moved["sr"] / moved["fp32"] - 1) < 0.03


def test_fsdp2_lazy_and_state(dist_env):
    import torch.distributed as dist
    from torch.distributed.checkpoint.state_dict import get_optimizer_state_dict, set_optimizer_state_dict
    from torch.distributed.fsdp import fully_shard

    dist.init_process_group("gloo", rank=0, world_size=1)

    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.lin = nn.Linear(C, C)
            self.tables = nn.Embedding(R, C)

        def forward(self, ids):
            return self.lin(self.tables(ids))

    torch.manual_seed(1)
    blk = Block()
    fully_shard(blk)
    groups = [{"params": [blk.tables.weight], "lazy": True}, {"params": [blk.lin.weight, blk.lin.bias]}]
    opt = LazyAdamW(groups, lr=1e-2)
    before = blk.tables.weight.full_tensor().clone()
    row1 = None
    for i in range(3):
        opt.zero_grad()
        ids = [[1, 2, 3]] if i == 0 else [[2, 3]]
        blk(torch.tensor(ids)).pow(2).sum().backward()
        opt.step()
        if i == 0:
            row1 = blk.tables.weight.full_tensor()[1].clone()
    w = blk.tables.weight.full_tensor()
    assert not torch.equal(w[2:4], before[2:4]) and torch.equal(w[4:], before[4:]) and torch.equal(w[0], before[0])
    assert torch.equal(w[1], row1)
    sd = get_optimizer_state_dict(blk, opt)
    opt2 = LazyAdamW([{"params": [blk.tables.weight], "lazy": True}, {"params": [blk.lin.weight, blk.lin.bias]}],
                     lr=1e-2)
    set_optimizer_state_dict(blk, opt2, sd)
    s1, s2 = opt.state[blk.tables.weight], opt2.state[blk.tables.weight]
    assert torch.equal(s1["exp_avg"].full_tensor(), s2["exp_avg"].full_tensor()) and float(s2["step"]) == 3
