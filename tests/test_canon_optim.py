"""Token merging (canon map) and LazyAdamW / rowwise Adam / stochastic rounding on CPU.

Oracles: an independently written hash, torch.optim.AdamW, and analytic properties
(untouched rows bit-identical, bias-corrected second moment = 1 under a constant gradient,
unbiased stochastic rounding)."""

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


def train_param(make_opt, grads, init, dtype=torch.float32):
    """A fresh parameter (init, in dtype) stepped once per gradient by make_opt([param])."""
    param = nn.Parameter(init.clone().to(dtype))
    opt = make_opt([param])
    for g in grads:
        opt.zero_grad()
        param.grad = g.clone().to(dtype)
        opt.step()
    return param.detach().float(), opt


def adamw(wd=0.0):
    return lambda ps: torch.optim.AdamW(ps, lr=1e-2, betas=(0.9, 0.999), eps=1e-8, weight_decay=wd, foreach=False)


def lazy_adamw(wd=0.0, **kw):
    return lambda ps: LazyAdamW(ps, lr=1e-2, betas=(0.9, 0.999), eps=1e-8, weight_decay=wd, **kw)


def only_state(opt):
    return next(iter(opt.state.values()))


R, C = 16, 8


@pytest.fixture
def grads():
    """(init [R, C], 5 dense gradients, 5 gradients touching rows 0-3 only, row 0 only in the first)."""
    torch.manual_seed(0)
    init = torch.randn(R, C)
    dense = [torch.randn(R, C) for _ in range(5)]
    sparse = []
    for step in range(5):
        g = torch.randn(R, C)
        g[4:].zero_()
        g[0].mul_(float(step == 0))
        sparse.append(g)
    return init, dense, sparse


def test_lazy_adam_vs_adamw(grads):
    init, dense, sparse = grads
    for wd in (0.0, 0.1):  # lazy on dense gradients is plain AdamW
        assert torch.allclose(train_param(adamw(wd), dense, init)[0],
                              train_param(lazy_adamw(wd, lazy=True), dense, init)[0], atol=1e-6)
    eager_ref = train_param(adamw(), sparse, init)[0]
    assert torch.allclose(eager_ref, train_param(lazy_adamw(lazy=False), sparse, init)[0], atol=1e-6)
    lazy, opt = train_param(lazy_adamw(lazy=True), sparse, init)
    row0_once = train_param(lazy_adamw(lazy=True), sparse[:1], init)[0][0]
    assert torch.equal(lazy[4:], init[4:]), "untouched rows moved"
    assert torch.equal(lazy[0], row0_once), "a row moved on steps where its gradient was zero"
    assert not torch.allclose(eager_ref[0], row0_once), "the eager optimizer should keep moving row 0"
    assert torch.allclose(lazy[1:4], eager_ref[1:4], atol=1e-6)
    st = only_state(opt)
    assert sorted(st) == ["exp_avg", "exp_avg_sq", "step"] and not st["exp_avg"][4:].any()
    low, opt_bf = train_param(lazy_adamw(lazy=True), sparse, init, dtype=torch.bfloat16)
    assert torch.equal(low[4:], init[4:].bfloat16().float()) and only_state(opt_bf)["exp_avg"].dtype == torch.bfloat16


def test_rowwise(grads):
    init, _, sparse = grads
    # gradients with one magnitude per row: the row mean of g^2 equals every element's g^2,
    # so row-wise Adam reduces to AdamW exactly
    scale = torch.rand(R, 1) + 0.5
    uniform = [scale * torch.randn(R, C).sign() * (k + 1) for k in range(5)]
    ref = train_param(adamw(0.1), uniform, init)[0]
    got, opt = train_param(lazy_adamw(0.1, lazy=False, rowwise=True), uniform, init)
    assert torch.allclose(ref, got, atol=1e-6)
    v = only_state(opt)["exp_avg_sq"]
    assert tuple(v.shape) == (R,) and v.dtype == torch.float32
    lazy, opt_l = train_param(lazy_adamw(lazy=True, rowwise=True), sparse, init)
    assert torch.equal(lazy[4:], init[4:]) and not only_state(opt_l)["exp_avg_sq"][4:].any()


def test_bf16_second_moment_freeze(grads):
    """With g = 1 the bias-corrected second moment tends to 1. A bf16 one rounded to nearest
    stalls far below (each 0.001 step is under half an ulp); stochastic rounding and the fp32
    row-wise moment get there."""
    init, _, _ = grads
    steps = 1500
    settings = {"bf16 nearest": dict(stochastic_rounding=False), "bf16 stochastic": {}, "row-wise fp32": dict(rowwise=True)}
    params = {name: nn.Parameter(init.clone().bfloat16()) for name in settings}
    opts = {name: LazyAdamW([params[name]], lr=0.0, **kw) for name, kw in settings.items()}
    for _ in range(steps):
        for name, opt in opts.items():
            params[name].grad = torch.ones_like(params[name])
            opt.step()
    corrected = {name: float(only_state(o)["exp_avg_sq"].float().mean()) / (1 - 0.999 ** steps)
                 for name, o in opts.items()}
    assert corrected["bf16 nearest"] < 0.5, corrected
    assert abs(corrected["bf16 stochastic"] - 1) < 0.02, corrected
    assert abs(corrected["row-wise fp32"] - 1) < 1e-4, corrected


def test_stochastic_rounding():
    target = 1.00149  # between two bf16 values
    for sign in (1, -1):
        x = torch.full((100_000,), sign * target)
        assert abs(float(stochastic_bf16(x).float().mean()) - sign * target) < 2e-5
    assert torch.isinf(stochastic_bf16(torch.tensor([float("inf")]))).all()

    def drift(lr, dtype, sr):
        torch.manual_seed(5)
        w = nn.Parameter(torch.full((2000, 8), 0.03, dtype=dtype))
        opt = LazyAdamW([{"params": [w], "lazy": True, "rowwise": True}], lr=lr, stochastic_rounding=sr)
        for _ in range(300):
            w.grad = torch.ones_like(w)
            opt.step()
        return float((0.03 - w.float()).mean())

    for lr in (2.5e-5, 6.25e-5):  # updates below half a bf16 ulp of 0.03
        exact = drift(lr, torch.float32, True)
        assert abs(drift(lr, torch.bfloat16, False) / exact - 1) > 0.2
        assert abs(drift(lr, torch.bfloat16, True) / exact - 1) < 0.03


def test_fsdp2_lazy_and_state(dist_env):
    """LazyAdamW on FSDP2 DTensor parameters: lazy rows stay put, and the optimizer state survives
    the distributed-checkpoint state-dict round trip."""
    import torch.distributed as dist
    from torch.distributed.checkpoint.state_dict import get_optimizer_state_dict, set_optimizer_state_dict
    from torch.distributed.fsdp import fully_shard

    dist.init_process_group("gloo", rank=0, world_size=1)
    torch.manual_seed(1)
    model = nn.Sequential(nn.Embedding(R, C), nn.Linear(C, C))
    fully_shard(model)
    table = model[0].weight

    def make():
        return LazyAdamW([{"params": [table], "lazy": True}, {"params": list(model[1].parameters())}], lr=1e-2)

    opt = make()
    start = table.full_tensor().clone()
    snapshots = []
    for ids in ([1, 2, 3], [2, 3], [2, 3]):
        opt.zero_grad()
        model(torch.tensor([ids])).square().sum().backward()
        opt.step()
        snapshots.append(table.full_tensor().clone())
    end = snapshots[-1]
    assert not torch.equal(end[2:4], start[2:4])
    assert torch.equal(end[4:], start[4:]) and torch.equal(end[0], start[0])
    assert torch.equal(end[1], snapshots[0][1]), "row 1 moved after its last lookup"
    restored = make()
    set_optimizer_state_dict(model, restored, get_optimizer_state_dict(model, opt))
    a, b = opt.state[table], restored.state[table]
    assert torch.equal(a["exp_avg"].full_tensor(), b["exp_avg"].full_tensor()) and float(b["step"]) == 3
