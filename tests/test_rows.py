"""Row-sharded tables against the full-table engram on real gloo processes (CPU).

World 3 with a 31-row table gives an uneven split (11/11/9). The oracle is the unsharded
engram with FSDP-style averaged gradients; checkpoints are saved on 3 ranks and loaded on 2.
"""
import copy
import os
import tempfile

import pytest
import torch
import torch.distributed as dist

from helpers import run_dist

W, N, D, E = 3, 31, 16, 4
PREFIX = "model.layers.3.micro_engram."


def _make_full(table_sizes=None, seed=0):
    from micro_engram.module import MicroEngram

    torch.manual_seed(seed)
    eng = MicroEngram(model_dim=D, table_size=N, engram_dim=E, num_heads=2, vocab_size=50, gate="scalar_sqrt",
                      table_sizes=table_sizes)
    with torch.no_grad():
        eng.value.weight.normal_(std=0.3)
        eng.q_scale.fill_(0.25)
    return eng


def _batch(rank, step=0):
    g = torch.Generator().manual_seed(100 + 10 * rank + step)
    ids = torch.randint(5, 50, (2, 9), generator=g)
    ids[0, :3] = 7
    return torch.randn(2, 9, D, generator=g) * 5, ids


def _avg_grads(full, world):
    out = []
    for t in full.tables:
        g = t.weight.grad.clone()
        dist.all_reduce(g)
        out.append(g / world)
    return out


def _fwd_bwd_worker(rank, world):
    from micro_engram.rows import RowTables, row_range

    start, count = row_range(N, rank, world)
    full = _make_full()
    sh = copy.deepcopy(full)
    sh.shard_rows(rank, world)
    assert count == (9 if rank == 2 else 11) and "tables" not in sh._modules
    assert not any(k.startswith("tables.") for k in sh.state_dict()) and len(sh.row_shards) == 4
    h, ids = _batch(rank)
    out_f, out_s = full(h, ids), sh(h, ids)
    assert torch.equal(out_f, out_s)
    out_f.pow(2).sum().backward()
    out_s.pow(2).sum().backward()
    want = _avg_grads(full, world)
    for p, w in zip(sh.row_shards, want):
        torch.testing.assert_close(p.grad, w[start:start + count], atol=1e-6, rtol=1e-5)
    torch.testing.assert_close(full.key.weight.grad, sh.key.weight.grad, atol=1e-6, rtol=1e-5)
    # sparse touched-row gradients (lazy optimizers): the same values, only the touched rows
    sp = copy.deepcopy(full)
    sp.zero_grad()
    sp.shard_rows(rank, world)
    RowTables([(PREFIX, sp)], lazy=True, rowwise=True, sparse_grads=True)
    sp(h, ids).pow(2).sum().backward()
    for p, w in zip(sp.row_shards, want):
        assert p.grad is None
        rows, g = p.sparse_grad
        dense = torch.zeros_like(w[start:start + count])
        dense[rows] = g
        torch.testing.assert_close(dense, w[start:start + count], atol=1e-6, rtol=1e-5)
    # clipping uses the global norm over every rank's rows
    rt = RowTables([(PREFIX, sh)])
    full_norm = float(torch.sqrt(sum(w.pow(2).sum() for w in want)))
    norm = rt.clip(0)
    assert abs(norm - full_norm) < 1e-4 * max(1.0, full_norm)
    rt.clip(full_norm / 2)
    clipped = float(torch.sqrt(sum(p.grad.pow(2).sum() for p in sh.row_shards)))
    tot = torch.tensor(clipped ** 2)
    dist.all_reduce(tot)
    assert abs(float(tot.sqrt()) - full_norm / 2) < 1e-3 * full_norm
    return True


def test_sharded_forward_backward_clip():
    run_dist(_fwd_bwd_worker, W)


def _mixed_worker(rank, world):
    from micro_engram.rows import row_range

    fm = _make_full({2: 31, 3: 47, 4: 13}, seed=3)
    sm = copy.deepcopy(fm)
    sm.shard_rows(rank, world)
    h, ids = _batch(rank)
    of, os_ = fm(h, ids), sm(h, ids)
    assert torch.equal(of, os_)
    of.pow(2).sum().backward()
    os_.pow(2).sum().backward()
    want = _avg_grads(fm, world)
    for p, w, a in zip(sm.row_shards, want, sm.row_info[2]):
        torch.testing.assert_close(p.grad, w[a:a + p.shape[0]], atol=1e-6, rtol=1e-5)
    assert [p.shape[0] for p in sm.row_shards] == [row_range(r, rank, world)[1] for r in fm.table_rows]
    # activation checkpointing re-runs the exchange inside the backward
    from torch.utils.checkpoint import checkpoint

    sc = copy.deepcopy(fm)
    sc.zero_grad()
    sc.shard_rows(rank, world)
    checkpoint(lambda x: sc(x, ids), h, use_reentrant=False).pow(2).sum().backward()
    for p, q in zip(sc.row_shards, sm.row_shards):
        torch.testing.assert_close(p.grad, q.grad, atol=1e-6, rtol=1e-5)
    return True


def test_mixed_sizes_and_checkpointing():
    run_dist(_mixed_worker, W)


def _train_worker(rank, world, opt_kind):
    from micro_engram.optim import LazyAdamW
    from micro_engram.rows import RowTables, row_range

    full = _make_full()
    sh = copy.deepcopy(full)
    sh.shard_rows(rank, world)
    lazy = opt_kind in ("lazy", "rowwise")
    rowwise = opt_kind == "rowwise"
    rt = RowTables([(PREFIX, sh)], lr=1e-2, lazy=lazy, rowwise=rowwise, sparse_grads=lazy)
    opt_full = LazyAdamW([{"params": [t.weight for t in full.tables], "lazy": lazy, "rowwise": rowwise}], lr=1e-2)
    for step in range(3):
        h, ids = _batch(rank, step)
        full.zero_grad()
        full(h, ids).pow(2).sum().backward()
        for t in full.tables:
            dist.all_reduce(t.weight.grad)
            t.weight.grad /= world
        opt_full.step()
        sh(h, ids).pow(2).sum().backward()
        rt.step(1e-2)
        for p in [sh.key.weight, sh.value.weight, sh.q_scale, sh.k_scale]:
            p.grad = None
    start, count = row_range(N, rank, world)
    for p, t in zip(sh.row_shards, full.tables):
        torch.testing.assert_close(p.detach(), t.weight.detach()[start:start + count], atol=1e-6, rtol=1e-5)
    return True


@pytest.mark.parametrize("opt_kind", ["adamw", "lazy", "rowwise"])
def test_three_steps_match_full(opt_kind):
    run_dist(_train_worker, W, opt_kind)


def _save_worker(rank, world, folder):
    from micro_engram.rows import ROWS_DIR, ROWS_OPTIM_DIR, RowTables

    full = _make_full()
    sh = copy.deepcopy(full)
    sh.shard_rows(rank, world)
    rt = RowTables([(PREFIX, sh)], lr=1e-2, lazy=True, rowwise=True, sparse_grads=True)
    h, ids = _batch(rank)
    sh(h, ids).pow(2).sum().backward()
    rt.step(1e-2)
    rt.save(os.path.join(folder, ROWS_DIR), os.path.join(folder, ROWS_OPTIM_DIR))
    dist.barrier()
    return [p.detach().clone() for p in sh.row_shards]


def _load_worker(rank, world, folder, as_lazy):
    from micro_engram.module import MicroEngram
    from micro_engram.rows import ROWS_DIR, ROWS_OPTIM_DIR, RowTables, row_range

    e = MicroEngram(model_dim=D, table_size=N, engram_dim=E, num_heads=2, vocab_size=50, gate="scalar_sqrt",
                    build_tables=False)
    e.shard_rows(rank, world)
    rt = RowTables([(PREFIX, e)], lr=1e-2, lazy=True, rowwise=not as_lazy, sparse_grads=True)
    n, opt_loaded = rt.load(os.path.join(folder, ROWS_DIR), os.path.join(folder, ROWS_OPTIM_DIR))
    st = rt.optimizer.state[e.row_shards[0]]
    return n, opt_loaded, [p.detach().clone() for p in e.row_shards], row_range(N, rank, world), \
        st["exp_avg_sq"].clone(), rt.converted


def test_save_on_3_load_on_2_and_convert():
    from micro_engram.rows import ROWS_DIR
    from micro_engram.weights import load_engram_weights

    folder = tempfile.mkdtemp()
    saved = run_dist(_save_worker, 3, folder)
    full_tables = [torch.cat([saved[r][k] for r in range(3)]) for k in range(4)]
    sd = load_engram_weights(os.path.join(folder, ROWS_DIR), layer=3)
    for k in range(4):
        assert torch.equal(sd[f"tables.{k}.weight"], full_tables[k])
    assert "key.weight" in sd and "q_scale" in sd and "mults" in sd
    for as_lazy in (False, True):
        loaded = run_dist(_load_worker, 2, folder, as_lazy)
        for r, (n, opt_loaded, shards, (a, c), sq, converted) in loaded.items():
            assert n == 4 and opt_loaded
            for k in range(4):
                assert torch.equal(shards[k], full_tables[k][a:a + c])
            if as_lazy:  # rowwise -> per-value second moment: every value gets its row's v
                assert converted == 4 and sq.shape == (c, E)
            else:
                assert converted == 0 and sq.shape == (c,)
