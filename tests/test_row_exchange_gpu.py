"""The row-gradient exchange kernels (engram_push_grads / engram_accumulate_grads) with two
ranks emulated on ONE GPU.

Each emulated rank has its own compact accumulators and exchange buffer; the launch order
push(0), push(1), accumulate(0), accumulate(1) means every flag a kernel waits for was set by a
launch that already finished, so no kernel depends on another running at the same time. The
oracle is a plain PyTorch fp32 scatter-add of every rank's events into the owners' dense
gradients. Two calls in a row check the ready/consumed protocol; a third call in which rank 1
never pushes checks that rank 0's accumulate gives up after its (short) limit and reports a
timeout instead of hanging."""
import pytest
import torch

pytestmark = pytest.mark.gpu

ROWS, DIM, WORLD, N = (1000, 2000, 3001), 64, 2, 700
_XREG = 512


def _align(n):
    return (n + 255) // 256 * 256


SLOTS = 4 * WORLD * N  # every event of every call may take a slot (races leave holes), as in RowStore


class _Rank:
    def __init__(self, dev, cap_tokens):
        self.per = [-(-r // WORLD) for r in ROWS]
        self.acc = [torch.zeros(SLOTS, DIM, device=dev) for _ in self.per]
        self.pos = [torch.zeros(p, dtype=torch.int32, device=dev) for p in self.per]
        self.lst = [torch.full((SLOTS,), -7, dtype=torch.int32, device=dev) for _ in self.per]
        self.cnt = [torch.zeros(4, dtype=torch.int32, device=dev) for _ in self.per]
        self.cap_e = cap_tokens * len(ROWS)
        self.rows_off = _align(self.cap_e * 8)
        self.region = _align(self.rows_off + self.cap_e * DIM * 2)
        self.x = torch.zeros(_XREG + WORLD * self.region, dtype=torch.uint8, device=dev)
        self.status = torch.zeros(2, dtype=torch.int32, device=dev)

    def dense(self, k):
        """This rank's accumulated gradient of table k as [per_k, DIM] (zeros where untouched)."""
        n = int(self.cnt[k][0])
        rows = self.lst[k][:n].long()
        keep = rows >= 0
        out = torch.zeros(self.per[k], DIM, device=self.acc[k].device)
        out[rows[keep]] = self.acc[k][:n][keep]
        return out


def _tables(ranks, dev):
    def table(attr):
        return torch.tensor([t.data_ptr() for r in ranks for t in getattr(r, attr)], dtype=torch.int64, device=dev)

    return (table("acc"), table("pos"), table("lst"), table("cnt"),
            torch.tensor(ranks[0].per, dtype=torch.int64, device=dev),
            torch.full((len(ROWS),), SLOTS, dtype=torch.int64, device=dev),
            torch.tensor([r.x.data_ptr() for r in ranks], dtype=torch.int64, device=dev))


def _inputs(seed, dev):
    g = torch.Generator().manual_seed(seed)
    idx = torch.stack([torch.randint(0, r, (N,), generator=g) for r in ROWS])
    idx[:, :50] = idx[:, :1]  # repeated rows: several events claim the same slot
    grads = torch.randn(N, len(ROWS) * DIM, generator=g).to(torch.bfloat16)
    return idx.to(dev), grads.to(dev)


def _expected(inputs, per, scale):
    out = [[torch.zeros(p, DIM, dtype=torch.float64) for p in per] for _ in range(WORLD)]
    for idx, grads in inputs:
        idx, grads = idx.cpu(), grads.cpu().double()
        for k in range(len(ROWS)):
            owner, local = idx[k] // per[k], idx[k] % per[k]
            for o in range(WORLD):
                sel = owner == o
                out[o][k].index_add_(0, local[sel], grads[sel, k * DIM:(k + 1) * DIM] * scale)
    return out


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_row_exchange_two_emulated_ranks():
    from micro_engram_fork_b200 import native

    C = native()
    dev = torch.device("cuda", 0)
    ranks = [_Rank(dev, N) for _ in range(WORLD)]
    acc_p, pos_p, lst_p, cnt_p, per_t, cap_t, xb = _tables(ranks, dev)
    scale = 1.0 / WORLD
    r0 = ranks[0]
    every = []
    for call in (1, 2):
        inputs = [_inputs(100 * call + r, dev) for r in range(WORLD)]
        every += inputs
        for me, (idx, grads) in enumerate(inputs):
            C.engram_push_grads(grads, idx, acc_p, pos_p, lst_p, cnt_p, per_t, cap_t, xb, me, scale, r0.cap_e,
                                r0.region, r0.rows_off, call, 5.0, ranks[me].status)
        for me in range(WORLD):
            C.engram_accumulate_grads(acc_p, pos_p, lst_p, cnt_p, per_t, cap_t, xb, len(ROWS), DIM, me, scale,
                                      r0.cap_e, r0.region, r0.rows_off, call, 5.0, ranks[me].status)
        torch.cuda.synchronize()
        for r in ranks:
            assert r.status.tolist() == [0, 0]
        want = _expected(every, r0.per, scale)
        for o, r in enumerate(ranks):
            for k in range(len(ROWS)):
                got = r.dense(k).double().cpu()
                err = (got - want[o][k]).abs().max().item()
                assert err <= 1e-5 * want[o][k].abs().max().item() + 1e-6, f"call {call} owner {o} table {k}: {err}"
    # call 3: rank 1 never pushes, so rank 0's accumulate must time out and say so
    idx, grads = _inputs(999, dev)
    C.engram_push_grads(grads, idx, acc_p, pos_p, lst_p, cnt_p, per_t, cap_t, xb, 0, scale, r0.cap_e, r0.region,
                        r0.rows_off, 3, 5.0, r0.status)
    C.engram_accumulate_grads(acc_p, pos_p, lst_p, cnt_p, per_t, cap_t, xb, len(ROWS), DIM, 0, scale, r0.cap_e,
                              r0.region, r0.rows_off, 3, 0.2, r0.status)
    torch.cuda.synchronize()
    assert r0.status.tolist() == [1, 301]  # ME_ERR_TIMEOUT, waiting on rank 1


_F_READY, _F_NTOK, _F_IDX = 0, 64, 256


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_owner_served_fetch_two_emulated_ranks():
    """engram_fetch_serve / engram_fetch_collect with two ranks emulated on one GPU: every owner
    copies the rows it holds into each requester's receive buffer; the oracle is indexing the
    full tables. The ready flags and token counts are published by the test before the launches
    (as each rank's serve kernel does for itself), and the launch order serve(0), serve(1),
    collect(0), collect(1) makes every wait one that an earlier launch satisfied. A third call
    in which rank 1 never serves must end rank 0's collect with a timeout status."""
    from micro_engram_fork_b200 import native

    C = native()
    dev = torch.device("cuda", 0)
    per = [-(-r // WORLD) for r in ROWS]
    g = torch.Generator(device=dev).manual_seed(4)
    full = [torch.randn(r, DIM, device=dev, generator=g).to(torch.bfloat16) for r in ROWS]
    shards = []  # per rank: its tables, padded to `per` rows
    for rk in range(WORLD):
        shards.append([torch.zeros(p, DIM, device=dev, dtype=torch.bfloat16) for p in per])
        for k, t in enumerate(full):
            part = t[rk * per[k]:(rk + 1) * per[k]]
            shards[rk][k][:part.shape[0]] = part
    cap, row_bytes = N, DIM * 2
    recv_off = _align(_F_IDX + len(ROWS) * cap * 8)
    bufs = [torch.zeros(recv_off + cap * len(ROWS) * row_bytes, dtype=torch.uint8, device=dev) for _ in range(WORLD)]
    fb = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=dev)
    wp = torch.tensor([t.data_ptr() for rk in range(WORLD) for t in shards[rk]], dtype=torch.int64, device=dev)
    per_t = torch.tensor(per, dtype=torch.int64, device=dev)
    status = [torch.zeros(2, dtype=torch.int32, device=dev) for _ in range(WORLD)]

    def publish(call, ntoks):
        for o in range(WORLD):
            words = bufs[o][:256].view(torch.int32)
            for r in range(WORLD):
                words[_F_NTOK // 4 + r] = ntoks[r]
                words[_F_READY // 4 + r] = call

    def args(me, n, call, timeout=5.0):
        return (fb, wp, per_t, me, len(ROWS), row_bytes, n, cap, recv_off, call, timeout, status[me])

    for call, ntoks in ((1, (N, N - 123)), (2, (N - 7, N))):
        idxs = []
        for me in range(WORLD):
            gi = torch.Generator().manual_seed(10 * call + me)
            idx = torch.stack([torch.randint(0, r, (ntoks[me],), generator=gi) for r in ROWS]).to(dev)
            bufs[me][_F_IDX:_F_IDX + len(ROWS) * cap * 8].view(torch.int64).view(len(ROWS), cap)[:, :ntoks[me]] = idx
            idxs.append(idx)
        publish(call, ntoks)
        outs = [torch.full((ntoks[me], len(ROWS) * DIM), float("nan"), device=dev, dtype=torch.bfloat16)
                for me in range(WORLD)]
        for me in range(WORLD):
            C.engram_fetch_serve(*args(me, ntoks[me], call))
        for me in range(WORLD):
            C.engram_fetch_collect(*args(me, ntoks[me], call), outs[me])
        torch.cuda.synchronize()
        for me in range(WORLD):
            assert status[me].tolist() == [0, 0]
            want = torch.cat([full[k][idxs[me][k]] for k in range(len(ROWS))], dim=1)
            assert torch.equal(outs[me], want), f"call {call} rank {me}"
    # call 3: rank 1 never serves its rows, so rank 0's collect must time out and say so
    publish(3, (N, N))
    out = torch.empty(N, len(ROWS) * DIM, device=dev, dtype=torch.bfloat16)
    C.engram_fetch_serve(*args(0, N, 3))
    C.engram_fetch_collect(*args(0, N, 3, timeout=0.2), out)
    torch.cuda.synchronize()
    assert status[0].tolist() == [1, 501]  # ME_ERR_TIMEOUT, waiting on rank 1's rows
