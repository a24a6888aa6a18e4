"""Host-side models of the peer-memory signalling protocols, run on CPU ranks (gloo for the
rendezvous, POSIX shared memory standing in for the peer-mapped buffers).

The CUDA kernels cannot be raced on purpose on a GPU, so their protocols are checked here: each
test replays, step for step, the order of stores, flag releases and bounded waits that the
kernels use, with random delays between the steps, and checks that every reader sees exactly
the data of its own call. The protocols:

  parity     one stage per rank and call parity, one flag word per (rank, peer): write the
             stage, release the call number into every peer's flag word, wait for every peer's,
             read every stage (p2p_allreduce_mean_kernel, p2p_gather_kernel, p2p_sum_slots_kernel:
             the dense all-reduce, the vocab-parallel loss, the TP row-parallel linear)
  inbox      one inbox per (owner, source), a ready flag per source at the owner and a consumed
             flag per owner at the source (row_push_kernel / row_accumulate_kernel)
  fetch      requesters publish their lookups (ready, token count), owners write the rows they
             hold into each requester's receive window and set done (rows_serve_kernel /
             rows_collect_kernel)

A negative control runs the parity protocol with ONE stage instead of two and must see a reader
get the next call's data. A rank that stops signalling must make every other rank's wait run out
and name that rank, within the limit, instead of waiting forever."""
import random
import time

import numpy as np
import pytest

from helpers import run_dist

WORLD, CALLS, N = 3, 6, 512
LIMIT_S = 5.0


class _Sym:
    """Every rank's buffer of `nbytes` in shared memory, mapped by every rank."""

    def __init__(self, nbytes, rank, world):
        import torch.distributed as dist
        from multiprocessing import shared_memory

        self.own = shared_memory.SharedMemory(create=True, size=nbytes)
        np.frombuffer(self.own.buf, dtype=np.uint8)[:] = 0
        names = [None] * world
        dist.all_gather_object(names, self.own.name)
        self.maps = [self.own if r == rank else shared_memory.SharedMemory(name=n) for r, n in enumerate(names)]

    def arr(self, r, off, n, dtype):
        return np.ndarray((n,), dtype=dtype, buffer=self.maps[r].buf, offset=off)

    def close(self, world_barrier):
        for m in self.maps:
            if m is not self.own:
                m.close()
        world_barrier()  # no peer still maps this rank's buffer
        self.own.close()
        self.own.unlink()


def _wait_geq(words, i, value, limit_s):
    """Bounded wait for words[i] >= value (the kernels' wait_flag_geq); False when it ran out."""
    t0 = time.monotonic()
    while int(words[i]) < value:
        if time.monotonic() - t0 > limit_s:
            return False
        time.sleep(0.0002)
    return True


def _jitter(rng, scale=0.002):
    time.sleep(rng.random() * scale)


def _value(rank, call, n):
    return (np.arange(n, dtype=np.int64) * 31 + rank * 1_000_003 + call * 7919)


# ------------------------------------------------------------------ parity (double-buffered stage)
def _parity_checks(rank, world, stages, slow_reader, limit_s, stop_at=None):
    import torch.distributed as dist

    flags_off, stage_off = 0, 64
    sym = _Sym(stage_off + stages * N * 8, rank, world)
    rng = random.Random(17 + rank)
    bad, timeout = [], None
    try:
        for call in range(1, CALLS + 1):
            if stop_at is not None and rank == world - 1 and call == stop_at:
                break  # this rank leaves: it never signals `call`
            par = call % stages
            mine = sym.arr(rank, stage_off + par * N * 8, N, np.int64)
            want = _value(rank, call, N)
            for lo in range(0, N, 128):  # the stage is written in pieces, with delays
                mine[lo:lo + 128] = want[lo:lo + 128]
                _jitter(rng)
            for p in range(world):  # release the call number into every peer's flag word
                sym.arr(p, flags_off, world, np.uint32)[rank] = call
            own_flags = sym.arr(rank, flags_off, world, np.uint32)
            late = [q for q in range(world) if not _wait_geq(own_flags, q, call, limit_s)]
            if late:
                timeout = (call, late)
                break
            for q in range(world):
                stage = sym.arr(q, stage_off + par * N * 8, N, np.int64)
                for lo in range(0, N, 128):
                    if slow_reader and rank == 0:
                        time.sleep(0.02)
                    elif not slow_reader:
                        _jitter(rng)
                    if not np.array_equal(stage[lo:lo + 128], _value(q, call, N)[lo:lo + 128]):
                        bad.append((call, q, lo))
    finally:
        sym.close(lambda: dist.barrier())
    return {"bad": bad, "timeout": timeout}


def test_parity_protocol_has_no_race():
    res = run_dist(_parity_checks, WORLD, 2, False, LIMIT_S)
    for rank, r in res.items():
        assert r["timeout"] is None, f"rank {rank}: {r['timeout']}"
        assert not r["bad"], f"rank {rank} read another call's data: {r['bad'][:5]}"


def test_parity_protocol_with_a_slow_reader():
    """Rank 0 reads slowly: with two stages nobody overwrites what it is still reading."""
    res = run_dist(_parity_checks, WORLD, 2, True, LIMIT_S)
    assert all(not r["bad"] and r["timeout"] is None for r in res.values()), res


def test_one_stage_is_caught():
    """Negative control: one stage per rank lets a fast peer overwrite the stage rank 0 is still
    reading, which this harness must see."""
    res = run_dist(_parity_checks, WORLD, 1, True, LIMIT_S)
    assert res[0]["bad"], "the harness missed the race of a single-buffered stage"


def test_missing_rank_times_out_and_is_named():
    t0 = time.monotonic()
    res = run_dist(_parity_checks, WORLD, 2, False, 0.5, 3)
    for rank in range(WORLD - 1):
        assert res[rank]["timeout"] == (3, [WORLD - 1]), res[rank]
        assert not res[rank]["bad"]
    assert time.monotonic() - t0 < 60


# ------------------------------------------------------------------ inbox (row-gradient exchange)
def _inbox_checks(rank, world, limit_s):
    import torch.distributed as dist

    # layout: ready[16] u32 @0, consumed[16] u32 @64, counts[16] i32 @128, regions @256
    cap = 256
    region = cap * 8
    sym = _Sym(256 + world * region, rank, world)
    rng = random.Random(5 + rank)
    bad, timeout = [], None

    def entries(src, owner, call):
        n = (src * 37 + owner * 11 + call * 13) % cap
        return np.arange(n, dtype=np.int64) * 3 + src * 100_000 + owner * 10_000 + call

    try:
        for call in range(1, CALLS + 1):
            # push: wait until every owner consumed the previous call from this rank's inbox
            consumed = sym.arr(rank, 64, world, np.uint32)
            late = [o for o in range(world) if o != rank and not _wait_geq(consumed, o, call - 1, limit_s)]
            if late:
                timeout = ("push", call, late)
                break
            for o in range(world):
                if o == rank:
                    continue
                e = entries(rank, o, call)
                box = sym.arr(o, 256 + rank * region, cap, np.int64)
                for lo in range(0, len(e), 64):
                    piece = e[lo:lo + 64]
                    box[lo:lo + len(piece)] = piece
                    _jitter(rng)
                sym.arr(o, 128, world, np.int32)[rank] = len(e)
                sym.arr(o, 0, world, np.uint32)[rank] = call  # ready, after the entries and count
            # accumulate: wait for every source, read its inbox, then tell it the inbox is free
            ready = sym.arr(rank, 0, world, np.uint32)
            late = [s for s in range(world) if s != rank and not _wait_geq(ready, s, call, limit_s)]
            if late:
                timeout = ("accumulate", call, late)
                break
            for s in range(world):
                if s == rank:
                    continue
                n = int(sym.arr(rank, 128, world, np.int32)[s])
                _jitter(rng)
                got = np.array(sym.arr(rank, 256 + s * region, cap, np.int64)[:n])
                if not np.array_equal(got, entries(s, rank, call)):
                    bad.append((call, s))
                sym.arr(s, 64, world, np.uint32)[rank] = call  # consumed
    finally:
        sym.close(lambda: dist.barrier())
    return {"bad": bad, "timeout": timeout}


def test_inbox_protocol_has_no_race():
    res = run_dist(_inbox_checks, WORLD, LIMIT_S)
    for rank, r in res.items():
        assert r["timeout"] is None and not r["bad"], (rank, r)


# ------------------------------------------------------------------ owner-served fetch
def _fetch_checks(rank, world, limit_s):
    import torch.distributed as dist

    # layout: ready[16] u32 @0, ntok[16] i32 @64, done[16] u32 @128, idx @256 [cap], recv after
    cap, per = 200, 1000
    idx_off, recv_off = 256, 256 + cap * 8
    sym = _Sym(recv_off + cap * 8, rank, world)
    rng = random.Random(9 + rank)
    bad, timeout = [], None

    def table_row(row):  # the value stored at a global row id, whoever owns it
        return row * 7 + 3

    try:
        for call in range(1, CALLS + 1):
            ntok = 50 + (rank * 29 + call * 17) % (cap - 50)
            ids = np.random.default_rng(call * 10 + rank).integers(0, per * world, ntok)
            sym.arr(rank, idx_off, cap, np.int64)[:ntok] = ids  # this rank's lookups for `call`
            # serve: publish (token count, then ready) at every owner
            for o in range(world):
                sym.arr(o, 64, world, np.int32)[rank] = ntok
                sym.arr(o, 0, world, np.uint32)[rank] = call
            ready = sym.arr(rank, 0, world, np.uint32)
            late = [r for r in range(world) if not _wait_geq(ready, r, call, limit_s)]
            if late:
                timeout = ("serve", call, late)
                break
            for r in range(world):  # the rows this rank owns, into r's receive window
                n = int(sym.arr(rank, 64, world, np.int32)[r])
                want = np.array(sym.arr(r, idx_off, cap, np.int64)[:n])
                recv = sym.arr(r, recv_off, cap, np.int64)
                mine = np.nonzero(want // per == rank)[0]
                for lo in range(0, len(mine), 32):
                    sel = mine[lo:lo + 32]
                    recv[sel] = table_row(want[sel])
                    _jitter(rng)
            for r in range(world):
                sym.arr(r, 128, world, np.uint32)[rank] = call  # done
            # collect: every owner wrote this call's rows, then copy them out
            done = sym.arr(rank, 128, world, np.uint32)
            late = [o for o in range(world) if not _wait_geq(done, o, call, limit_s)]
            if late:
                timeout = ("collect", call, late)
                break
            _jitter(rng)
            got = np.array(sym.arr(rank, recv_off, cap, np.int64)[:ntok])
            if not np.array_equal(got, table_row(ids)):
                bad.append(call)
    finally:
        sym.close(lambda: dist.barrier())
    return {"bad": bad, "timeout": timeout}


def test_fetch_protocol_has_no_race():
    res = run_dist(_fetch_checks, WORLD, LIMIT_S)
    for rank, r in res.items():
        assert r["timeout"] is None and not r["bad"], (rank, r)


if __name__ == "__main__":
    pytest.main([__file__, "-q"])
