"""Device storage of one engram's row-sharded tables on one rank (CUDA path).

Every rank holds ceil(rows/world) rows of each table (the DTensor Shard(0) split of
micro_engram/rows.py:39-44; the last ranks hold fewer real rows but the same padded
layout), in ONE buffer laid out identically on every rank so a peer's row is at
`ptr[owner] + offset(table) + local_row * row_bytes`:

    per table k:  weight [per_k, dim]  (table dtype)   read by peers' gathers
                  acc    [cap_k, dim]  fp32            compact: peers' row gradients land in slots
                  pos    [per_k] i32                   row -> slot + 1 (0: untouched this step)
                  list   [cap_k] i32                   slot -> row (-1: a slot lost to a race)
                  count  [4] i32                       slots handed out this step

cap_k = capacity: the number of (token, table) lookups one optimizer step can push to a rank
(tokens per step per rank x ranks); every lookup takes at most one slot, so the compact
accumulator cannot overflow, and it replaces a dense fp32 accumulator as large as the table
(2x the bf16 table) with a few hundred MB. Without a capacity (inference, tests) cap_k = per_k.

With world > 1 the buffer is a SymmBuffer (CUDA IPC over NVLink); kernels index it
through device tables of per-rank addresses. With a capacity, the forward fetch is served by
the owners (each owner reads its rows locally and writes them into the requester's receive
buffer: random reads of peer memory are slow, writes into one window are not) and row
gradients return through per-source inbox regions (no remote atomics); see gather and
push_grads. The optimizer moments live in ordinary local
memory (only the owner touches them).
"""
import torch

from .. import native

_ALIGN = 256


def _align(n):
    return (n + _ALIGN - 1) // _ALIGN * _ALIGN


class RowStore:
    _created = 0

    def __init__(self, table_rows, dim, dtype, rank, world, device, group=None, capacity=None):
        RowStore._created += 1
        self.salt = RowStore._created  # decorrelates the rounding bits of different engrams
        self.coef = None  # device clip coefficient for the next optimizer step
        self.table_rows = [int(r) for r in table_rows]
        self.dim = int(dim)
        self.dtype = dtype
        self.rank, self.world = int(rank), int(world)
        self.device = torch.device(device)
        self.nt = len(self.table_rows)
        self.per = [-(-r // self.world) for r in self.table_rows]
        # every lookup event reserves at most one slot (a race loser leaves a hole), so `capacity`
        # events per step always fit; capping at the shard's rows could overflow through holes
        self.cap = [p if capacity is None else max(1, int(capacity)) for p in self.per]
        self.counts = []
        for r, p in zip(self.table_rows, self.per):
            start = min(self.rank * p, r)
            self.counts.append(max(0, min(p, r - start)))
        esz = torch.empty((), dtype=dtype).element_size()
        self.layout = []  # per table: dict of byte offsets
        off = 0
        for p, c in zip(self.per, self.cap):
            ent = {}
            ent["weight"] = off
            off = _align(off + p * self.dim * esz)
            ent["acc"] = off
            off = _align(off + c * self.dim * 4)
            ent["pos"] = off
            off = _align(off + p * 4)
            ent["list"] = off
            off = _align(off + c * 4)
            ent["count"] = off
            off = _align(off + 16)
            self.layout.append(ent)
        self.nbytes = off
        if self.world > 1:
            from .symm import SymmBuffer

            self.buf = SymmBuffer(self.nbytes, self.device, group)
            base_ptrs = self.buf.ptrs

            def view(o, shape, dt):
                return self.buf.view(o, shape, dt)
        else:
            self.buf = None
            self._raw = torch.zeros(self.nbytes, dtype=torch.uint8, device=self.device)
            base_ptrs = [self._raw.data_ptr()]

            def view(o, shape, dt):
                n = 1
                for s in shape:
                    n *= s
                nb = n * torch.empty((), dtype=dt).element_size()
                return self._raw[o:o + nb].view(dt).view(*shape)
        self.weights, self.acc, self.pos, self.list, self.count = [], [], [], [], []
        for k, (p, c, ent) in enumerate(zip(self.per, self.cap, self.layout)):
            self.weights.append(view(ent["weight"], (p, self.dim), dtype))
            self.acc.append(view(ent["acc"], (c, self.dim), torch.float32))
            self.pos.append(view(ent["pos"], (p,), torch.int32))
            self.list.append(view(ent["list"], (c,), torch.int32))
            self.count.append(view(ent["count"], (4,), torch.int32))

        def table(kind):
            return torch.tensor([base_ptrs[r] + self.layout[k][kind] for r in range(self.world)
                                 for k in range(self.nt)], dtype=torch.int64, device=self.device)

        self.w_ptrs = table("weight")
        self.acc_ptrs = table("acc")
        self.pos_ptrs = table("pos")
        self.list_ptrs = table("list")
        self.cnt_ptrs = table("count")
        # this rank's own entries (for the optimizer and the norm)
        own = slice(self.rank * self.nt, (self.rank + 1) * self.nt)
        self.own_acc_ptrs = self.acc_ptrs[own].contiguous()
        self.own_list_ptrs = self.list_ptrs[own].contiguous()
        self.own_cnt_ptrs = self.cnt_ptrs[own].contiguous()
        self.per_t = torch.tensor(self.per, dtype=torch.int64, device=self.device)
        self.cap_t = torch.tensor(self.cap, dtype=torch.int64, device=self.device)
        self.status = torch.zeros(2, dtype=torch.int32, device=self.device)
        self.pending = False  # row gradients were pushed since the last optimizer step
        self._setup_exchange(capacity, group)

    # ---------------------------------------------------------------- multi-GPU gradient return
    def _setup_exchange(self, capacity, group):
        """With world > 1 and a capacity, row gradients return to their owners through inbox
        regions (engram_push_grads / engram_accumulate_grads: plain NVLink stores, owner-side
        local atomics). An inbox region holds what one rank can send one owner in a backward
        call: capacity / world tokens x n_tables events of (table, row) + dim bf16 values."""
        self.x = None
        if self.world == 1 or capacity is None or self.dim % 8:
            return
        import os

        import torch.distributed as dist

        from .symm import SymmBuffer

        self.x_tokens = max(1, int(capacity) // self.world)
        self.cap_e = self.x_tokens * self.nt
        self.x_rows_off = _align(self.cap_e * 8)
        self.x_region = _align(self.x_rows_off + self.cap_e * self.dim * 2)
        self.x = SymmBuffer(512 + self.world * self.x_region, self.device, group)
        self.x.view(0, (128,), torch.int32).zero_()  # flags and counters
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)  # every rank's flags are zero before anyone signals
        self.xbases = torch.tensor(self.x.ptrs, dtype=torch.int64, device=self.device)
        self.x_calls = 0
        self.x_timeout = float(os.environ.get("MICRO_ENGRAM_PEER_TIMEOUT_S", "10"))
        # the owner-served forward fetch: this rank's lookups, then the rows its owners send it
        esz = torch.empty((), dtype=self.dtype).element_size()
        self.f_row_bytes = self.dim * esz
        self.f_recv_off = _align(256 + self.nt * self.x_tokens * 8)
        self.f = SymmBuffer(self.f_recv_off + self.x_tokens * self.nt * self.f_row_bytes, self.device, group)
        self.f.view(0, (64,), torch.int32).zero_()
        self.f_idx = self.f.view(256, (self.nt, self.x_tokens), torch.int64)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)
        self.fbases = torch.tensor(self.f.ptrs, dtype=torch.int64, device=self.device)
        self.f_calls = 0

    # ---------------------------------------------------------------- views
    def shard(self, k):
        """This rank's real rows of table k (a view; the Parameter wraps it)."""
        return self.weights[k][:self.counts[k]]

    def touched(self, k):
        """(local rows, fp32 grads) of table k's touched rows, in slot order: one host sync
        (tests/logging)."""
        n = min(int(self.count[k][0]), self.cap[k])
        rows = self.list[k][:n].long()
        keep = rows >= 0
        return rows[keep], self.acc[k][:n][keep]

    def dense_grad(self, k):
        """Table k's accumulated gradient as a dense fp32 [per_k, dim] tensor (the non-lazy
        optimizer's input; zeros on untouched rows)."""
        rows, g = self.touched(k)
        out = torch.zeros(self.per[k], self.dim, dtype=torch.float32, device=self.device)
        out.index_copy_(0, rows, g)
        return out

    # ---------------------------------------------------------------- kernels
    def gather(self, idx, out_dtype):
        """idx [n_tables, N] global rows -> mem [N, n_tables*dim] from the owners' shards.

        world > 1 with a fetch buffer: the owners serve the rows (engram_fetch; collective, every
        rank calls it in the same order); otherwise one kernel reads them where they live."""
        n = idx.shape[1]
        if getattr(self, "x", None) is not None and n <= self.x_tokens:
            self.f_calls += 1
            self.f_idx[:, :n].copy_(idx)
            rows = torch.empty(n, self.nt * self.dim, dtype=self.dtype, device=self.device)
            args = (self.fbases, self.w_ptrs, self.per_t, self.rank, self.nt, self.f_row_bytes, n, self.x_tokens,
                    self.f_recv_off, self.f_calls, self.x_timeout, self.status)
            native().engram_fetch_serve(*args)
            native().engram_fetch_collect(*args, rows)
            return rows if rows.dtype == out_dtype else rows.to(out_dtype)
        src = 0 if self.dtype == torch.bfloat16 else 1
        return native().engram_gather(idx, self.w_ptrs, self.per_t, self.world, self.dim, src, out_dtype,
                                      self.status)

    def push_grads(self, g, idx, scale):
        """Row gradients g [N, n_tables*dim] of the looked-up rows -> the owners' accumulators.

        world > 1 with an exchange buffer: collective (every rank calls it in the same order);
        otherwise one kernel of atomics into the owners' accumulators."""
        C = native()
        g = g.contiguous()
        if self.x is not None and g.dtype == torch.bfloat16 and idx.shape[1] <= self.x_tokens:
            self.x_calls += 1
            C.engram_push_grads(g, idx, self.acc_ptrs, self.pos_ptrs, self.list_ptrs, self.cnt_ptrs, self.per_t,
                                self.cap_t, self.xbases, self.rank, float(scale), self.cap_e, self.x_region,
                                self.x_rows_off, self.x_calls, self.x_timeout, self.status)
            C.engram_accumulate_grads(self.acc_ptrs, self.pos_ptrs, self.list_ptrs, self.cnt_ptrs, self.per_t,
                                      self.cap_t, self.xbases, self.nt, self.dim, self.rank, float(scale), self.cap_e,
                                      self.x_region, self.x_rows_off, self.x_calls, self.x_timeout, self.status)
        else:
            C.engram_scatter_grad(g, idx, self.acc_ptrs, self.pos_ptrs, self.list_ptrs, self.cnt_ptrs, self.per_t,
                                  self.cap_t, self.world, float(scale), self.status, self.rank)
        self.pending = True

    def sqnorm_into(self, sq):
        native().engram_touched_sqnorm(self.own_acc_ptrs, self.own_cnt_ptrs, self.cap_t, self.dim, sq)

    def clear_counts(self):
        for c in self.count:
            c.zero_()
        self.pending = False

    def zero_grads(self):
        """Drop pending gradients (zero_grad without a step): clears only the used slots and
        their rows' pos entries."""
        for k in range(self.nt):
            n = min(int(self.count[k][0]), self.cap[k])
            if n:
                rows = self.list[k][:n].long()
                self.pos[k].index_fill_(0, rows[rows >= 0], 0)
                self.acc[k][:n].zero_()
        self.clear_counts()

    def check_status(self):
        st = self.status.tolist()
        if st[0] != 0:
            raise RuntimeError(f"[micro_engram] row store kernel error code {st[0]} (detail {st[1]})")

    def close(self):
        if self.buf is not None:
            self.buf.close()
            self.buf = None
        if getattr(self, "x", None) is not None:
            self.x.close()
            self.f.close()
            self.x = None
