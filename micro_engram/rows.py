"""Row-sharded engram tables (micro_engram_sharding: rows).

Each rank owns ceil(rows/world) rows of every table (the DTensor Shard(0) split) and the
tables never pass through FSDP. A lookup needs only the rows a batch uses:

  CUDA   the rows sit in a RowStore (parallel/row_store.py) mapped into every peer over
         NVLink; one gather kernel reads each row straight from its owner, and the backward
         pushes row gradients into the owner's fp32 accumulator with peer atomics. No host
         sync, no all_to_all.
  CPU    (gloo; the oracle) unique ids are bucketed by owner and exchanged with
         all_to_all: counts, requested ids, rows; the backward sends the coalesced fp32
         gradients back.

Either way the owner sums every rank's contribution and divides by the world size (FSDP's
averaging), clipping uses the global norm over all tables, and checkpoints are DCP folders
holding the complete engram under its usual names (reshardable to any world size).
Reference: micro_engram/rows.py:1-343.
"""
import os

import torch
import torch.distributed as dist

from .optim import LazyAdamW
from .weights import _local_name, layer_of_key

ROWS_DIR = "micro_engram_rows"
ROWS_OPTIM_DIR = "micro_engram_rows_optim"

_GROUPS = {}


def dist_rank_world():
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def row_range(n_rows, rank, world):
    """(first row, number of rows) owned by `rank`: ceil(n/world) each, the tail to the last."""
    per = -(-n_rows // world)
    start = min(rank * per, n_rows)
    return start, max(0, min(per, n_rows - start))


def _group(world):
    """The row-exchange process group (its own communicator, created on first use)."""
    if world == 1:
        return None
    if "rows" not in _GROUPS:
        _GROUPS["rows"] = dist.new_group(list(range(world)))
    return _GROUPS["rows"]


def _exchange(x, recv_counts, send_counts, group):
    """all_to_all of rows of x: send_counts[r] rows go to rank r; recv_counts[r] come back."""
    if group is None:
        return x
    out = x.new_empty((sum(recv_counts),) + tuple(x.shape[1:]))
    dist.all_to_all_single(out, x.contiguous(), recv_counts, send_counts, group=group)
    return out


def _table_of(flat, bounds):
    """flat global ids (table offset + row) -> (table index, row); bounds = [0, end_0, ...]."""
    t = torch.searchsorted(bounds, flat, right=True) - 1
    return t, flat - bounds[t]


class _RowLookup(torch.autograd.Function):
    """CPU/gloo row exchange: flat ids [M] -> rows [M, dim] fetched from their owners."""

    @staticmethod
    def forward(ctx, flat, info, *shards):
        offsets, pers, rank, world = info
        group = _group(world)
        dev = flat.device
        bounds = torch.tensor(offsets, dtype=torch.long, device=dev)
        per = torch.tensor(pers, dtype=torch.long, device=dev)
        uniq, inv = torch.unique(flat, return_inverse=True)
        tab, row = _table_of(uniq, bounds)
        owner = row // per[tab]
        order = torch.argsort(owner, stable=True)
        send_counts_t = torch.bincount(owner, minlength=world)
        if group is not None:
            recv_counts_t = torch.empty_like(send_counts_t)
            dist.all_to_all_single(recv_counts_t, send_counts_t, group=group)
        else:
            recv_counts_t = send_counts_t
        send_counts, recv_counts = send_counts_t.tolist(), recv_counts_t.tolist()
        wanted = _exchange(uniq[order], recv_counts, send_counts, group)
        w_tab, w_row = _table_of(wanted, bounds)
        w_local = w_row - rank * per[w_tab]
        rows = shards[0].new_empty(wanted.numel(), shards[0].shape[1])
        for k, shard in enumerate(shards):
            sel = (w_tab == k).nonzero().squeeze(1)
            if sel.numel():
                rows[sel] = shard.index_select(0, w_local[sel])
        got = _exchange(rows, send_counts, recv_counts, group)
        by_uniq = torch.empty_like(got)
        by_uniq[order] = got
        ctx.save_for_backward(inv, order, w_tab, w_local)
        ctx.counts = (send_counts, recv_counts)
        ctx.info, ctx.n_uniq = info, uniq.numel()
        ctx.shapes = [(s.shape, s.dtype) for s in shards]
        ctx.shards = shards if any(getattr(s, "_sparse_rows", False) for s in shards) else None
        return by_uniq[inv]

    @staticmethod
    def backward(ctx, grad):
        inv, order, w_tab, w_local = ctx.saved_tensors
        world = ctx.info[3]
        group = _group(world)
        send_counts, recv_counts = ctx.counts
        g_uniq = torch.zeros(ctx.n_uniq, grad.shape[1], dtype=torch.float32, device=grad.device)
        g_uniq.index_add_(0, inv, grad.float())
        g_owned = _exchange(g_uniq[order], recv_counts, send_counts, group)
        grads = []
        for k, (shape, dtype) in enumerate(ctx.shapes):
            if not ctx.needs_input_grad[2 + k]:
                grads.append(None)
                continue
            sel = (w_tab == k).nonzero().squeeze(1)
            if ctx.shards is not None and getattr(ctx.shards[k], "_sparse_rows", False):
                add_sparse_grad(ctx.shards[k], w_local[sel], g_owned[sel].div_(world))
                grads.append(None)
                continue
            g = torch.zeros(shape, dtype=torch.float32, device=grad.device)
            g.index_add_(0, w_local[sel], g_owned[sel])
            grads.append(g.div_(world).to(dtype))
        return (None, None, *grads)


def add_sparse_grad(p, rows, g):
    """Accumulate fp32 row gradients into p.sparse_grad = (unique rows, summed grads)."""
    cur = getattr(p, "sparse_grad", None)
    if cur is not None:
        rows, g = torch.cat([cur[0], rows]), torch.cat([cur[1], g])
    u, inv = torch.unique(rows, return_inverse=True)
    acc = torch.zeros(u.numel(), g.shape[1], dtype=torch.float32, device=g.device)
    acc.index_add_(0, inv, g.float())
    p.sparse_grad = (u, acc)


def row_lookup(engram, idx):
    """Per-table rows [*idx shape, dim] for hashed ids `idx` (one tensor per table)."""
    shards = engram.row_shards
    store = getattr(engram, "row_store", None)
    m = idx[0].numel()
    if store is not None and shards[0].is_cuda:
        from micro_engram_fork_b200.ops.engram import gather_rows

        flat = torch.stack([i.reshape(-1).to(shards[0].device) for i in idx])
        mem = gather_rows(flat, store, shards[0].dtype, shards)
        dim = engram.engram_dim
        return [mem[:, k * dim:(k + 1) * dim].reshape(*idx[0].shape, dim) for k in range(len(shards))]
    rank, world, _starts, pers = engram.row_info
    offsets = [0]
    for rows in engram.table_rows:
        offsets.append(offsets[-1] + rows)
    dev = shards[0].device
    flat = torch.cat([i.reshape(-1).to(dev) + offsets[k] for k, i in enumerate(idx)])
    out = _RowLookup.apply(flat, (offsets, pers, rank, world), *shards)
    return [out[k * m:(k + 1) * m].reshape(*idx[0].shape, -1) for k in range(len(shards))]


# ----------------------------------------------------------------------------- training side
def _dtensor(t, n_rows, world):
    """This rank's rows as a Shard(0) DTensor of the whole table (same storage)."""
    from torch.distributed.device_mesh import DeviceMesh
    from torch.distributed.tensor import DTensor, Shard

    key = ("mesh", t.device.type)
    if key not in _GROUPS:
        group = _group(world) if world > 1 else dist.group.WORLD
        _GROUPS[key] = DeviceMesh.from_group(group, t.device.type)
    shape = (n_rows,) + tuple(t.shape[1:])
    stride = tuple(torch.empty(shape, device="meta").stride())
    return DTensor.from_local(t, _GROUPS[key], [Shard(0)], run_check=False, shape=shape, stride=stride)


class RowTables:
    """The row-sharded tables of every engram of a run: optimizer, clipping, save/load.

    entries: [(prefix, engram)] with prefixes like "model.language_model.layers.0.micro_engram.".
    """

    def __init__(self, entries, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0, lazy=False,
                 rowwise=False, stochastic_rounding=True, sparse_grads=False):
        self.entries = entries
        self.world = dist_rank_world()[1]
        train = [p for _, e in entries for p in e.row_shards if p.requires_grad]
        if sparse_grads and not lazy:
            raise ValueError("sparse row gradients need a lazy optimizer (lazy_adam / rowwise_adam): "
                             "plain AdamW updates every row every step")
        self.sparse = bool(sparse_grads)
        for _, e in entries:
            store = getattr(e, "row_store", None)
            for k, p in enumerate(e.row_shards):
                p._sparse_rows = self.sparse
                if store is not None:
                    p._row_store = (store, k)
        self.optimizer = LazyAdamW([{"params": train, "lazy": lazy, "rowwise": rowwise}], lr=lr, betas=betas,
                                   eps=eps, weight_decay=weight_decay,
                                   stochastic_rounding=stochastic_rounding) if train else None
        self.last_grad_norm = None
        self.converted = 0

    def params(self):
        return [p for _, e in self.entries for p in e.row_shards]

    def stores(self):
        seen = []
        for _, e in self.entries:
            s = getattr(e, "row_store", None)
            if s is not None and any(p.requires_grad for p in e.row_shards) and s not in seen:
                seen.append(s)
        return seen

    def clip(self, max_norm):
        """Global L2 norm of the table gradients (each row lives on one rank), scaled down to
        max_norm when larger. Collective: every rank calls it."""
        ps = [p for p in self.params() if p.requires_grad]
        if not ps:
            return None
        dev = ps[0].device
        sq = torch.zeros(1, dtype=torch.float32, device=dev)
        for store in self.stores():
            if store.pending:
                store.sqnorm_into(sq)
        for p in ps:
            if getattr(p, "_row_store", None) is not None:
                continue
            if p.grad is not None:
                sq += p.grad.float().pow(2).sum()
            sg = getattr(p, "sparse_grad", None)
            if sg is not None:
                sq += sg[1].pow(2).sum()
        if self.world > 1:
            dist.all_reduce(sq, group=_group(self.world))
        if dev.type == "cuda" and self.stores():
            from micro_engram_fork_b200 import native

            coef = torch.empty(1, dtype=torch.float32, device=dev)
            norm = torch.empty(1, dtype=torch.float32, device=dev)
            native().engram_clip_coef(sq, float(max_norm or 0.0), coef, norm)
            for store in self.stores():
                store.coef = coef
        else:
            norm = sq.sqrt()
            coef = (max_norm / (norm + 1e-6)).clamp(max=1.0) if (max_norm and max_norm > 0) else None
        if max_norm and max_norm > 0:
            for p in ps:
                if getattr(p, "_row_store", None) is not None:
                    continue
                if p.grad is not None:
                    p.grad.mul_(coef.to(p.grad.dtype))
                sg = getattr(p, "sparse_grad", None)
                if sg is not None:
                    sg[1].mul_(coef)
        self.last_grad_norm = float(norm)
        return self.last_grad_norm

    def step(self, lr):
        if self.optimizer is None:
            return
        for g in self.optimizer.param_groups:
            g["lr"] = lr
        self.optimizer.step()
        self.zero_grad()

    def zero_grad(self):
        if self.optimizer is not None:
            self.optimizer.zero_grad(set_to_none=True)
        for p in self.params():
            p.sparse_grad = None
        for store in self.stores():
            if store.pending:
                store.zero_grads()
            store.coef = None

    # ------------------------------------------------------------------ checkpoints (collective)
    def _table_items(self, frozen_too=False):
        for prefix, e in self.entries:
            if not frozen_too and not any(p.requires_grad for p in e.row_shards):
                continue
            for k, p in enumerate(e.row_shards):
                yield f"{prefix}tables.{k}.weight", e.table_rows[k], p

    def save(self, folder, optim_folder=None):
        """The complete engram (tables + dense weights + buffers) to `folder` and the tables'
        optimizer state to `optim_folder`, as DCP. Frozen engrams are skipped."""
        import torch.distributed.checkpoint as dcp

        sd = {}
        for prefix, e in self.entries:
            if not any(p.requires_grad for p in e.row_shards):
                continue
            sd.update({prefix + k: v for k, v in e.state_dict().items()})
        for key, rows, p in self._table_items():
            sd[key] = _dtensor(p.detach(), rows, self.world)
        if sd:
            dcp.save(sd, checkpoint_id=folder)
        if optim_folder and self.optimizer is not None:
            osd = {}
            for key, rows, p in self._table_items():
                st = self.optimizer.state.get(p)
                if st:
                    osd[f"{key}.exp_avg"] = _dtensor(st["exp_avg"], rows, self.world)
                    osd[f"{key}.exp_avg_sq"] = _dtensor(st["exp_avg_sq"], rows, self.world)
                    osd[f"{key}.step"] = st["step"].detach().clone().reshape(())
            if osd:
                dcp.save(osd, checkpoint_id=optim_folder)

    def load(self, folder, optim_folder=None):
        """Tables from a DCP folder (micro_engram_rows, or an FSDP checkpoint), resharded to this
        run's world. Returns (tables loaded, whether optimizer state was loaded)."""
        import torch.distributed.checkpoint as dcp

        meta = dcp.FileSystemReader(folder).read_metadata().state_dict_metadata
        by_name = {}
        for key in meta:
            local = _local_name(key)
            if local is not None and local.startswith("tables."):
                by_name[(layer_of_key(key), local)] = key
        want = {}
        for prefix, e in self.entries:
            layer = layer_of_key(prefix + "x")
            for k, p in enumerate(e.row_shards):
                found = by_name.get((layer, f"tables.{k}.weight")) or by_name.get((None, f"tables.{k}.weight"))
                if found is None:
                    raise ValueError(f"[micro_engram] {folder} has no tables.{k}.weight for {prefix.rstrip('.')}")
                saved_rows = meta[found].size[0]
                if saved_rows != e.table_rows[k]:
                    raise ValueError(f"[micro_engram] {folder}: tables.{k}.weight has {saved_rows:,} rows, this "
                                     f"engram's table {k} (order {e._table_orders[k]}) has {e.table_rows[k]:,}: "
                                     f"different table sizes can't resume (start a new run, or keep the sizes)")
                want[found] = (e.table_rows[k], p)
        templ = {key: _dtensor(p.data, rows, self.world) for key, (rows, p) in want.items()}
        dcp.load(templ, checkpoint_id=folder)
        optim_loaded = False
        if optim_folder and self.optimizer is not None and os.path.isdir(optim_folder):
            ometa = dcp.FileSystemReader(optim_folder).read_metadata().state_dict_metadata
            otempl, steps, convert = {}, {}, {}
            group = self.optimizer.param_groups[0]
            for key, rows, p in self._table_items():
                if f"{key}.exp_avg" not in ometa:
                    continue
                st = self.optimizer.state[p]
                if not st:
                    LazyAdamW.init_state(st, p, group, self.optimizer._on_host(p, group))
                otempl[f"{key}.exp_avg"] = _dtensor(st["exp_avg"], rows, self.world)
                saved_dims = len(ometa[f"{key}.exp_avg_sq"].size)
                sq = st["exp_avg_sq"]
                if saved_dims != sq.dim():  # written by the other lazy optimizer
                    sq = torch.zeros(p.shape if saved_dims == p.dim() else p.shape[:1], dtype=torch.float32,
                                     device=p.device)
                    convert[p] = sq
                otempl[f"{key}.exp_avg_sq"] = _dtensor(sq, rows, self.world)
                otempl[f"{key}.step"] = steps[p] = torch.zeros((), dtype=torch.float32)
            if otempl:
                dcp.load(otempl, checkpoint_id=optim_folder)
                for p, s in steps.items():
                    self.optimizer.state[p]["step"] = s
                for p, sq in convert.items():
                    st = self.optimizer.state[p]
                    if sq.dim() > st["exp_avg_sq"].dim():
                        # per value -> per row: v is linear in g^2, so the row mean is exact
                        st["exp_avg_sq"].copy_(sq.flatten(1).mean(dim=1))
                    else:  # per row -> per value
                        st["exp_avg_sq"].copy_(sq.reshape(-1, *([1] * (p.dim() - 1))).expand_as(p))
                self.converted = len(convert)
                optim_loaded = True
        return len(want), optim_loaded
