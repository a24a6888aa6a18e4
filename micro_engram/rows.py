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
import itertools
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
    pending = getattr(p, "sparse_grad", None)
    all_rows = rows if pending is None else torch.cat([pending[0], rows])
    all_g = g.float() if pending is None else torch.cat([pending[1], g.float()])
    uniq, where = torch.unique(all_rows, return_inverse=True)
    p.sparse_grad = (uniq, all_g.new_zeros(uniq.numel(), all_g.shape[1]).index_add_(0, where, all_g))


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
    # one flat id space over all tables: table k's rows start at the sum of the earlier tables
    offsets = [0, *itertools.accumulate(engram.table_rows)]
    dev = shards[0].device
    flat = torch.cat([ids.reshape(-1).to(dev) + offsets[k] for k, ids in enumerate(idx)])
    rows = _RowLookup.apply(flat, (offsets, pers, rank, world), *shards)
    return [part.reshape(*idx[0].shape, -1) for part in rows.split(m)]


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


class _TableRef:
    """One table shard of one engram: its checkpoint key, full row count and Parameter."""
    __slots__ = ("key", "rows", "param", "engram", "index")

    def __init__(self, key, rows, param, engram, index):
        self.key, self.rows, self.param, self.engram, self.index = key, rows, param, engram, index

    @property
    def trains(self):
        return any(p.requires_grad for p in self.engram.row_shards)


def _grad_sq(p):
    """Squared L2 norm of a table shard's gradient held outside a row store (dense .grad
    and/or the coalesced sparse (rows, grads) pair), as a 1-element fp32 tensor."""
    total = torch.zeros(1, dtype=torch.float32, device=p.device)
    if p.grad is not None:
        total += p.grad.float().square().sum()
    sparse = getattr(p, "sparse_grad", None)
    if sparse is not None:
        total += sparse[1].square().sum()
    return total


def _scale_grad(p, coef):
    if p.grad is not None:
        p.grad.mul_(coef.to(p.grad.dtype))
    sparse = getattr(p, "sparse_grad", None)
    if sparse is not None:
        sparse[1].mul_(coef)


def _convert_second_moment(saved, target, p):
    """Copy a loaded second moment written by the other lazy optimizer into `target`: per value
    -> per row is the row mean (v is linear in g^2, so this is exact for a fresh row); per row ->
    per value repeats the row's value."""
    if saved.dim() > target.dim():
        target.copy_(saved.flatten(1).mean(dim=1))
    else:
        target.copy_(saved.reshape(-1, *([1] * (p.dim() - 1))).expand_as(p))


class RowTables:
    """Every row-sharded table of a run: the optimizer over the shards, global-norm clipping,
    and checkpoints (collective: every rank calls clip / save / load).

    entries: [(prefix, engram)], prefix being the engram's module path plus a dot, e.g.
    "model.language_model.layers.0.micro_engram.".
    """

    def __init__(self, entries, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0, lazy=False,
                 rowwise=False, stochastic_rounding=True, sparse_grads=False):
        if sparse_grads and not lazy:
            raise ValueError("sparse row gradients need a lazy optimizer (lazy_adam or rowwise_adam); plain AdamW "
                             "steps every row every step")
        self.entries = entries
        self.world = dist_rank_world()[1]
        self.sparse = bool(sparse_grads)
        self.refs = [_TableRef(f"{prefix}tables.{k}.weight", e.table_rows[k], p, e, k)
                     for prefix, e in entries for k, p in enumerate(e.row_shards)]
        for ref in self.refs:
            ref.param._sparse_rows = self.sparse
            store = getattr(ref.engram, "row_store", None)
            if store is not None:
                ref.param._row_store = (store, ref.index)
        trained = [r.param for r in self.refs if r.param.requires_grad]
        self.optimizer = None
        if trained:
            self.optimizer = LazyAdamW([{"params": trained, "lazy": lazy, "rowwise": rowwise}], lr=lr, betas=betas,
                                       eps=eps, weight_decay=weight_decay, stochastic_rounding=stochastic_rounding)
        self.last_grad_norm = None
        self.converted = 0

    def params(self):
        return [r.param for r in self.refs]

    def stores(self):
        """The row stores holding gradients of trained tables (each once)."""
        out = []
        for r in self.refs:
            store = getattr(r.engram, "row_store", None)
            if store is not None and r.trains and store not in out:
                out.append(store)
        return out

    # ------------------------------------------------------------------ clipping
    def clip(self, max_norm):
        """Scale every table gradient by min(1, max_norm / global norm) and return the global
        norm (a row lives on exactly one rank, so the squared norms add across ranks). On CUDA
        the coefficient stays on the device and the touched-row update applies it."""
        trained = [p for p in self.params() if p.requires_grad]
        if not trained:
            return None
        dev = trained[0].device
        sq = torch.zeros(1, dtype=torch.float32, device=dev)
        for store in self.stores():
            if store.pending:
                store.sqnorm_into(sq)
        loose = [p for p in trained if getattr(p, "_row_store", None) is None]
        for p in loose:
            sq += _grad_sq(p)
        if self.world > 1:
            dist.all_reduce(sq, group=_group(self.world))
        clipping = bool(max_norm) and max_norm > 0
        if dev.type == "cuda" and self.stores():
            from micro_engram_fork_b200 import native

            coef = torch.empty(1, dtype=torch.float32, device=dev)
            norm = torch.empty(1, dtype=torch.float32, device=dev)
            native().engram_clip_coef(sq, float(max_norm or 0.0), coef, norm)
            for store in self.stores():
                store.coef = coef
        else:
            norm = sq.sqrt()
            coef = torch.clamp(max_norm / (norm + 1e-6), max=1.0) if clipping else None
        if clipping:
            for p in loose:
                _scale_grad(p, coef)
        self.last_grad_norm = norm
        return norm

    def step(self, lr):
        """One table update at learning rate `lr`, then the gradients are dropped."""
        if self.optimizer is not None:
            for group in self.optimizer.param_groups:
                group["lr"] = lr
            self.optimizer.step()
            self.zero_grad()

    def zero_grad(self):
        """Drop every pending table gradient: dense .grad, sparse (rows, grads) and the row
        stores' used slots (a step consumes them already; this covers a skipped step)."""
        if self.optimizer is not None:
            self.optimizer.zero_grad(set_to_none=True)
        for p in self.params():
            p.sparse_grad = None
        for store in self.stores():
            store.coef = None
            if store.pending:
                store.zero_grads()

    # ------------------------------------------------------------------ checkpoints
    def _trained_refs(self):
        return [r for r in self.refs if r.trains]

    def save(self, folder, optim_folder=None):
        """DCP checkpoint of every trained engram: tables (as Shard(0) DTensors of the whole
        table, reshardable to any world size), dense weights and buffers under their module
        names in `folder`; the tables' optimizer moments and step in `optim_folder`."""
        import torch.distributed.checkpoint as dcp

        trained = {id(e) for _, e in self.entries if any(p.requires_grad for p in e.row_shards)}
        state = {}
        for prefix, e in self.entries:
            if id(e) in trained:
                state.update((prefix + k, v) for k, v in e.state_dict().items())
        for r in self._trained_refs():
            state[r.key] = _dtensor(r.param.detach(), r.rows, self.world)
        if state:
            dcp.save(state, checkpoint_id=folder)
        if optim_folder and self.optimizer is not None:
            moments = {}
            for r in self._trained_refs():
                st = self.optimizer.state.get(r.param)
                if not st:
                    continue
                moments[f"{r.key}.exp_avg"] = _dtensor(st["exp_avg"], r.rows, self.world)
                moments[f"{r.key}.exp_avg_sq"] = _dtensor(st["exp_avg_sq"], r.rows, self.world)
                moments[f"{r.key}.step"] = st["step"].detach().clone().reshape(())
            if moments:
                dcp.save(moments, checkpoint_id=optim_folder)

    def _saved_table_keys(self, meta):
        """{(layer or None, 'tables.k.weight'): saved key} of a DCP checkpoint's table tensors."""
        found = {}
        for key in meta:
            local = _local_name(key)
            if local is not None and local.startswith("tables."):
                found[(layer_of_key(key), local)] = key
        return found

    def load(self, folder, optim_folder=None):
        """Load tables from a DCP folder (micro_engram_rows, or an FSDP checkpoint holding the
        engram), resharded to this run's world size; then the optimizer moments when
        `optim_folder` has them (converting between the two lazy optimizers' second-moment
        shapes). Returns (number of tables loaded, whether optimizer state was loaded)."""
        import torch.distributed.checkpoint as dcp

        meta = dcp.FileSystemReader(folder).read_metadata().state_dict_metadata
        saved = self._saved_table_keys(meta)
        targets = {}
        for r in self.refs:
            layer = layer_of_key(r.key)
            local = f"tables.{r.index}.weight"
            key = saved.get((layer, local)) or saved.get((None, local))
            if key is None:
                raise ValueError(f"[micro_engram] {folder} holds no {local} for {r.key.rsplit('.tables.', 1)[0]}")
            if meta[key].size[0] != r.rows:
                raise ValueError(f"[micro_engram] {folder}: {local} was saved with {meta[key].size[0]:,} rows but "
                                 f"table {r.index} (order {r.engram._table_orders[r.index]}) has {r.rows:,}; "
                                 "a run cannot resume with other table sizes")
            targets[key] = _dtensor(r.param.data, r.rows, self.world)
        dcp.load(targets, checkpoint_id=folder)
        loaded_optim = False
        if optim_folder and self.optimizer is not None and os.path.isdir(optim_folder):
            loaded_optim = self._load_moments(optim_folder)
        return len(targets), loaded_optim

    def _load_moments(self, optim_folder):
        import torch.distributed.checkpoint as dcp

        ometa = dcp.FileSystemReader(optim_folder).read_metadata().state_dict_metadata
        group = self.optimizer.param_groups[0]
        targets, steps, foreign = {}, {}, {}
        for r in self._trained_refs():
            if f"{r.key}.exp_avg" not in ometa:
                continue
            p, st = r.param, self.optimizer.state[r.param]
            if not st:
                LazyAdamW.init_state(st, p, group, self.optimizer._on_host(p, group))
            targets[f"{r.key}.exp_avg"] = _dtensor(st["exp_avg"], r.rows, self.world)
            saved_ndim = len(ometa[f"{r.key}.exp_avg_sq"].size)
            v = st["exp_avg_sq"]
            if saved_ndim != v.dim():  # written by the other lazy optimizer: load, then convert
                v = torch.zeros(p.shape if saved_ndim == p.dim() else p.shape[:1], dtype=torch.float32,
                                device=p.device)
                foreign[p] = v
            targets[f"{r.key}.exp_avg_sq"] = _dtensor(v, r.rows, self.world)
            steps[p] = targets[f"{r.key}.step"] = torch.zeros((), dtype=torch.float32)
        if not targets:
            return False
        dcp.load(targets, checkpoint_id=optim_folder)
        for p, step in steps.items():
            self.optimizer.state[p]["step"] = step
        for p, v in foreign.items():
            _convert_second_moment(v, self.optimizer.state[p]["exp_avg_sq"], p)
        self.converted = len(foreign)
        return True
