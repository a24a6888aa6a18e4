"""Engram tables split by rows across tensor-parallel GPUs (reference: micro_engram_vllm/tp.py).

Each TP rank keeps rows [start, start + count) of every table (micro_engram.rows.row_range).

Two lookups:
  * the peer-memory path (default on GPUs that can map each other's memory): the rows live in
    a RowStore whose buffers are mapped into every TP rank, so the fused serving op reads each
    row straight from its owner over NVLink; no collective at all. The model layer calls
    `micro_engram_b200::serve_inject` for it (micro_engram_vllm/model.py).
  * `tp_lookup` (host-offloaded rows, or no peer access): the rows this rank owns, zeros for the
    others, then one all-reduce. Every row has one owner, so the sum is exact in any dtype. The
    shapes never depend on the data, so it captures in CUDA graphs.
"""
import torch
import torch.nn.functional as F

from micro_engram.module import check_loaded


def _masked_rows(shard, ids, start):
    """Rows of `ids` that fall in this rank's shard [start, start + len), zeros for the others."""
    n, width = shard.shape
    if n == 0:  # more ranks than rows: this rank owns none of this table
        return shard.new_zeros(*ids.shape, width)
    local = ids.long() - start
    owned = ((local >= 0) & (local < n)).unsqueeze(-1)
    return F.embedding(local.clamp(0, n - 1), shard) * owned.to(shard.dtype)


def tp_lookup(all_reduce):
    """A MicroEngram.row_lookup_fn: masked local lookup, then `all_reduce` (sum over TP)."""

    def lookup(engram, idx):
        _rank, world, starts, _pers = engram.row_info
        tables = engram.__dict__.get("row_views") or engram.row_shards  # UVA views when offloaded
        mem = torch.cat([_masked_rows(t, ids, a) for t, ids, a in zip(tables, idx, starts)], dim=-1)
        if world > 1:  # every row has exactly one owner: the sum is exact in any dtype
            mem = all_reduce(mem)
        return list(mem.split(engram.engram_dim, dim=-1))

    return lookup


def _check_hash_seed(engram, sd, where):
    saved = sd.get("mults")
    if saved is not None and not torch.equal(saved.to(engram.mults.device).long(), engram.mults.long()):
        raise ValueError(f"[micro_engram] {where}: the saved hash multipliers differ from this engram's "
                         f"seed; the seed is wrong for these weights")


def load_rows(engram, sd, where, complete=True):
    """Load an engram state dict (full tables, usual names) into a row-sharded engram.

    Each `tables.k.weight` is sliced to this rank's rows (into the row store when there is
    one); everything else loads as usual (delta scales converted by the module's hook).
    complete=False: `sd` may be part of the engram (weights streamed from a checkpoint), so
    nothing is reported missing. Returns the set of table indices loaded."""
    rest = {k: v for k, v in sd.items() if not k.startswith("tables.")}
    tables = {k: v for k, v in sd.items() if k.startswith("tables.")}
    _rank, _world, starts, _pers = engram.row_info
    known = {f"tables.{k}.weight": k for k in range(len(engram.row_shards))}
    unknown = [name for name in tables if name not in known]
    if unknown:
        raise ValueError(f"[micro_engram] {where}: tables this engram does not have: {unknown[:5]}")
    loaded = set()
    for name, full in tables.items():
        k = known[name]
        shard = engram.row_shards[k]
        want = (engram.table_rows[k], engram.engram_dim)
        if tuple(full.shape) != want:
            raise ValueError(f"[micro_engram] {where}: {name} is {tuple(full.shape)}, this engram needs {want}")
        with torch.no_grad():
            shard.copy_(full[starts[k]:starts[k] + shard.shape[0]])
        loaded.add(k)
    if complete:
        absent = sorted(set(range(len(engram.row_shards))) - loaded)
        if absent:
            raise ValueError(f"[micro_engram] {where}: missing tables {absent}")
        check_loaded(engram, rest, where)
    elif rest:
        _check_hash_seed(engram, rest, where)
        res = engram.load_state_dict(rest, strict=False)
        if res.unexpected_keys:
            raise ValueError(f"[micro_engram] {where}: unexpected engram tensors {res.unexpected_keys[:10]}")
    return loaded


def serve_inject(engram, hidden, hist, keep=None):
    """Fused serving injection over the peer-mapped row store (one custom op per engram)."""
    from micro_engram_fork_b200.ops.registry import serve_inject as _op

    store = engram.row_store
    canon, mults, orders, rows = engram._consts(hidden.device)
    sqrt_gate = engram.gate == "scalar_sqrt"
    qs = ks = None
    if sqrt_gate:
        qs, ks = (s.float().contiguous() for s in engram.norm_scales())
    src = 0 if store.dtype == torch.bfloat16 else 1
    return _op(hidden, hist, canon, mults, orders, rows, int(engram.pad_id), store.w_ptrs, store.per_t, store.world,
               store.dim, src, engram.key.weight, engram.value.weight, qs, ks, keep, sqrt_gate, store.status)


def fused_ok(engram, hidden):
    """True when the fused peer-memory op can serve this engram for `hidden`."""
    return (engram.row_store is not None and engram.row_lookup_fn is None and hidden.is_cuda
            and hidden.dtype == torch.bfloat16 and engram.gate in engram.SCALAR_GATES
            and engram.key.weight.dtype == torch.bfloat16 and engram.value.weight.dtype == torch.bfloat16)
