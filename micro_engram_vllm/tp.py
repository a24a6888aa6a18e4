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


def tp_lookup(all_reduce):
    """A MicroEngram.row_lookup_fn: masked local lookup, then `all_reduce` (sum over TP)."""

    def lookup(engram, idx):
        _rank, world, starts, _pers = engram.row_info
        tables = engram.__dict__.get("row_views") or engram.row_shards  # UVA views when offloaded
        parts = []
        for shard, i, start in zip(tables, idx, starts):
            n = shard.shape[0]
            if n == 0:  # more ranks than rows: this rank owns none of this table
                parts.append(shard.new_zeros(*i.shape, shard.shape[1]))
                continue
            local = i.long() - start
            mine = (local >= 0) & (local < n)
            rows = F.embedding(local.clamp(0, n - 1), shard)
            parts.append(rows * mine.unsqueeze(-1).to(rows.dtype))
        out = torch.cat(parts, dim=-1)
        if world > 1:
            out = all_reduce(out)
        return list(out.split(engram.engram_dim, dim=-1))

    return lookup


def load_rows(engram, sd, where, complete=True):
    """Load an engram state dict (full tables, usual names) into a row-sharded engram.

    Each `tables.k.weight` is sliced to this rank's rows (into the row store when there is
    one); everything else loads as usual (delta scales converted by the module's hook).
    complete=False: `sd` may be part of the engram (weights streamed from a checkpoint), so
    nothing is reported missing. Returns the set of table indices loaded."""
    sd = dict(sd)
    _rank, _world, starts, _pers = engram.row_info
    loaded = set()
    for k, shard in enumerate(engram.row_shards):
        t = sd.pop(f"tables.{k}.weight", None)
        if t is None:
            continue
        want = (engram.table_rows[k], engram.engram_dim)
        if tuple(t.shape) != want:
            raise ValueError(f"[micro_engram] {where}: tables.{k}.weight is {tuple(t.shape)}, this engram "
                             f"needs {want}")
        with torch.no_grad():
            shard.copy_(t[starts[k]:starts[k] + shard.shape[0]])
        loaded.add(k)
    extra = [k for k in sd if k.startswith("tables.")]
    if extra:
        raise ValueError(f"[micro_engram] {where}: tables this engram does not have: {extra[:5]}")
    if complete:
        missing = [k for k in range(len(engram.row_shards)) if k not in loaded]
        if missing:
            raise ValueError(f"[micro_engram] {where}: missing tables {missing}")
        check_loaded(engram, sd, where)
    elif sd:
        if "mults" in sd and not torch.equal(sd["mults"].to(engram.mults.device).long(), engram.mults.long()):
            raise ValueError(f"[micro_engram] {where}: the saved hash multipliers differ from this engram's "
                             f"seed; the seed is wrong for these weights")
        res = engram.load_state_dict(sd, strict=False)
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
