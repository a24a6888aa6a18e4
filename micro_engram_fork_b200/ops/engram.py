"""Engram ops on the sm_100a kernels: hashing, the row gather from the owners (with the
row-gradient push to the owners' accumulators as its backward), and the fused gate.

Semantics follow micro_engram/module.py:183-265 (hash, gate) and micro_engram/rows.py:76-147
(owner-side averaging of row gradients by the world size).
"""
import torch

from .. import native


# ------------------------------------------------------------------------- hashing
def hash_ids(ids, pos, canon, mults, orders_t, rows_t, pad_id):
    """[n_tables, B, T] int64 hashed rows (ids [B, T], pos [B, T] or None)."""
    if ids.dim() == 1:
        ids = ids[None]
        if pos is not None and pos.dim() == 1:
            pos = pos[None]
    return native().engram_hash(ids, pos, canon, mults, orders_t, rows_t, int(pad_id))


def hash_prev(ids, canon, mults, orders_t, rows_t, pad_id):
    """[n_tables, N] int64 hashed rows from [N, max_order] token histories (-1 = none)."""
    return native().engram_hash_prev(ids, canon, mults, orders_t, rows_t, int(pad_id))


# ------------------------------------------------------------------------- row gather
class GatherRows(torch.autograd.Function):
    """mem [N, n_tables*dim] = the looked-up rows. Backward pushes the row gradients (÷ world,
    as FSDP-style averaging) into the owners' fp32 accumulators in the row store; the shard
    Parameters themselves get no .grad (the optimizer reads the store)."""

    @staticmethod
    def forward(ctx, idx, store, out_dtype, *shards):
        ctx.store = store
        ctx.save_for_backward(idx)
        return store.gather(idx, out_dtype)

    @staticmethod
    def backward(ctx, g):
        (idx,) = ctx.saved_tensors
        store = ctx.store
        if any(ctx.needs_input_grad[3:]):
            store.push_grads(g, idx, 1.0 / store.world)
        return (None, None, None) + (None,) * (len(ctx.needs_input_grad) - 3)


def gather_rows(idx, store, out_dtype, shards):
    return GatherRows.apply(idx, store, out_dtype, *shards)


# ------------------------------------------------------------------------- gate
class Gate(torch.autograd.Function):
    """out = h + bf16(sigmoid(s) * v) for the scalar / scalar_sqrt gates, with
    s = <rms(h)*qs, rms(k)*ks>/sqrt(d) (signed sqrt for scalar_sqrt). qs/ks are the stored
    deltas (scale - 1) or None."""

    @staticmethod
    def forward(ctx, h, k, v, q_delta, k_delta, keep, sqrt_gate, gate_acc):
        qs = (1 + q_delta.float()).contiguous() if q_delta is not None else None
        ks = (1 + k_delta.float()).contiguous() if k_delta is not None else None
        keep_u8 = keep.reshape(-1).to(torch.uint8).contiguous() if keep is not None else None
        hc, kc, vc = h.contiguous(), k.contiguous(), v.contiguous()
        out, stats = native().engram_gate_fwd(hc, kc, vc, qs, ks, keep_u8, bool(sqrt_gate), gate_acc)
        ctx.save_for_backward(hc, kc, vc, qs, ks, keep_u8, stats)
        ctx.sqrt_gate = bool(sqrt_gate)
        ctx.delta_dtypes = (q_delta.dtype if q_delta is not None else None,
                            k_delta.dtype if k_delta is not None else None)
        return out

    @staticmethod
    def backward(ctx, g):
        h, k, v, qs, ks, keep, stats = ctx.saved_tensors
        dh, dk, dv, dqs, dks = native().engram_gate_bwd(g, h, k, v, qs, ks, keep, stats, ctx.sqrt_gate)
        dq = dqs.to(ctx.delta_dtypes[0]) if qs is not None and ctx.needs_input_grad[3] else None
        dkk = dks.to(ctx.delta_dtypes[1]) if ks is not None and ctx.needs_input_grad[4] else None
        return dh, dk, dv, dq, dkk, None, None, None


def gate(h, k, v, q_delta=None, k_delta=None, keep=None, sqrt_gate=False, gate_acc=None):
    return Gate.apply(h, k, v, q_delta, k_delta, keep, sqrt_gate, gate_acc)


# ------------------------------------------------------------------------- optimizer kernels
def adam_touched(p, m, v, acc, pos, lst, cnt, coef, lr, beta1, beta2, eps, wd, bc1, bc2, sr, seed, step,
                 table_id):
    """AdamW on the rows of one table shard that hold a slot of the compact accumulator `acc`
    [cap, dim] (slot -> row in `lst`, row -> slot + 1 in `pos`); clears slots and pos."""
    native().engram_adam_touched(p, m, v, acc, pos, lst, cnt, coef, lr, beta1, beta2, eps, wd, bc1, bc2, sr,
                                 seed, step, table_id)


def adam_dense(p, g, m, v, lr, beta1, beta2, eps, wd, bc1, bc2, gscale=1.0, sr=True, seed=0, step=0):
    native().adam_dense(p, g, m, v, lr, beta1, beta2, eps, wd, bc1, bc2, gscale, sr, seed, step)
