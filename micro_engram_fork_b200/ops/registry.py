"""Dispatcher-visible custom ops over the sm_100a kernels (torch.library, namespace
`micro_engram_b200`).

Registering a kernel entry point as a custom op makes it one opaque node for
`torch.compile` (vLLM compiles its model forward; an unregistered pybind call would break
the graph there) and gives it a fake (meta) implementation for shape propagation.
Registration failure on an unusual torch build falls back to the plain callable, with one
warning, so the kernel keeps working outside compiled graphs. Reference counterpart:
micro_engram/train/vendor/op_registry.py:40-67 (the same decorator contract).

Ops registered here are the serving path's: the history fill, the n-gram hash, the fused
row-parallel linear of tensor-parallel serving (GEMM -> reduce-scatter -> all-gather), and the
whole engram injection (hash -> row gather -> key/value projections -> gate -> residual),
which runs as one op so a compiled decoder layer sees a single node per engram.
"""
from __future__ import annotations

import logging
from typing import Callable, Optional, Sequence

import torch

from .. import native

LOG = logging.getLogger(__name__)
NAMESPACE = "micro_engram_b200"
_warned = False


def _unregistered(fn: Callable) -> Callable:
    """The surface of a registered op (call, register_fake) on the bare function itself."""
    fn.register_fake = lambda fake: fake
    return fn


def register_kernel_op(name: str, mutates_args: Sequence[str] = ()) -> Callable:
    """Decorator: register `fn` as torch.ops.micro_engram_b200.<name>; if this torch build
    refuses, keep `fn` callable as it is and say so once."""
    qualname = f"{NAMESPACE}::{name}"

    def deco(fn: Callable):
        global _warned
        try:
            return torch.library.custom_op(qualname, mutates_args=tuple(mutates_args))(fn)
        except Exception as exc:  # noqa: BLE001 - any registration failure keeps the kernel usable
            if not _warned:
                _warned = True
                LOG.warning("%s not registered (%s: %s): it runs as a plain call that torch.compile traces into",
                            qualname, type(exc).__name__, exc)
            return _unregistered(fn)

    return deco


@register_kernel_op("fill_ids", mutates_args=("out",))
def fill_ids(out: torch.Tensor, input_ids: torch.Tensor, positions: torch.Tensor, idx_mapping: torch.Tensor,
             query_start_loc: torch.Tensor, all_token_ids: torch.Tensor, num_reqs: int, num_tokens: int,
             num_tokens_padded: int) -> None:
    native().engram_fill_ids(out, input_ids, positions, idx_mapping, query_start_loc, all_token_ids,
                             num_reqs, num_tokens, num_tokens_padded)


@register_kernel_op("hash_prev")
def hash_prev(ids: torch.Tensor, canon: torch.Tensor, mults: torch.Tensor, orders: torch.Tensor,
              rows: torch.Tensor, pad_id: int) -> torch.Tensor:
    return native().engram_hash_prev(ids.long().contiguous(), canon, mults, orders, rows, pad_id)


@hash_prev.register_fake
def _(ids, canon, mults, orders, rows, pad_id):
    return ids.new_empty((mults.shape[0], ids.shape[0]), dtype=torch.int64)


@register_kernel_op("serve_inject", mutates_args=("status",))
def serve_inject(hidden: torch.Tensor, hist: torch.Tensor, canon: torch.Tensor, mults: torch.Tensor,
                 orders: torch.Tensor, rows: torch.Tensor, pad_id: int, w_ptrs: torch.Tensor, per: torch.Tensor,
                 world: int, dim: int, src_dtype: int, key_w: torch.Tensor, value_w: torch.Tensor,
                 q_scale: Optional[torch.Tensor], k_scale: Optional[torch.Tensor], keep: Optional[torch.Tensor],
                 sqrt_gate: bool, status: Optional[torch.Tensor]) -> torch.Tensor:
    """hidden [N, d] bf16 + the gated engram memory of the token histories `hist` [N, max_order].

    Rows are read straight from their owners' row stores (w_ptrs: per-rank table addresses),
    so a tensor-parallel server needs no all-reduce. q_scale/k_scale are the fp32 norm
    weights (1 + delta) for scalar_sqrt, None for scalar."""
    C = native()
    n = hidden.shape[0]
    idx = C.engram_hash_prev(hist[:n].long().contiguous(), canon, mults, orders, rows, pad_id)
    mem = C.engram_gather(idx, w_ptrs, per, world, dim, src_dtype, torch.bfloat16, status)
    k = C.gemm(mem, key_w.contiguous(), True, None)  # the tcgen05 GEMM, no library GEMM on this path
    v = C.gemm(mem, value_w.contiguous(), True, None)
    keep_u8 = keep.reshape(-1).to(torch.uint8).contiguous() if keep is not None else None
    out, _stats = C.engram_gate_fwd(hidden.contiguous(), k, v, q_scale, k_scale, keep_u8, sqrt_gate, None)
    return out


@serve_inject.register_fake
def _(hidden, hist, canon, mults, orders, rows, pad_id, w_ptrs, per, world, dim, src_dtype, key_w, value_w,
      q_scale, k_scale, keep, sqrt_gate, status):
    return torch.empty_like(hidden)


# Fused row-parallel linears (parallel/tp_linear.py) by handle: the op carries an int, the
# object (its peer buffers and call counter) stays on the host.
_TP_LINEARS: list = []


def add_tp_linear(obj) -> int:
    """Make a TPRowLinear callable through tp_row_linear; returns its handle."""
    _TP_LINEARS.append(obj)
    return len(_TP_LINEARS) - 1


@register_kernel_op("tp_row_linear")
def tp_row_linear(x: torch.Tensor, weight: torch.Tensor, handle: int) -> torch.Tensor:
    """x [M, K_local] . weight[N, K_local]^T summed over the tensor-parallel ranks, on every rank:
    the GEMM's epilogue reduce-scatters its fp32 partial over NVLink, then a slot sum and an
    all-gather. Collective (every rank calls it in the same order); eager only, since the call
    counter that pairs the ranks' buffers lives in the host object."""
    return _TP_LINEARS[handle](x, weight)


@tp_row_linear.register_fake
def _(x, weight, handle):
    return x.new_empty((x.shape[0], weight.shape[0]))
