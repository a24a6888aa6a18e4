"""Vocab-parallel tied embedding and chunked softcapped loss (full logits never exist).

Each rank keeps row_range(V) of the tied embedding / output head (outside the base):

  embed  every rank fetches its tokens' rows from their owners and scales by sqrt(d) (in
         the weight dtype, like Gemma4TextScaledWordEmbedding). CUDA: one gather kernel reads
         the owners' rows straight from their peer-mapped shards. CPU: the row all_to_all.
  loss   per chunk of tokens, the chunk's hidden states are gathered from all ranks, each rank
         computes logits against its own vocab rows (bf16 GEMM, fp32 softcap), and the
         per-row (max, sum-exp, target logit) partials are combined across ranks into the LSE.
         CUDA: the logits GEMM's epilogue produces the partials, the logits are overwritten in
         place with (softmax - onehot) * w * softcap', and the dH GEMM's epilogue stores each
         token's rows on its owner's GPU; every exchange between ranks goes through peer
         memory (micro_engram_fork_b200/parallel/vocab_comm.py), none through NCCL.

Every rank runs the same chunk count: the chunk size comes from ceil(V/world), never from
this rank's own row count (micro_engram/train/head.py:38-42 of the reference). Loss terms
are sums; the trainer divides by the step's trained-token count.
"""
import torch
import torch.distributed as dist

from micro_engram_fork_b200.ops import use_native

from ..rows import _group, _RowLookup, row_range

IGNORE = -100


class VocabShard:
    """This rank's rows of the tied embedding / output head and the loss over them."""

    def __init__(self, weight, rank, world, embed_scale=None, softcap=None, chunk_tokens=2048,
                 chunk_bytes=256 << 20, device=None, dtype=None):
        V, d = weight.shape
        self.V, self.d, self.rank, self.world = int(V), int(d), rank, world
        self.per = -(-self.V // world)  # rows per rank (the last ranks may hold fewer real ones)
        self.start, self.rows = row_range(self.V, rank, world)
        device = weight.device if device is None else torch.device(device)
        dtype = dtype or weight.dtype
        self._buf = self._comm = None
        local = weight.detach()[self.start:self.start + self.rows]
        if device.type == "cuda" and world > 1 and use_native(torch.empty(0, device=device)):
            # peer-mapped shard (padded to `per` rows, same layout on every rank)
            from micro_engram_fork_b200.parallel.symm import SymmBuffer

            esz = torch.empty((), dtype=dtype).element_size()
            per8 = -(-self.per // 8) * 8
            self._buf = SymmBuffer(per8 * self.d * esz, device, _group(world))
            full = self._buf.view(0, (per8, self.d), dtype)
            full.zero_()
            full[:self.rows].copy_(local.to(device=device, dtype=dtype))
            self.weight = full[:self.rows]
            # the tcgen05 head GEMMs read whole 16-byte rows of logits: rows padded with zeros
            # to a multiple of 8 (zero rows add nothing to dH; the loss masks their columns)
            self.gemm_weight = full[:-(-self.rows // 8) * 8]
            self._ptrs = torch.tensor(self._buf.ptrs, dtype=torch.int64, device=device)
        else:
            self.weight = local.to(device=device, dtype=dtype).clone()
            self._ptrs = None
            pad = -(-self.rows // 8) * 8 - self.rows
            self.gemm_weight = (torch.cat([self.weight, self.weight.new_zeros(pad, self.d)]) if pad else self.weight)
        self._per_t = None
        self.embed_scale = embed_scale
        self.softcap = softcap
        fit = max(64, chunk_bytes // max(1, world * self.per * 4))
        self.chunk = max(1, min(chunk_tokens, fit))
        # the CUDA path keeps each chunk's logits in bf16 (and overwrites them with their
        # gradient): 1 GiB of logits per chunk, i.e. 2048-token chunks at the benchmark vocab
        fit16 = max(64, (1 << 30) // max(1, world * self.per * 2))
        self.chunk_bf16 = max(1, min(chunk_tokens, fit16))

    @property
    def group(self):
        return _group(self.world)

    def comm(self):
        """The peer-memory exchange of the CUDA loss (built on first use; collective)."""
        if self._comm is None:
            import os

            from micro_engram_fork_b200.parallel.vocab_comm import VocabComm

            timeout = float(os.environ.get("MICRO_ENGRAM_PEER_TIMEOUT_S", "10"))
            self._comm = VocabComm(self.chunk_bf16, self.d, self.weight.device, self.group, timeout_s=timeout)
        return self._comm

    def check_status(self):
        if self._comm is not None:
            self._comm.check_status()

    @torch.no_grad()
    def embed(self, ids):
        """[*ids.shape, d] embeddings (frozen, no autograd), times sqrt(d) in the weight dtype."""
        flat = ids.reshape(-1).to(self.weight.device)
        if use_native(flat):
            from micro_engram_fork_b200 import native

            if self._ptrs is None:
                out = self.weight.index_select(0, flat)
            else:
                if self._per_t is None:
                    self._per_t = torch.tensor([self.per], dtype=torch.int64, device=flat.device)
                src = 0 if self.weight.dtype == torch.bfloat16 else 1
                out = native().engram_gather(flat.long().reshape(1, -1).contiguous(), self._ptrs, self._per_t,
                                             self.world, self.d, src, self.weight.dtype, None)
        else:
            out = _RowLookup.apply(flat, ([0, self.V], [self.per], self.rank, self.world), self.weight)
        out = out.reshape(*ids.shape, self.d)
        if self.embed_scale is not None:
            out = out * torch.tensor(self.embed_scale, dtype=self.weight.dtype, device=out.device)
        return out

    def loss_sum(self, hidden, labels):
        """(sum of this rank's token losses, its trained-token count). hidden [N, d] requires
        grad; labels [N] with -100 untrained. Collective: every rank calls it with the same N."""
        count = (labels != IGNORE).sum()
        labels = labels.to(hidden.device)
        if use_native(hidden) and self.weight.dtype == torch.bfloat16:
            total = _FusedVocabCE.apply(hidden, labels, self, torch.is_grad_enabled() and hidden.requires_grad)
        else:
            total = _VocabParallelCE.apply(hidden, labels, self)
        return total, count


def _gather(x, group, world):
    if world == 1:
        return x
    out = x.new_empty((world * x.shape[0],) + tuple(x.shape[1:]))
    dist.all_gather_into_tensor(out, x.contiguous(), group=group)
    return out


def _reduce_scatter(x, n, d, group, world):
    if world == 1:
        return x
    out = torch.empty(n, d, dtype=x.dtype, device=x.device)
    dist.reduce_scatter_tensor(out, x.contiguous(), group=group)
    return out


def _softcapped_logits(h, w, softcap):
    """fp32 logits of a chunk against this rank's vocab rows (from the bf16 product, as the
    model computes them), softcapped as c * tanh(z / c)."""
    z = (h @ w.t()).float()
    return torch.tanh(z / softcap) * softcap if softcap else z


def _local_partials(z, labels, start, rows):
    """Per token: this rank's row max m, sum of exp(z - m) over its vocab rows, and the target
    logit when the label is one of its rows (else 0)."""
    m = z.amax(dim=1)
    s = torch.exp(z - m[:, None]).sum(dim=1)
    col = labels - start
    here = (labels != IGNORE) & (col >= 0) & (col < rows)
    picked = z.gather(1, col.clamp(0, rows - 1)[:, None]).squeeze(1)
    return m, s, torch.where(here, picked, torch.zeros_like(picked))


def _merge_ranks(m, s, tgt, group, world):
    """(log-sum-exp over the whole vocabulary, target logit): every rank's (m, s, target)
    partials are all-gathered once and merged locally."""
    if world == 1:
        return m + torch.log(s), tgt
    mine = torch.stack([m, s, tgt])
    every = mine.new_empty((world * 3, mine.shape[1]))
    dist.all_gather_into_tensor(every, mine.contiguous(), group=group)
    every = every.view(world, 3, -1)
    top = every[:, 0].amax(dim=0)
    total = (every[:, 1] * torch.exp(every[:, 0] - top)).sum(dim=0)
    return top + torch.log(total), every[:, 2].sum(dim=0)


class _VocabParallelCE(torch.autograd.Function):
    """PyTorch path (CPU / gloo, and the oracle of the CUDA path). Forward: per chunk of tokens
    (gathered from every rank), partials against this rank's vocab rows, merged over ranks into
    each token's log-sum-exp; only the LSEs are kept. Backward: the chunk's logits again,
    softmax - onehot (times softcap'), weighted by each token's own rank's loss weight, through
    the head into dH, reduce-scattered back to the tokens' ranks."""

    @staticmethod
    def forward(ctx, hidden, labels, shard):
        world, group, w = shard.world, shard.group, shard.weight
        h = hidden.detach().to(w.dtype)
        total = torch.zeros((), dtype=torch.float32, device=hidden.device)
        lses = []
        for a, b in _chunks(hidden.shape[0], shard.chunk):
            L = _gather(labels[a:b].contiguous(), group, world)
            z = _softcapped_logits(_gather(h[a:b], group, world), w, shard.softcap)
            lse, tgt = _merge_ranks(*_local_partials(z, L, shard.start, shard.rows), group, world)
            mine = slice(shard.rank * (b - a), (shard.rank + 1) * (b - a))
            trained = L[mine] != IGNORE
            total = total + torch.where(trained, lse[mine] - tgt[mine], torch.zeros_like(tgt[mine])).sum()
            lses.append(lse)
        ctx.shard = shard
        ctx.save_for_backward(hidden.detach(), labels, *lses)
        return total

    @staticmethod
    def backward(ctx, g):
        shard = ctx.shard
        hidden, labels, *lses = ctx.saved_tensors
        world, group, w = shard.world, shard.group, shard.weight
        weights = _gather(g.detach().float().reshape(1), group, world)  # each rank's loss weight
        h = hidden.to(w.dtype)
        grad = torch.empty(hidden.shape[0], shard.d, dtype=hidden.dtype, device=hidden.device)
        for (a, b), lse in zip(_chunks(hidden.shape[0], shard.chunk), lses):
            n = b - a
            L = _gather(labels[a:b].contiguous(), group, world)
            z = _softcapped_logits(_gather(h[a:b], group, world), w, shard.softcap)
            p = torch.exp(z - lse[:, None])
            col = L - shard.start
            here = ((L != IGNORE) & (col >= 0) & (col < shard.rows)).nonzero().squeeze(1)
            p[here, col[here]] -= 1
            row_weight = weights.repeat_interleave(n) * (L != IGNORE).float()
            p *= row_weight[:, None]
            if shard.softcap:
                p *= 1 - (z / shard.softcap).square()
            dH = (p.to(w.dtype) @ w).float()
            grad[a:b] = _reduce_scatter(dH, n, shard.d, group, world).to(grad.dtype)
        return grad, None, None


def _chunks(n, size):
    return [(a, min(n, a + size)) for a in range(0, n, size)]


class _FusedVocabCE(torch.autograd.Function):
    """CUDA path, per chunk of tokens (gathered from every rank):

      1. one tcgen05 GEMM of the chunk against this rank's vocab rows whose epilogue softcaps
         the bf16 logits and reduces each 256-column tile to a partial sum of exp(zc - cap) plus
         the target logit (gemm_ce); with a softcap every partial shares the offset `cap`, so the
         ranks combine by a plain sum: lse = cap + log(sum of partials). The bf16 logits are
         kept only when a gradient is needed;
      2. the logits are overwritten in place with (softmax - onehot) * softcap' (ce_bwd_inplace,
         SFU exp/tanh, one pass) and multiplied into dH on the tcgen05 GEMM with fp32 output,
         whose epilogue stores each token's rows straight into its owner's receive slot.

    Across ranks every exchange goes through peer memory (VocabComm: the chunk's hidden states
    and labels, the (max, sum, target) partials, dH), with no NCCL call; the partials are
    merged in rank order, so the loss is the same on every run.

    The backward only scales this rank's dH rows by the incoming gradient (the loss is linear
    in it), so the logits GEMM runs once per chunk. Reference semantics:
    micro_engram/train/head.py:76-165 (softcap as tanh(z/c)*c on the fp32 value of the bf16
    logits; loss = sum over trained tokens of lse - target)."""

    @staticmethod
    def forward(ctx, hidden, labels, shard, need_grad):
        from micro_engram_fork_b200 import native

        C = native()
        world, w = shard.world, shard.gemm_weight
        N, c = hidden.shape[0], shard.chunk_bf16
        cap = float(shard.softcap or 0.0)
        comm = shard.comm() if world > 1 else None
        h = hidden.detach().to(w.dtype).contiguous()
        total = torch.zeros((), dtype=torch.float32, device=hidden.device)
        dh = torch.empty(N, shard.d, dtype=torch.float32, device=hidden.device) if need_grad else None
        for a in range(0, N, c):
            b = min(N, a + c)
            n = b - a
            H, L = comm.gather(h[a:b], labels[a:b].contiguous()) if comm else (h[a:b], labels[a:b].contiguous())
            s_part, m_part, tgt, z = C.gemm_ce(H, w, L, shard.start, cap, need_grad, shard.rows)
            if cap > 0:  # every partial shares the offset cap
                m, s = torch.full_like(tgt, cap), s_part.sum(1)
            else:
                m = m_part.amax(1)
                s = (s_part * torch.exp(m_part - m[:, None])).sum(1)
            if comm:
                lse, tgt = comm.merge(m, s, tgt)
            else:
                lse = m + torch.log(s)
            own = slice(shard.rank * n, (shard.rank + 1) * n)
            valid = L[own] != IGNORE
            total = total + torch.where(valid, lse[own] - tgt[own], torch.zeros_like(lse[own])).sum()
            if need_grad:
                C.ce_bwd_inplace(z, L, shard.start, cap, lse, (L != IGNORE).float())
                if comm:
                    comm.scatter_sum(z, w, dh[a:b])
                else:
                    dh[a:b] = C.gemm_f32(z, w)
            del z
        ctx.dh, ctx.hdtype = dh, hidden.dtype
        return total

    @staticmethod
    def backward(ctx, g):
        dh, ctx.dh = ctx.dh, None
        return (dh * g.float()).to(ctx.hdtype), None, None, None


def reference_loss_sum(hidden, labels, weight, softcap=None):
    """Summed token cross-entropy over the whole vocabulary, the plain way (the tests' oracle for
    the vocab-parallel loss): fp32 logits hidden . weight^T, the optional softcap
    cap * tanh(z / cap), then log-sum-exp minus the target logit, over tokens whose label is not
    IGNORE."""
    logits = torch.mm(hidden.to(weight.dtype), weight.t()).float()
    if softcap:
        logits = softcap * torch.tanh(logits / softcap)
    keep = labels.ne(IGNORE)
    picked = torch.take_along_dim(logits, labels.masked_fill(~keep, 0).unsqueeze(1), dim=1).squeeze(1)
    return ((torch.logsumexp(logits, dim=1) - picked) * keep).sum()
