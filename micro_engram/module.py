"""MicroEngram: a hashed n-gram memory injected into the residual stream of a frozen decoder.

Public surface and math match the reference (micro_engram/module.py:1-393): order-major
table layout, hashing `(sum_i tok[t-i] * mult[k,i]) % (2^31-1) % rows_k` with the canon map
and position_ids document boundaries, the scalar / scalar_sqrt / ple gates with a zero-init
output projection (exact no-op at step 0), delta-stored norm scales, row sharding and the
attachment hooks.

B200 path: on CUDA the hash is one kernel, row-sharded tables live in a RowStore (peer
memory over NVLink when world > 1) and are fetched by a gather kernel that reads the
owner's shard directly, and the scalar gates run as one fused forward / backward kernel.
The PyTorch code below is the CPU path and the oracle.
"""
import torch
import torch.nn as nn
import torch.nn.functional as F

from micro_engram_fork_b200.ops import use_native
from micro_engram_fork_b200.ops.linear import projection

_PRIME = 2_147_483_647  # 2^31 - 1


def resolve_order_sizes(table_size, orders=(2, 3), table_sizes=None):
    """{order: rows per table}, sorted by order.

    Each order of `orders` starts with `table_size` rows; `table_sizes` (int or string keys,
    as from JSON/YAML) overrides or adds orders. Orders whose size is 0 or None are dropped.
    """
    merged = {int(n): table_size for n in orders}
    merged.update({int(n): v for n, v in (table_sizes or {}).items()})
    sizes = {n: int(merged[n]) for n in sorted(merged) if merged[n]}
    if not sizes:
        raise ValueError("micro_engram: every n-gram order has size 0/None: nothing left to hash")
    if min(sizes) < 1 or min(sizes.values()) < 1:
        raise ValueError(f"micro_engram: bad orders/sizes {sizes}")
    return sizes


def hash_multipliers(seed, n_tables, max_order):
    """The odd multipliers of the n-gram hash, one row per table. This is a stored contract:
    trained tables are addressed through these numbers, so they must be reproduced bit for bit
    from the seed (a CPU torch.Generator seeded with `seed`, one randint draw of shape
    [n_tables, max_order] in [1, 2^31 - 1), low bit forced on)."""
    gen = torch.Generator().manual_seed(seed)
    return torch.randint(1, _PRIME, (n_tables, max_order), generator=gen, device="cpu") | 1


class MicroEngram(nn.Module):
    """Hashed n-gram memory (Engram-style) whose rows are gated into a decoder's hidden state.

    For position t, every n-gram order (2, 3, optionally 4) has `num_heads` tables; the n-gram
    ending at t is hashed into each of them and the rows found are concatenated into `mem`
    [.., n_tables * engram_dim] (tables in order-major, then head, order).

    Gates:
      scalar       h += sigmoid(<rms(h), rms(key(mem))> / sqrt(d)) * value(mem)
      scalar_sqrt  the same with a signed square root on the score, and learnable RMS-norm
                   scales on both sides of the score (kept as offsets from 1, see norm_scales)
      ple          h += up(gelu_tanh(down(rms(h))) * mem)
    The output projection (value, or up) starts at zero, so a new engram changes nothing.
    """

    GATES = ("scalar", "ple", "scalar_sqrt")
    SCALAR_GATES = ("scalar", "scalar_sqrt")
    DELTA_SCALES = ("q_scale", "k_scale")

    # row-sharding state lives in plain attributes, outside parameters() and the state dict
    row_shards = None
    row_info = None
    row_store = None
    row_lookup_fn = None  # a server's own lookup over row-sharded tables (vLLM tensor parallelism)

    def __init__(self, model_dim, table_size=65_536, engram_dim=128, num_heads=4, orders=(2, 3), pad_id=0,
                 seed=0, vocab_size=262_144, canon=None, gate="scalar", build_tables=True, table_sizes=None):
        super().__init__()
        if gate not in self.GATES:
            raise ValueError(f"gate must be one of {self.GATES}, got {gate!r}")
        self.gate, self.engram_dim, self.seed, self.pad_id = gate, engram_dim, seed, pad_id
        self._layout(table_size, orders, table_sizes, num_heads)
        if build_tables:
            self.tables = nn.ModuleList(nn.Embedding(rows, engram_dim) for rows in self.table_rows)
            for table in self.tables:
                nn.init.normal_(table.weight, std=0.02)
        self._gate_weights(model_dim, engram_dim * len(self._table_orders))
        self.register_buffer("mults", hash_multipliers(seed, len(self._table_orders), max(self.orders)))
        self.register_buffer("canon", self._canon_map(canon, vocab_size))
        self._dev_consts = {}

    def _layout(self, table_size, orders, table_sizes, num_heads):
        self.order_sizes = resolve_order_sizes(table_size, orders, table_sizes)
        self.orders = tuple(self.order_sizes)
        self._table_orders = [n for n in self.orders for _ in range(num_heads)]
        self.table_rows = [self.order_sizes[n] for n in self._table_orders]
        uniform = len(set(self.table_rows)) == 1
        self.table_size = self.table_rows[0] if uniform else None

    def _gate_weights(self, model_dim, mem_dim):
        if self.gate == "ple":
            self.down = nn.Linear(model_dim, mem_dim, bias=False)
            self.up = nn.Linear(mem_dim, model_dim, bias=False)
            nn.init.zeros_(self.up.weight)
            return
        self.key = nn.Linear(mem_dim, model_dim, bias=False)
        self.value = nn.Linear(mem_dim, model_dim, bias=False)
        nn.init.zeros_(self.value.weight)
        if self.gate == "scalar_sqrt":
            # stored as offsets from 1: in bf16 the spacing near 1.0 is 1/128, so an Adam step on
            # the scale itself would mostly round away
            self.q_scale = nn.Parameter(torch.zeros(model_dim))
            self.k_scale = nn.Parameter(torch.zeros(model_dim))

    @staticmethod
    def _canon_map(canon, vocab_size):
        if canon is None:
            return torch.arange(vocab_size)
        canon = torch.as_tensor(canon).long().clone()
        if canon.shape != (vocab_size,):
            raise ValueError(f"canon must have shape ({vocab_size},), got {tuple(canon.shape)}")
        return canon

    # ------------------------------------------------------------------ row sharding
    def shard_rows(self, rank, world, device=None, dtype=None, requires_grad=True, empty=False, pin_memory=False,
                   group=None, row_capacity=None):
        """Keep only this rank's rows of every table (ceil(rows/world) per rank).

        Rows come from the loaded tables when they exist, else a fresh N(0, 0.02) init with
        the per-rank seed `seed*1_000_003 + rank`, or stay uninitialised with `empty=True`
        (a server that loads the real rows next). On a CUDA device the rows live in a
        RowStore (peer-mapped when world > 1) that the fused lookup reads directly;
        `row_capacity` bounds the rows one optimizer step can touch on a rank (its compact
        gradient accumulator; a frozen or serving copy gets none).
        """
        from .rows import row_range

        spans = [row_range(rows, rank, world) for rows in self.table_rows]
        pers = [-(-rows // world) for rows in self.table_rows]
        device = torch.device(device) if device is not None else None
        src = None
        if "tables" in self._modules:
            src = [t.weight.detach()[a:a + c] for t, (a, c) in zip(self.tables, spans)]
            dtype = dtype or src[0].dtype
            del self.tables
        dtype = dtype or torch.float32
        on_cuda = device is not None and device.type == "cuda" and not pin_memory
        if on_cuda:
            from micro_engram_fork_b200.parallel.row_store import RowStore

            cap = row_capacity if requires_grad else 1
            store = RowStore(self.table_rows, self.engram_dim, dtype, rank, world, device, group=group, capacity=cap)
            shards = []
            gen = None
            for k, (_a, c) in enumerate(spans):
                view = store.shard(k)
                if src is not None:
                    view.copy_(src[k])
                elif not empty:
                    if gen is None:  # device generator: tables of tens of GB initialise in place
                        gen = torch.Generator(device=device).manual_seed(self.seed * 1_000_003 + rank)
                    view.copy_(torch.randn(c, self.engram_dim, generator=gen, device=device) * 0.02)
                shards.append(nn.Parameter(view, requires_grad=requires_grad))
            self.__dict__["row_store"] = store
        else:
            if src is None and empty:
                pin = pin_memory and torch.cuda.is_available()
                src = [torch.empty(c, self.engram_dim, device=None if pin else device, dtype=dtype, pin_memory=pin)
                       for _, c in spans]
                shards = [nn.Parameter(t, requires_grad=requires_grad) for t in src]
            else:
                if src is None:
                    gen = torch.Generator().manual_seed(self.seed * 1_000_003 + rank)
                    src = [torch.randn(c, self.engram_dim, generator=gen) * 0.02 for _, c in spans]
                shards = [nn.Parameter(t.to(device=device, dtype=dtype).clone(), requires_grad=requires_grad)
                          for t in src]
            self.__dict__["row_store"] = None
        self.__dict__["row_shards"] = shards
        self.__dict__["row_info"] = (rank, world, [a for a, _ in spans], pers)
        return shards

    def all_parameters(self):
        """Registered parameters plus this rank's table rows when row-sharded."""
        return list(self.parameters()) + list(self.row_shards or [])

    def lookup(self, idx):
        """Table rows for the hashed ids `idx` (one tensor per table): the module's own tables,
        or, when row-sharded, the installed lookup (vLLM's TP path) or the row exchange."""
        if self.row_shards is None:
            return [tab(i) for tab, i in zip(self.tables, idx)]
        if self.row_lookup_fn is None:
            from .rows import row_lookup

            return row_lookup(self, idx)
        return self.row_lookup_fn(self, idx)

    # ------------------------------------------------------------------ delta scales
    def norm_scales(self):
        """(q scale, k scale) in fp32: 1 + delta, with the delta made fp32 first."""
        return 1 + self.q_scale.float(), 1 + self.k_scale.float()

    def _shift_scales(self, sd, prefix, offset):
        """Module deltas <-> stored scales: a state dict holds 1 + delta in fp32 (in bf16 a small
        delta would round away), the module holds the delta itself."""
        for key in [prefix + n for n in self.DELTA_SCALES if prefix + n in sd]:
            sd[key] = sd[key].detach().float() + offset

    def _save_to_state_dict(self, destination, prefix, keep_vars):
        super()._save_to_state_dict(destination, prefix, keep_vars)
        self._shift_scales(destination, prefix, 1.0)

    def _load_from_state_dict(self, state_dict, prefix, *rest):
        self._shift_scales(state_dict, prefix, -1.0)
        super()._load_from_state_dict(state_dict, prefix, *rest)

    # ------------------------------------------------------------------ hashing
    def _consts(self, device):
        """Device copies of the hash constants (built once per device)."""
        key = str(device)
        c = self._dev_consts.get(key)
        if c is None or c[0].device != device:
            c = (self.canon.to(device=device, dtype=torch.long).contiguous(),
                 self.mults.to(device=device, dtype=torch.long).contiguous(),
                 torch.tensor(self._table_orders, dtype=torch.int32, device=device),
                 torch.tensor(self.table_rows, dtype=torch.long, device=device))
            self._dev_consts[key] = c
        return c

    def _apply(self, fn, *args, **kwargs):
        self._dev_consts = {}
        return super()._apply(fn, *args, **kwargs)

    def hash_ids(self, input_ids, position_ids=None):
        """One [B, T] tensor of row ids per table, for token ids [B, T]."""
        ids = input_ids.long()
        if use_native(ids):
            from micro_engram_fork_b200.ops.engram import hash_ids as _hash

            canon, mults, orders, rows = self._consts(ids.device)
            pos = position_ids.to(ids.device) if position_ids is not None else None
            out = _hash(ids, pos, canon, mults, orders, rows, self.pad_id)
            return list(out.reshape(len(self.table_rows), *ids.shape).unbind(0))
        canon = self.canon.to(ids.device)
        ids = canon[ids.clamp(0, canon.numel() - 1)]
        T = ids.shape[-1]
        max_n = max(self.orders)
        padded = F.pad(ids, (max_n - 1, 0), value=self.pad_id)
        # back[i][:, t] = token t - i (the pad id before the row start)
        back = [padded[..., max_n - 1 - i: max_n - 1 - i + T] for i in range(max_n)]
        if position_ids is not None:
            pos = position_ids.to(ids.device).expand_as(ids)
            back = [b if i == 0 else torch.where(pos >= i, b, torch.full_like(b, self.pad_id))
                    for i, b in enumerate(back)]
        return self._combine(back)

    def _combine(self, back):
        """Row ids per table from token columns back[i] = canonical token at t - i (pad where
        there is none): (sum_i back[i] * mults[k, i]) mod p mod rows_k, int64 arithmetic."""
        mults = self.mults.to(back[0].device)
        rows = []
        for k, order in enumerate(self._table_orders):
            terms = [back[i] * mults[k, i] for i in range(order)]
            rows.append((torch.stack(terms).sum(0) % _PRIME) % self.table_rows[k])
        return rows

    def hash_prev(self, ids):
        """Hashes from [N, max_order] histories: column i = token at t-i, -1 = none."""
        ids = ids.long()
        if use_native(ids):
            from micro_engram_fork_b200.ops.engram import hash_prev as _hash_prev

            canon, mults, orders, rows = self._consts(ids.device)
            return list(_hash_prev(ids.contiguous(), canon, mults, orders, rows, self.pad_id).unbind(0))
        canon = self.canon.to(ids.device)
        known = ids >= 0
        cols = canon[ids.clamp(0, canon.numel() - 1)].masked_fill(~known, self.pad_id)
        return self._combine(list(cols.unbind(1)))

    # ------------------------------------------------------------------ injection
    def _fused_ok(self, hidden):
        store = self.row_store
        return (store is not None and self.row_lookup_fn is None and use_native(hidden)
                and self.gate in self.SCALAR_GATES and hidden.dtype == torch.bfloat16
                and self.key.weight.dtype == torch.bfloat16 and self.value.weight.dtype == torch.bfloat16)

    def inject(self, hidden, idx, keep=None):
        """Add the gated memory for hashed rows `idx` to `hidden`.

        keep: optional [n_tokens] bool; False tokens get no memory (media placeholders)."""
        if self._fused_ok(hidden):
            return self._inject_fused(hidden, idx, keep)
        mem = torch.cat(self.lookup(idx), dim=-1)
        scalar = self.gate in self.SCALAR_GATES
        if self.row_shards is not None:  # gathered rows arrive in the table dtype
            mem = mem.to((self.key if scalar else self.up).weight.dtype)
        if scalar and (use_native(hidden) and hidden.dtype == torch.bfloat16 and mem.dtype == torch.bfloat16
                       and self.key.weight.dtype == torch.bfloat16):
            return self._gate_native(hidden, projection(mem, self.key.weight), projection(mem, self.value.weight),
                                     keep)
        added = self._scalar_gate_torch(hidden, mem) if scalar else self._ple_gate_torch(hidden, mem)
        if keep is not None:
            added = added * keep.reshape(*added.shape[:-1], 1).to(added.dtype)
        return hidden + added.to(hidden.dtype)

    def _scalar_gate_torch(self, hidden, mem):
        """sigmoid(<rms(h) q, rms(key(mem)) k> / sqrt(d)) * value(mem) in fp32; the scalar_sqrt gate
        takes the signed square root of the score and uses the learned norm scales."""
        d = hidden.shape[-1]
        qs, ks = self.norm_scales() if self.gate == "scalar_sqrt" else (None, None)
        score = (F.rms_norm(hidden.float(), (d,), weight=qs) * F.rms_norm(self.key(mem).float(), (d,), weight=ks))
        score = score.sum(-1, keepdim=True) / d ** 0.5
        if self.gate == "scalar_sqrt":
            score = torch.sign(score) * torch.sqrt(score.abs().clamp_min(1e-6))
        alpha = torch.sigmoid(score)
        if self.training:
            self._record_gate(alpha)
        return self.value(mem).float() * alpha

    def _ple_gate_torch(self, hidden, mem):
        """up(gelu_tanh(down(rms(h))) * mem) in fp32 (the per-layer-embedding style gate)."""
        normed = F.rms_norm(hidden.float(), (hidden.shape[-1],)).to(self.down.weight.dtype)
        return self.up(F.gelu(self.down(normed), approximate="tanh") * mem).float()

    def _gate_native(self, hidden, k, v, keep):
        from micro_engram_fork_b200.ops.engram import gate

        sqrt_gate = self.gate == "scalar_sqrt"
        acc = self._gate_acc(hidden.device) if self.training else None
        qd = self.q_scale if sqrt_gate else None
        kd = self.k_scale if sqrt_gate else None
        shape = hidden.shape
        d = shape[-1]
        out = gate(hidden.reshape(-1, d), k.reshape(-1, d), v.reshape(-1, d), qd, kd, keep, sqrt_gate, acc)
        return out.reshape(shape)

    def _inject_fused(self, hidden, idx, keep):
        from micro_engram_fork_b200.ops.engram import gather_rows

        flat = torch.stack([i.reshape(-1) for i in idx]) if isinstance(idx, (list, tuple)) else idx
        flat = flat.reshape(len(self.table_rows), -1).to(hidden.device).contiguous()
        mem = gather_rows(flat, self.row_store, torch.bfloat16, self.row_shards)
        k = projection(mem, self.key.weight)
        v = projection(mem, self.value.weight)
        return self._gate_native(hidden, k, v, keep)

    def forward(self, hidden, input_ids, position_ids=None):
        idx = self.hash_ids(input_ids.to(hidden.device), position_ids)
        return self.inject(hidden, idx)

    # ------------------------------------------------------------------ gate statistics
    def _gate_acc(self, device):
        acc = getattr(self, "_gate_stats", None)
        if acc is None or acc.device != device:
            acc = torch.zeros(3, device=device)
            self._gate_stats = acc
        return acc

    def _record_gate(self, alpha):
        a = alpha.detach().float()
        acc = self._gate_acc(a.device)
        acc += torch.stack([a.sum(), torch.tensor(float(a.numel()), device=a.device), (a > 0.99).float().sum()])

    def pop_gate_stats(self):
        """(mean gate, share of tokens with gate > 0.99) since the last call, or None."""
        stats = getattr(self, "_gate_stats", None)
        self._gate_stats = None
        if stats is None:
            return None
        s, n, sat = stats.tolist()
        if n == 0:
            return None
        return s / n, sat / n


def find_text_layers(model):
    """(name, ModuleList) of the language model's decoder layers (not a vision/audio tower).

    Preference order: a `...layers` list under a `language_model` module, then any `...layers`
    list outside a vision or audio tower."""
    def rank(name):
        if "language_model" in name:
            return 0
        return 1 if ("vision" not in name and "audio" not in name) else None

    best = None
    for name, mod in model.named_modules():
        if not (isinstance(mod, nn.ModuleList) and name.endswith("layers")):
            continue
        r = rank(name)
        if r is not None and (best is None or r < best[0]):
            best = (r, name, mod)
    if best is None:
        raise RuntimeError("Could not find text decoder layers; print(model) and set the path by hand.")
    return best[1], best[2]


def engram_from_spec(spec, model_dim, vocab_size, pad_default=0, canon=None, build_tables=True):
    """Build the MicroEngram a config spec describes (weights.engram_specs); its seed fixes the
    hash, so the same spec always addresses the same rows."""
    pad = spec.get("pad_id")
    kw = dict(table_size=spec["table_size"], table_sizes=spec.get("table_sizes"), engram_dim=spec["engram_dim"],
              num_heads=spec["num_heads"], orders=tuple(spec.get("orders") or (2, 3)),
              pad_id=pad_default if pad is None else pad, seed=spec.get("seed") or 0, gate=spec.get("gate") or "scalar")
    return MicroEngram(model_dim=model_dim, vocab_size=vocab_size, canon=canon, build_tables=build_tables, **kw)


def check_loaded(engram, sd, where):
    """Load `sd` into `engram`, refusing any mismatch. Saved `mults` may be missing (the seed
    rebuilds them); when present they must be the seed's, or the seed is wrong for the tables."""
    saved_mults = sd.get("mults")
    if saved_mults is not None and not torch.equal(saved_mults.to(engram.mults.device).long(), engram.mults.long()):
        raise ValueError(f"[micro_engram] {where}: the saved hash multipliers are not the ones this engram's seed "
                         "gives, so the seed does not belong to these weights")
    result = engram.load_state_dict(sd, strict=False)
    mismatch = [k for k in result.missing_keys if k != "mults"] + list(result.unexpected_keys)
    if mismatch:
        raise ValueError(f"[micro_engram] {where} does not fit the engram settings: {mismatch[:10]}")
    return result


_QUANTIZED_PARAMS = ("Params4bit", "Int8Params", "NF4Weight")


def layer_device_dtype(layer):
    """(device, compute dtype) for an engram placed in `layer`: the first real floating-point
    weight, else a quantized module's compute dtype, else bf16."""
    weights = list(layer.parameters())
    if not weights:
        raise RuntimeError("decoder layer has no parameters")
    plain = [w for w in weights if w.is_floating_point() and type(w).__name__ not in _QUANTIZED_PARAMS]
    if plain:
        return plain[0].device, plain[0].dtype
    declared = (getattr(m, "compute_dtype", None) for m in layer.modules())
    dtype = next((d for d in declared if isinstance(d, torch.dtype) and d.is_floating_point), torch.bfloat16)
    return weights[0].device, dtype


def attach_engram(model, engram, layer_idx, dtype=None, get_ids=None):
    """Nest `engram` in decoder layer `layer_idx` and inject it into that layer's output.

    get_ids: optional callable -> (input_ids, position_ids) for the current forward; by
    default a pre-hook on `model` captures them from its forward kwargs.
    Returns (the layer's module name, [hook handles]).
    """
    name, layers = find_text_layers(model)
    target = layers[layer_idx]
    device, layer_dtype = layer_device_dtype(target)
    engram.to(device=device, dtype=dtype or layer_dtype)
    target.add_module("micro_engram", engram)
    seen = {"input_ids": None, "position_ids": None}

    def capture(_mod, args, kwargs):
        seen["input_ids"] = kwargs.get("input_ids", args[0] if args else None)
        seen["position_ids"] = kwargs.get("position_ids")

    def current_ids():
        return get_ids() if get_ids is not None else (seen["input_ids"], seen["position_ids"])

    def inject(_mod, _args, output):
        ids, pos = current_ids()
        if ids is None:
            return output
        hidden = output[0] if isinstance(output, tuple) else output
        mixed = engram(hidden, ids, pos)
        return (mixed, *output[1:]) if isinstance(output, tuple) else mixed

    handles = [target.register_forward_hook(inject)]
    if get_ids is None:
        handles.append(model.register_forward_pre_hook(capture, with_kwargs=True))
    return f"{name}.{layer_idx}", handles
