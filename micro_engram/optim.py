"""LazyAdamW and stochastic bf16 rounding (semantics of micro_engram/optim.py:1-133).

AdamW with decoupled weight decay and a global step count, state names as
torch.optim.AdamW (step, exp_avg, exp_avg_sq). Per parameter group:

  lazy=True      a row whose gradient is all zero is left exactly as it is (weight and both
                 moments), like SparseAdam, also on dense gradients
  rowwise=True   ONE fp32 second moment per row, the running mean of the row's g^2 (FBGEMM /
                 TorchRec partial row-wise Adam); kept fp32 whatever the weight dtype, since a
                 bf16 v = 0.999 v + 0.001 g^2 stops moving once v has grown

bf16 weights and states are written back with stochastic rounding when enabled.

On CUDA the update runs in the sm_100a kernels: row-sharded tables with a RowStore are
updated on their touched rows only, every lazy table of a store in one launch (8 lanes per
row with 16-byte accesses, Philox4x32-10 rounding bits, the accumulator cleared in the same
pass); other CUDA parameters use a fused elementwise AdamW.
"""
import torch

from micro_engram_fork_b200.ops import use_native


def _nonzero_rows(g):
    """Indices of the rows of g (first dimension) that hold any non-zero value."""
    return g.reshape(g.shape[0], -1).ne(0).any(dim=1).nonzero().squeeze(1)


def _local(t):
    to_local = getattr(t, "to_local", None)
    return to_local() if to_local is not None else t


def stochastic_bf16(x):
    """fp32 -> bf16 with stochastic rounding: 16 random bits are added below the kept mantissa
    and cut off, so a value rounds up with probability equal to the dropped fraction. The
    sign is its own bit, so this is unbiased for both signs; inf/nan pass through."""
    x = x.float().contiguous()
    noise = torch.randint(0, 1 << 16, x.shape, dtype=torch.int32, device=x.device)
    bits = (x.view(torch.int32) + noise) & -65536
    out = torch.where(torch.isfinite(x), bits.view(torch.float32), x)
    return out.to(torch.bfloat16)


_SEED_BASE = 0x5EED


def _batchable(p):
    """Row-store tables the batched touched-row kernel takes: bf16 or fp32, width a multiple of 8."""
    return p.is_cuda and p.dtype in (torch.bfloat16, torch.float32) and p.dim() == 2 and p.shape[1] % 8 == 0 \
        and p.shape[1] <= 256


def _evaluate(closure):
    if closure is None:
        return None
    with torch.enable_grad():
        return closure()


class _Hyper:
    """One group's AdamW constants at a given step (bias corrections included)."""

    __slots__ = ("lr", "beta1", "beta2", "eps", "wd", "bc1", "bc2", "sr", "step")

    @classmethod
    def of(cls, group, step):
        h = cls()
        h.beta1, h.beta2 = group["betas"]
        h.lr, h.eps, h.wd = group["lr"], group["eps"], group["weight_decay"]
        h.bc1, h.bc2 = 1 - h.beta1 ** step, 1 - h.beta2 ** step
        h.sr = bool(group.get("stochastic_rounding", True))
        h.step = int(step)
        return h


class LazyAdamW(torch.optim.Optimizer):
    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0, lazy=False, rowwise=False,
                 stochastic_rounding=True):
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, lazy=lazy,
                                      rowwise=rowwise, stochastic_rounding=stochastic_rounding))
        self.row_moments_on_host = False

    @staticmethod
    def _host_moment(p):
        """Lazy row-store tables can keep their table-sized moments in pinned host memory: the
        touched-row kernel reads and writes them in place over PCIe (mapped memory), a few
        rows per step."""
        return getattr(p, "_row_store", None) is not None and p.is_cuda

    @staticmethod
    def init_state(state, p, group, on_host=False):
        """Fresh state: exp_avg like p (pinned host memory with `on_host`); exp_avg_sq like p,
        or [rows] fp32 when row-wise."""
        state["step"] = torch.zeros((), dtype=torch.float32)
        if on_host:
            state["exp_avg"] = torch.zeros(p.shape, dtype=p.dtype, pin_memory=True)
        else:
            state["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
        if group.get("rowwise") and p.dim() >= 2:
            state["exp_avg_sq"] = torch.zeros(p.shape[0], dtype=torch.float32, device=p.device)
        elif on_host:
            state["exp_avg_sq"] = torch.zeros(p.shape, dtype=p.dtype, pin_memory=True)
        else:
            state["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)

    def _on_host(self, p, group):
        return self.row_moments_on_host and group["lazy"] and self._host_moment(p)

    @torch.no_grad()
    def materialize_state(self):
        """Create every parameter's state now (instead of at the first step), so memory
        planning sees the optimizer's full footprint."""
        for group in self.param_groups:
            for p in group["params"]:
                if not self.state[p]:
                    self.init_state(self.state[p], p, group, self._on_host(p, group))

    @torch.no_grad()
    def move_row_moments_to_host(self):
        """Move the lazy row-store tables' exp_avg (and a per-value exp_avg_sq), each as large
        as the tables, to pinned host memory, now and for state created later. Returns the
        device bytes freed."""
        self.row_moments_on_host = True
        freed = 0
        for group in self.param_groups:
            for p in group["params"]:
                st = self.state[p]
                if not (st and self._on_host(p, group)):
                    continue
                for key in ("exp_avg", "exp_avg_sq"):  # exp_avg_sq only when it is per value
                    t = st[key]
                    if t.is_cuda and t.shape == p.shape:
                        host = torch.empty(p.shape, dtype=t.dtype, pin_memory=True)
                        host.copy_(t)
                        freed += t.numel() * t.element_size()
                        st[key] = host
        return freed

    @torch.no_grad()
    def step(self, closure=None):
        loss = _evaluate(closure)
        done = {}  # row stores whose touched rows the kernels consumed (and cleared) this step
        batches = {}  # (store, group) -> lazy tables updated by one batched launch
        for group, p in ((g, p) for g in self.param_groups for p in g["params"]):
            owner = getattr(p, "_row_store", None)
            if owner is None:
                self._step_param(p, group)
                continue
            store = owner[0]
            if group["lazy"] and store.pending and _batchable(p):
                batches.setdefault((id(store), id(group)), (store, group, []))[2].append(p)
            else:
                self._step_store(p, group)
            done[id(store)] = store
        for store, group, params in batches.values():
            self._step_store_batch(store, group, params)
        for store in done.values():
            store.pending, store.coef = False, None
        return loss

    def _advance(self, p, group, on_host=False):
        """Create the state on first use, count the step and return the update's constants."""
        state = self.state[p]
        if not state:
            self.init_state(state, p, group, on_host)
        state["step"] += 1
        return state, _Hyper.of(group, float(state["step"]))

    # ------------------------------------------------------------------ row-store tables (CUDA)
    def _step_store(self, p, group):
        store, k = p._row_store
        if not store.pending:
            return
        state, h = self._advance(p, group, self._on_host(p, group))
        seed = (_SEED_BASE + 7919 * store.rank + 104729 * getattr(store, "salt", 0)) & 0x7FFFFFFF
        from micro_engram_fork_b200.ops.engram import adam_dense, adam_touched

        coef = getattr(store, "coef", None)
        if group["lazy"]:
            adam_touched(p.data, state["exp_avg"], state["exp_avg_sq"], store.acc[k], store.pos[k],
                         store.list[k], store.count[k], coef, h.lr, h.beta1, h.beta2, h.eps, h.wd, h.bc1, h.bc2,
                         h.sr, seed, h.step, k)
        else:  # every row steps: densify the compact accumulator for this table
            n = p.shape[0]
            g = store.dense_grad(k)[:n]
            if coef is not None:
                g.mul_(coef)
            adam_dense(p.data, g, state["exp_avg"], state["exp_avg_sq"], h.lr, h.beta1, h.beta2, h.eps, h.wd, h.bc1,
                       h.bc2, 1.0, h.sr, seed, h.step)
            del g
            used = min(int(store.count[k][0]), store.cap[k])
            rows = store.list[k][:used].long()
            store.pos[k].index_fill_(0, rows[rows >= 0], 0)
            store.acc[k][:used].zero_()
        store.count[k].zero_()

    def _step_store_batch(self, store, group, params):
        """The lazy update of several tables of one row store in one kernel launch."""
        from micro_engram_fork_b200 import native

        seed = (_SEED_BASE + 7919 * store.rank + 104729 * getattr(store, "salt", 0)) & 0x7FFFFFFF
        cols = {key: [] for key in ("p", "m", "v", "acc", "pos", "list", "cnt", "k", "bc1", "bc2", "step")}
        h = None
        for p in params:
            k = p._row_store[1]
            state, h = self._advance(p, group, self._on_host(p, group))
            for key, val in (("p", p.data), ("m", state["exp_avg"]), ("v", state["exp_avg_sq"]), ("acc", store.acc[k]),
                             ("pos", store.pos[k]), ("list", store.list[k]), ("cnt", store.count[k]), ("k", k),
                             ("bc1", h.bc1), ("bc2", h.bc2), ("step", h.step)):
                cols[key].append(val)
        native().engram_adam_rows(cols["p"], cols["m"], cols["v"], cols["acc"], cols["pos"], cols["list"], cols["cnt"],
                                  cols["k"], cols["bc1"], cols["bc2"], cols["step"], getattr(store, "coef", None),
                                  h.lr, h.beta1, h.beta2, h.eps, h.wd, h.sr, seed)
        torch._foreach_zero_(cols["cnt"])

    # ------------------------------------------------------------------ everything else
    def _step_param(self, p, group):
        sparse = getattr(p, "sparse_grad", None)
        if sparse is None and p.grad is None:
            return
        state, h = self._advance(p, group)
        lr, beta1, beta2, eps, wd, bc1, bc2, sr = h.lr, h.beta1, h.beta2, h.eps, h.wd, h.bc1, h.bc2, h.sr
        P, M, V = _local(p), _local(state["exp_avg"]), _local(state["exp_avg_sq"])
        fused = (sparse is None and not group["lazy"] and use_native(P) and M.dim() == V.dim()
                 and P.dtype in (torch.bfloat16, torch.float32) and P.is_contiguous())
        if fused:
            from micro_engram_fork_b200.ops.engram import adam_dense

            G = _local(p.grad)
            G = G if G.dtype in (torch.float32, P.dtype) else G.float()
            adam_dense(P, G.contiguous(), M, V, lr, beta1, beta2, eps, wd, bc1, bc2, 1.0,
                       sr and P.dtype == torch.bfloat16, _SEED_BASE ^ (id(p) & 0xFFFF), h.step)
            return
        rows = None
        if sparse is not None:
            if not group["lazy"]:
                raise ValueError("sparse row gradients need lazy=True")
            rows, g = sparse
            live = _nonzero_rows(g)
            rows, g = rows[live], g[live]
            if rows.numel() == 0:
                return
            pw = P.index_select(0, rows).float()
            m, v = M.index_select(0, rows).float(), V.index_select(0, rows).float()
        elif group["lazy"] and P.dim() >= 2:
            G = _local(p.grad)
            rows = _nonzero_rows(G)
            if rows.numel() == 0:
                return
            pw, g = P.index_select(0, rows).float(), G.index_select(0, rows).float()
            m, v = M.index_select(0, rows).float(), V.index_select(0, rows).float()
        else:
            G = _local(p.grad)
            pw, g, m, v = P.float(), G.float(), M.float(), V.float()
        if wd:
            pw.mul_(1 - lr * wd)
        m.mul_(beta1).add_(g, alpha=1 - beta1)
        if v.dim() < g.dim():
            v.mul_(beta2).add_(g.pow(2).flatten(1).mean(dim=1), alpha=1 - beta2)
            denom = (v.sqrt() / bc2 ** 0.5).add_(eps).reshape(-1, *([1] * (g.dim() - 1)))
        else:
            v.mul_(beta2).addcmul_(g, g, value=1 - beta2)
            denom = (v.sqrt() / bc2 ** 0.5).add_(eps)
        pw.addcdiv_(m, denom, value=-lr / bc1)

        def cast(x, dtype):
            return stochastic_bf16(x) if sr and dtype == torch.bfloat16 else x.to(dtype)

        if rows is None:
            P.copy_(cast(pw, P.dtype))
            M.copy_(cast(m, M.dtype))
            V.copy_(cast(v, V.dtype))
        else:
            P.index_copy_(0, rows, cast(pw, P.dtype))
            M.index_copy_(0, rows, cast(m, M.dtype))
            V.index_copy_(0, rows, cast(v, V.dtype))
