"""micro_engram.train: the training loop (plain PyTorch + the sm_100a engine, one process per GPU).

What runs where, per GPU:
  base model      frozen Gemma-4-style decoder (our own, sm_100a kernels), replicated when it
                  fits in HBM (it does for 31B bf16 on B200), activation checkpointing per
                  layer with optional host offload of the layer inputs
  embedding/head  vocab rows split over the GPUs (head.VocabShard): peer-read embedding,
                  chunked vocab-parallel softcapped loss
  engram tables   row-sharded (rows.RowTables) in peer-mapped row stores: fused fetch, row
                  gradients pushed to the owners, touched-row AdamW + stochastic rounding
  engram dense    key/value/gate/scales replicated, gradients all-reduced, fused AdamW

Flow and outputs follow the reference trainer (micro_engram/train/loop.py:1-595): same
build order, per-token mean loss over the whole step, clipping of the dense part and of
the tables (global norm), LR schedules, JSONL logs, checkpoints (trainer_state.json last),
rotation, resume at any GPU count, profile_step, and fail-fast exit.
"""
import json
import logging
import math
import os
import shutil
import time

import torch
import torch.distributed as dist

from ..rows import ROWS_DIR, ROWS_OPTIM_DIR, RowTables, dist_rank_world
from ..runconfig import (CONFIG_NAME, _params, _safe_fingerprint, build_config, build_slot, check_canon,
                         engram_requests, epoch_step_scheduler, write_config)
from ..stats import module_stats
from . import model as M
from .data import EpochPlan, collate, prepare
from .offload import ActivationOffload

LOG = logging.getLogger("micro_engram.train")
STATE_FILE = "trainer_state.json"
DENSE_FILE = "micro_engram_dense_optim.pt"


def _log0(msg):
    if dist_rank_world()[0] == 0:
        LOG.warning(msg)


def setup_dist(timeout_s=None):
    rank, world = dist_rank_world()
    if world == 1 and "MASTER_ADDR" not in os.environ:  # single process without a launcher
        import socket

        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            port = s.getsockname()[1]
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", str(port))
    local = int(os.environ.get("LOCAL_RANK", 0))
    cuda = torch.cuda.is_available() and os.environ.get("MICRO_ENGRAM_CPU") != "1"
    if cuda:
        torch.cuda.set_device(local)
        device = torch.device("cuda", local)
    else:
        device = torch.device("cpu")
    if not dist.is_initialized():
        import datetime

        kw = {"device_id": device} if cuda else {}
        if timeout_s:
            kw["timeout"] = datetime.timedelta(seconds=timeout_s)
        dist.init_process_group("nccl" if cuda else "gloo", rank=rank, world_size=world, **kw)
    return rank, world, local, device


class _null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


class Trainer:
    def __init__(self, cfg):
        self.cfg = cfg
        self.rank, self.world, self.local, self.device = setup_dist()
        self.ctx = {"ids": None, "pos": None}
        self.global_step, self.epoch, self.step_in_epoch = 0, 0, 0
        self.wandb = None
        self.pbar = None
        if cfg.kernels == "reference":
            os.environ["MICRO_ENGRAM_REFERENCE_OPS"] = "1"
        if cfg.tf32 and self.device.type == "cuda":
            torch.backends.cuda.matmul.allow_tf32 = True
            torch.backends.cudnn.allow_tf32 = True

    # ------------------------------------------------------------------ setup
    def build(self, samples=None, tokenizer=None):
        """Everything a run needs. `samples`/`tokenizer` may be given directly (synthetic data)."""
        cfg = self.cfg
        torch.manual_seed(cfg.seed)
        tok_path = cfg.tokenizer_config or cfg.base_model
        if samples is None:
            from transformers import AutoTokenizer

            self.tokenizer = AutoTokenizer.from_pretrained(tok_path)
            self.samples = prepare(cfg, self.tokenizer, tok_path, rank=self.rank,
                                   barrier=dist.barrier if self.world > 1 else None)
        else:
            self.tokenizer, self.samples = tokenizer, samples
        self.plan = EpochPlan(self.samples, cfg, self.world)
        pad = getattr(self.tokenizer, "pad_token_id", None) if self.tokenizer is not None else None
        self.pad_id = pad if pad is not None else 0

        M.apply_kernel_patches(cfg, self.device.type == "cuda")
        model, meta = M.load_base(cfg, self.rank, self.local, self.device)
        self.model = model
        self.text_name, self.text = M.text_model(model)
        text_cfg = self.text.config
        self.placement = M.place_base(self.text, cfg, self.device, self.world)
        self.vocab = M.take_vocab(model, self.text, self.rank, self.world, self.device, broadcast=False,
                                  chunk_tokens=cfg.loss_chunk_tokens)

        canon = None
        if cfg.micro_engram_canon_path:
            canon = check_canon(torch.load(cfg.micro_engram_canon_path, map_location="cpu"), text_cfg.vocab_size)
            _log0(f"[micro_engram] token merging ON: {canon.numel():,} ids -> {int(torch.unique(canon).numel()):,} "
                  f"classes ({cfg.micro_engram_canon_path})")
        from ..rows import _group

        self.slots = []
        # one optimizer step looks up at most (bins per step over all ranks) x sequence_len rows
        # per table on any rank: the bound of the row stores' compact gradient accumulators
        row_capacity = self.plan.per_step * cfg.sequence_len
        for spec, init_from, frozen in engram_requests(cfg):
            spec["canon_path"] = cfg.micro_engram_canon_path
            self.slots.append(build_slot(spec, init_from, frozen, model, text_cfg, canon, dtype=cfg.micro_engram_dtype,
                                         sharding="rows", get_ids=lambda: (self.ctx["ids"], self.ctx["pos"]),
                                         device=self.device, group=_group(self.world), row_capacity=row_capacity))
        for s in self.slots:
            if s.frozen:
                for p in _params(s.engram):
                    p.requires_grad_(False)
        if not cfg.micro_engram_train_scales:
            n = 0
            for s in self.slots:
                for name in getattr(s.engram, "DELTA_SCALES", ()):
                    p = getattr(s.engram, name, None)
                    if isinstance(p, torch.nn.Parameter) and p.requires_grad:
                        p.requires_grad_(False)
                        n += 1
            _log0(f"[micro_engram] micro_engram_train_scales: false: {n} gate norm scales frozen"
                  + ("" if n else " (none: no scalar_sqrt gate in this run)"))
        self._place_engrams()
        self.dense = [p for s in self.slots for p in s.engram.parameters() if p.requires_grad]
        trained = [s.layer for s in self.slots if not s.frozen]
        self.first_trained = min(trained) if trained else None
        if self.first_trained is None:
            raise ValueError("every engram is frozen: nothing to train")
        self.base_conf = {
            "model_dim": text_cfg.hidden_size, "vocab_size": text_cfg.vocab_size,
            "canon_path": cfg.micro_engram_canon_path, "base_model": cfg.base_model,
            "base_fingerprint": _safe_fingerprint(cfg.base_model) if self.rank == 0 and cfg.base_init == "load" else None,
        }
        no_grad_upto = self.first_trained if cfg.no_grad_prefix else None
        M.checkpointing(model, self.text, cfg, no_grad_upto)
        model.train()

        from ..optim import LazyAdamW

        a = cfg
        self.dense_lr = a.micro_engram_dense_lr if a.micro_engram_dense_lr is not None else a.learning_rate
        self.dense_opt = LazyAdamW([{"params": self.dense, "lazy": False}], lr=self.dense_lr,
                                   betas=(a.adam_beta1, a.adam_beta2), eps=a.adam_epsilon, weight_decay=a.weight_decay,
                                   stochastic_rounding=a.micro_engram_stochastic_rounding is not False)
        opt = cfg.micro_engram_optimizer
        self.rows = RowTables([(f"{s.where}.micro_engram.", s.engram) for s in self.slots],
                              lr=a.learning_rate, betas=(a.adam_beta1, a.adam_beta2), eps=a.adam_epsilon,
                              weight_decay=a.weight_decay, lazy=opt in ("lazy_adam", "rowwise_adam"),
                              rowwise=opt == "rowwise_adam",
                              stochastic_rounding=a.micro_engram_stochastic_rounding is not False,
                              sparse_grads=bool(cfg.sparse_row_grads and opt in ("lazy_adam", "rowwise_adam")))
        if cfg.optimizer and not str(cfg.optimizer).startswith("adamw"):
            _log0(f"[micro_engram] optimizer: {cfg.optimizer} is not used; key/value/scales use AdamW")
        ropt = self.rows.optimizer if self.device.type == "cuda" else None
        host_moments = cfg.table_moments_on_host
        if ropt is not None:
            if host_moments is True:
                ropt.row_moments_on_host = True
            ropt.materialize_state()  # the tables' Adam state counts in memory planning
        if cfg.gradient_checkpointing and cfg.gradient_checkpointing_policy == "auto" and self.device.type == "cuda":
            self._plan_checkpointing(no_grad_upto)
            trained = sum(self.ckpt_plan.values())
            if ropt is not None and host_moments == "auto" and self.ckpt_plan["none"] < trained:
                # HBM is short of keeping every layer's activations: the table moments go to
                # pinned host memory (same decision on every rank: the plan is min over ranks)
                freed = ropt.move_row_moments_to_host()
                torch.cuda.empty_cache()
                _log0(f"[micro_engram] table optimizer moments -> pinned host memory ({freed / 2**30:.1f} GiB "
                      f"of HBM freed); re-planning")
                self._plan_checkpointing(no_grad_upto)
        self.table_moments_on_host = bool(ropt is not None and ropt.row_moments_on_host)
        self.total_steps = self._count_steps()
        self.scheduler = self._scheduler()
        self.offload = ActivationOffload(self.device) if (cfg.activation_offloading and self.device.type == "cuda") \
            else None
        self._report()

    def _plan_checkpointing(self, no_grad_upto):
        """HBM-budgeted checkpointing plan (gradient_checkpointing_policy: auto): the free memory
        after setup, minus headroom for one layer's backward working set, the loss chunks and
        the allocator, decides which layers keep what. Identical on every rank (min over ranks)."""
        torch.cuda.synchronize(self.device)
        free, total = torch.cuda.mem_get_info(self.device)
        cached = torch.cuda.memory_reserved(self.device) - torch.cuda.memory_allocated(self.device)
        reserve = float(self.cfg.gradient_checkpointing_reserve_gib) * 2 ** 30 + 0.04 * total
        budget = torch.tensor([float(free + cached - reserve)], device=self.device)
        if self.world > 1:
            dist.all_reduce(budget, op=dist.ReduceOp.MIN)
        tokens = self.cfg.micro_batch_size * self.cfg.sequence_len
        plan = self.text.plan_checkpointing(tokens, max(0.0, float(budget)), upto=no_grad_upto)
        counts = {m: sum(1 for v in plan.values() if v == m) for m in ("none", "selective", "full")}
        _log0(f"[micro_engram] activation checkpointing plan ({float(budget) / 2**30:.1f} GiB budget): "
              f"{counts['none']} layers keep everything, {counts['selective']} keep the attention half, "
              f"{counts['full']} keep only their input")
        self.ckpt_plan = counts

    def _place_engrams(self):
        """Dense engram params/buffers on this GPU, identical on every rank (rank 0's)."""
        for s in self.slots:
            e = s.engram
            e.to(self.device)
            if self.world > 1:
                for t in list(e.parameters()) + list(e.buffers()):
                    dist.broadcast(t.data, src=0)

    def _count_steps(self):
        cfg = self.cfg
        if cfg.max_steps:
            return int(cfg.max_steps)
        full, frac = int(math.floor(cfg.num_epochs)), cfg.num_epochs - math.floor(cfg.num_epochs)
        n = sum(self.plan.steps_per_epoch(e) for e in range(full))
        if frac > 0:
            n += int(self.plan.steps_per_epoch(full) * frac)
        if n <= 0:
            raise ValueError(f"no optimizer steps: {len(self.samples):,} samples pack into "
                             f"{len(self.plan.bins(0)):,} bins, fewer than one step needs ({self.plan.per_step})")
        return n

    def _scheduler(self):
        cfg = self.cfg
        warm = cfg.warmup_steps if cfg.warmup_steps is not None else (
            math.ceil(cfg.warmup_ratio * self.total_steps) if cfg.warmup_ratio else 0)
        self.warmup = warm
        if cfg.micro_engram_lr_epoch_decay:
            return epoch_step_scheduler(self.dense_opt, self.total_steps, warm, float(cfg.num_epochs),
                                        cfg.micro_engram_lr_epoch_decay)
        from transformers import get_scheduler

        name, kw = cfg.lr_scheduler, dict(cfg.lr_scheduler_kwargs or {})
        if name == "cosine" and cfg.cosine_min_lr_ratio is not None:
            name, kw = "cosine_with_min_lr", {**kw, "min_lr_rate": cfg.cosine_min_lr_ratio}
        if name == "constant":
            warm = 0
        return get_scheduler(name, self.dense_opt, num_warmup_steps=warm, num_training_steps=self.total_steps,
                             scheduler_specific_kwargs=kw or None)

    def _report(self):
        n_dense = sum(p.numel() for p in self.dense)
        n_rows = sum(p.numel() for p in self.rows.params() if p.requires_grad)
        n_base_train = sum(p.numel() for p in self.text.parameters() if p.requires_grad) - n_dense
        parts = [f"layer {s.layer}{' (frozen)' if s.frozen else ''}: "
                 f"{sum(p.numel() for p in s.engram.row_shards) / 1e6:.1f}M table params on this GPU, "
                 f"{sum(p.numel() for p in s.engram.parameters()) / 1e6:.1f}M dense" for s in self.slots]
        _log0(f"[micro_engram] trainable: engram only ({n_rows / 1e6:.1f}M table params on this GPU + "
              f"{n_dense / 1e6:.1f}M dense); base: frozen, {self.placement}; " + "; ".join(parts))
        if n_base_train:
            raise RuntimeError(f"{n_base_train} base parameters are trainable")
        _log0(f"[micro_engram] {len(self.samples):,} samples, {len(self.plan.bins(0)):,} bins of "
              f"{self.cfg.sequence_len} tokens, {self.plan.per_step} bins per step, {self.total_steps} steps; "
              f"no-grad prefix through layer {self.first_trained if self.cfg.no_grad_prefix else '-'}; "
              f"vocab rows {self.vocab.rows:,} of {self.vocab.V:,} on this GPU (loss chunk {self.vocab.chunk} tokens); "
              f"table gradients: {'sparse (touched rows only)' if self.rows.sparse else 'dense'}")
        if self.device.type == "cuda":
            _log0(f"[micro_engram] after setup: {torch.cuda.memory_allocated(self.device) / 2**30:.2f} GiB allocated "
                  f"on GPU {self.local}")

    # ------------------------------------------------------------------ one step
    def _micro_batch(self, bins):
        b = collate(self.samples, bins, self.cfg.sequence_len, self.pad_id, pin=self.device.type == "cuda")
        return {k: v.to(self.device, non_blocking=True) for k, v in b.items()}

    def forward_loss(self, batch, scale):
        """Sum of this GPU's token losses of one micro-batch; runs the backward of loss*scale."""
        ids, pos, labels = batch["input_ids"], batch["position_ids"], batch["labels"]
        ids, pos, labels = (t.reshape(1, -1) for t in (ids, pos, labels))  # one packed row
        self.ctx["ids"], self.ctx["pos"] = ids, pos
        emb = self.vocab.embed(ids)
        off = self.offload.context() if self.offload else _null()
        with off, M.grad_from_layer(self.text, self.first_trained, self.cfg.no_grad_prefix):
            h = self.text(emb, pos)
        h = h.reshape(-1, h.shape[-1])
        total, _ = self.vocab.loss_sum(h, labels.reshape(-1))
        (total * scale).backward()
        if self.offload:
            self.offload.end_step()
        self.ctx["ids"] = self.ctx["pos"] = None
        return total.detach()

    def train_step(self, micro, batches=None):
        """One optimizer step over the gradient_accumulation_steps micro-batches."""
        if batches is None:
            batches = [self._micro_batch(b) for b in micro]
        count = torch.stack([(b["labels"] != -100).sum() for b in batches]).sum().float()
        if self.world > 1:
            dist.all_reduce(count)
        count = count.clamp_min(1)
        scale = self.world / count
        loss = torch.zeros((), device=self.device)
        for b in batches:
            loss += self.forward_loss(b, scale)
        if self.world > 1:
            dist.all_reduce(loss)
            self._reduce_dense()
        dense_norm = torch.nn.utils.clip_grad_norm_(self.dense, self.cfg.max_grad_norm or float("inf"))
        table_norm = self.rows.clip(self.cfg.max_grad_norm)
        dense_lr = self.dense_opt.param_groups[0]["lr"]
        lr = self.cfg.learning_rate * self._lr_factor()
        self.dense_opt.step()
        self.rows.step(lr)
        self.dense_opt.zero_grad(set_to_none=True)
        self.scheduler.step()
        mean = float(loss / count)
        return {"loss": mean, "ppl": math.exp(min(mean, 50.0)), "grad_norm": float(dense_norm),
                "table_grad_norm": table_norm, "learning_rate": lr, "dense_lr": dense_lr, "tokens": int(count)}

    def _lr_factor(self):
        return self.scheduler.lr_lambdas[0](self.scheduler.last_epoch)

    def _reduce_dense(self):
        """Mean of the replicated dense parameters' gradients over ranks (fp32). CUDA with
        dense_allreduce: p2p: the fused peer-memory kernel over every dense parameter (a rank
        without a gradient contributes zeros; only existing gradients are overwritten);
        otherwise one flat NCCL all_reduce."""
        if (1 < self.world <= 16 and self.device.type == "cuda" and self.cfg.dense_allreduce == "p2p"
                and self.dense):  # one node: the kernel's peer table holds up to 16 ranks
            if getattr(self, "_p2p_ar", None) is None:
                from micro_engram_fork_b200.parallel.allreduce import P2PAllReduce

                self._p2p_ar = P2PAllReduce(sum(p.numel() for p in self.dense), self.device)
            flat = self._p2p_ar([p.grad if p.grad is not None else torch.zeros_like(p) for p in self.dense])
            k = 0
            for p in self.dense:
                n = p.numel()
                if p.grad is not None:
                    p.grad.copy_(flat[k:k + n].view_as(p.grad))
                k += n
            return
        grads = [p.grad for p in self.dense if p.grad is not None]
        if not grads:
            return
        flat = torch.cat([g.reshape(-1).float() for g in grads])
        dist.all_reduce(flat)
        flat /= self.world
        k = 0
        for g in grads:
            n = g.numel()
            g.copy_(flat[k:k + n].view_as(g))
            k += n

    # ------------------------------------------------------------------ loop
    def train(self):
        cfg = self.cfg
        self._maybe_resume()
        if self.rank == 0:
            os.makedirs(cfg.output_dir, exist_ok=True)
            write_config(build_config(self.base_conf, self.slots, lambda s: None), cfg.output_dir)
            self._init_wandb()
            try:
                from tqdm import tqdm

                self.pbar = tqdm(total=self.total_steps, initial=self.global_step, dynamic_ncols=True, unit="step",
                                 bar_format="{percentage:3.0f}%|{bar}| {n}/{total} [{elapsed}<{remaining}, "
                                            "{rate_inv_fmt}]")
            except ImportError:
                self.pbar = None
        t_last, toks = time.time(), 0
        snap = cfg.micro_engram_memory_snapshot
        if snap and self.device.type == "cuda":
            torch.cuda.memory._record_memory_history(max_entries=200_000)
        while self.global_step < self.total_steps:
            n_ep = self.plan.steps_per_epoch(self.epoch)
            if self.step_in_epoch >= n_ep:
                self.epoch, self.step_in_epoch = self.epoch + 1, 0
                continue
            if self.device.type == "cuda":
                torch.cuda.reset_peak_memory_stats(self.device)
            micro = self.plan.micro_batches(self.epoch, self.step_in_epoch, self.rank)
            if cfg.profile_step and self.global_step + 1 == cfg.profile_step:
                logs = self._profiled_step(micro)
            else:
                logs = self.train_step(micro)
            self.global_step += 1
            self.step_in_epoch += 1
            toks += logs.pop("tokens")
            if snap and self.device.type == "cuda" and self.global_step == snap:
                self._write_memory_snapshot()
            if self.pbar is not None:
                self.pbar.update(1)
                ppl = logs["ppl"]
                stats = f"loss {logs['loss']:.4f}  ppl {ppl:.0f}" if ppl >= 100 else \
                    f"loss {logs['loss']:.4f}  ppl {ppl:.2f}"
                self.pbar.bar_format = ("{percentage:3.0f}%|{bar}| {n}/{total} [{elapsed}<{remaining}, "
                                        "{rate_inv_fmt}]  " + stats)
                self.pbar.refresh()
            if self.global_step % cfg.logging_steps == 0 or self.global_step == self.total_steps:
                dt = time.time() - t_last
                for slot in self.slots:  # a row-store kernel error (bounds, capacity, timeout) stops the run
                    store = slot.engram.__dict__.get("row_store")
                    if store is not None:
                        store.check_status()
                if getattr(self, "_p2p_ar", None) is not None:
                    self._p2p_ar.check_status()
                logs.update(self._memory())
                logs.update(self._engram_logs())
                logs.update({"epoch": round(self.epoch + self.step_in_epoch / max(1, n_ep), 4),
                             "step": self.global_step, "s_per_step": round(dt / cfg.logging_steps, 2),
                             "trained_tokens_per_s": round(toks / max(dt, 1e-9), 1)})
                self._log(logs)
                t_last, toks = time.time(), 0
            if cfg.save_steps and self.global_step % cfg.save_steps == 0:
                self.save_checkpoint()
        if self.pbar is not None:
            self.pbar.close()
            self.pbar = None
        if not cfg.save_steps or self.global_step % cfg.save_steps:
            self.save_checkpoint()
        self.rows.save(os.path.join(cfg.output_dir, ROWS_DIR))
        if self.rank == 0:
            write_config(build_config(self.base_conf, self.slots, lambda s: ROWS_DIR), cfg.output_dir)
            _log0(f"[micro_engram] done: {cfg.output_dir}/{ROWS_DIR} holds the engram; serve it with "
                  f"--additional-config '{{\"micro_engram\": \"{cfg.output_dir}/{CONFIG_NAME}\"}}'")
            if self.wandb:
                self.wandb.finish()

    def _write_memory_snapshot(self):
        folder = os.path.join(self.cfg.output_dir, "memory_snapshot")
        os.makedirs(folder, exist_ok=True)
        path = os.path.join(folder, f"rank{self.rank}_step{self.global_step}.pickle")
        try:
            torch.cuda.memory._dump_snapshot(path)
            LOG.warning(f"[micro_engram] memory snapshot written: {path}")
        finally:
            torch.cuda.memory._record_memory_history(enabled=None)

    def _profiled_step(self, micro):
        """One step under torch.profiler; rank 0 writes profile/rank0_step<N>.{json,txt}."""
        from torch.profiler import ProfilerActivity, profile

        acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if self.device.type == "cuda" else [])
        with profile(activities=acts, record_shapes=False) as prof:
            logs = self.train_step(micro)
            if self.device.type == "cuda":
                torch.cuda.synchronize(self.device)
        if self.rank == 0:
            folder = os.path.join(self.cfg.output_dir, "profile")
            os.makedirs(folder, exist_ok=True)
            base = os.path.join(folder, f"rank0_step{self.global_step + 1}")
            try:
                prof.export_chrome_trace(base + ".json")
                key = "cuda_time_total" if self.device.type == "cuda" else "cpu_time_total"
                with open(base + ".txt", "w") as f:
                    f.write(prof.key_averages().table(sort_by=key, row_limit=40))
                LOG.warning(f"[micro_engram] profile written: {base}.txt (top kernels), {base}.json (timeline)")
            except Exception as e:  # noqa: BLE001
                LOG.warning(f"[micro_engram] writing the profile failed (training continues): {e}")
        return logs

    def _memory(self):
        if self.device.type != "cuda":
            return {}
        m = torch.tensor([torch.cuda.max_memory_allocated(self.device), torch.cuda.max_memory_reserved(self.device)],
                         dtype=torch.float64, device=self.device) / 2**30
        allm = [torch.zeros_like(m) for _ in range(self.world)]
        if self.world > 1:
            dist.all_gather(allm, m)
        else:
            allm = [m]
        allm = torch.stack(allm)
        return {"mem_peak_alloc_gib": round(float(allm[:, 0].max()), 2),
                "mem_peak_reserved_gib": round(float(allm[:, 1].max()), 2),
                "mem_peak_alloc_per_gpu": [round(float(x), 2) for x in allm[:, 0]]}

    def _engram_logs(self):
        out = {}
        every = self.cfg.micro_engram_stats_steps
        gates = [s.engram.pop_gate_stats() for s in self.slots]
        if self.rank != 0 or not every or self.global_step % every:
            return out
        for s, gate in zip(self.slots, gates):
            if s.frozen:
                continue
            try:
                st = module_stats(s.engram)
                if gate is not None:
                    st["engram/gate_mean"], st["engram/gate_saturated"] = gate
            except Exception as e:  # noqa: BLE001
                LOG.warning(f"[micro_engram] stats failed: {e}")
                continue
            if len(self.slots) > 1:
                st = {k.replace("engram/", f"engram_L{s.layer}/", 1): v for k, v in st.items()}
            out.update(st)
        return out

    def _log(self, logs):
        if self.rank != 0:
            return
        line = json.dumps({k: (round(v, 6) if isinstance(v, float) else v) for k, v in logs.items()})
        if self.pbar is not None:
            self.pbar.write(line)
        else:
            print(line, flush=True)
        with open(os.path.join(self.cfg.output_dir, "train_log.jsonl"), "a") as f:
            f.write(line + "\n")
        if self.wandb:
            self.wandb.log({k: v for k, v in logs.items() if isinstance(v, (int, float))}, step=self.global_step)

    def _init_wandb(self):
        cfg = self.cfg
        if not cfg.wandb_project or cfg.wandb_mode == "disabled":
            return
        import wandb

        self.wandb = wandb
        wandb.init(project=cfg.wandb_project, name=cfg.wandb_name, entity=cfg.wandb_entity, mode=cfg.wandb_mode,
                   config=cfg.model_dump(), resume="allow")

    # ------------------------------------------------------------------ checkpoints
    def save_checkpoint(self):
        cfg = self.cfg
        folder = os.path.join(cfg.output_dir, f"checkpoint-{self.global_step}")
        self.rows.save(os.path.join(folder, ROWS_DIR), os.path.join(folder, ROWS_OPTIM_DIR))
        if self.rank == 0:
            os.makedirs(folder, exist_ok=True)
            torch.save({"dense_optimizer": self.dense_opt.state_dict(), "scheduler": self.scheduler.state_dict(),
                        "rng": torch.get_rng_state()}, os.path.join(folder, DENSE_FILE))
            write_config(build_config(self.base_conf, self.slots, lambda s: ROWS_DIR), folder)
            write_config(build_config(self.base_conf, self.slots,
                                      lambda s: f"checkpoint-{self.global_step}/{ROWS_DIR}"), cfg.output_dir)
            with open(os.path.join(folder, STATE_FILE), "w") as f:  # last: marks the checkpoint complete
                json.dump({"global_step": self.global_step, "epoch": self.epoch, "step_in_epoch": self.step_in_epoch,
                           "total_steps": self.total_steps, "trainer": "micro_engram.train"}, f, indent=2)
            self._rotate()
        if self.world > 1:
            dist.barrier()
        _log0(f"[micro_engram] saved {folder}")

    def _rotate(self):
        limit = self.cfg.save_total_limit
        if not limit:
            return
        import glob
        import re

        done = sorted((int(m.group(1)), c) for c in glob.glob(os.path.join(self.cfg.output_dir, "checkpoint-*"))
                      if (m := re.search(r"checkpoint-(\d+)$", c)) and os.path.isfile(os.path.join(c, STATE_FILE)))
        for _, c in done[:-limit]:
            shutil.rmtree(c, ignore_errors=True)

    def _maybe_resume(self):
        from ..weights import latest_checkpoint

        cfg = self.cfg
        ckpt = cfg.resume_from_checkpoint
        if ckpt is None and cfg.auto_resume_from_checkpoints and os.path.isdir(cfg.output_dir):
            ckpt = latest_checkpoint(cfg.output_dir)
        if not ckpt:
            return
        with open(os.path.join(ckpt, STATE_FILE)) as f:
            st = json.load(f)
        if st.get("trainer") != "micro_engram.train":
            raise ValueError(f"{ckpt} was written by another trainer (Axolotl?): start from it with "
                             f"micro_engram_init_from instead of resuming")
        n, opt = self.rows.load(os.path.join(ckpt, ROWS_DIR), os.path.join(ckpt, ROWS_OPTIM_DIR))
        self._load_dense(os.path.join(ckpt, ROWS_DIR))
        blob = torch.load(os.path.join(ckpt, DENSE_FILE), map_location="cpu", weights_only=False)
        self.dense_opt.load_state_dict(blob["dense_optimizer"])
        self.scheduler.load_state_dict(blob["scheduler"])
        self.scheduler.base_lrs = [self.dense_lr]
        for g in self.dense_opt.param_groups:
            g["initial_lr"] = self.dense_lr
            g["lr"] = self.dense_lr * self._lr_factor()
        self.global_step, self.epoch, self.step_in_epoch = st["global_step"], st["epoch"], st["step_in_epoch"]
        if st.get("total_steps") not in (None, self.total_steps):
            _log0(f"[micro_engram] resume: the run now has {self.total_steps} steps (checkpoint said "
                  f"{st['total_steps']}); the LR schedule follows the new count")
        _log0(f"[micro_engram] resumed from {ckpt}: step {self.global_step}, epoch {self.epoch} "
              f"(+{self.step_in_epoch} steps), {n} tables" + ("" if opt else ", NO table optimizer state"))

    def _load_dense(self, folder):
        from ..weights import load_engram_weights

        for s in self.slots:
            if s.frozen:
                continue
            sd = {k: v for k, v in load_engram_weights(folder, layer=s.layer).items() if not k.startswith("tables.")}
            tables_missing = {f"tables.{k}.weight" for k in range(len(s.engram.row_shards))}
            res = s.engram.load_state_dict(sd, strict=False)
            bad = [k for k in res.missing_keys if k not in tables_missing and k != "mults"] + list(res.unexpected_keys)
            if bad:
                raise ValueError(f"[micro_engram] resume: engram at layer {s.layer} does not match {folder}: {bad[:10]}")


def main(argv=None):
    import argparse

    from .config import load_config

    ap = argparse.ArgumentParser(description="Train micro_engram on a frozen base (torchrun -m micro_engram.train cfg.yaml)")
    ap.add_argument("config")
    args = ap.parse_args(argv)
    logging.basicConfig(level=logging.WARNING, format="%(asctime)s %(message)s")
    if os.environ.get("RANK", "0") != "0":
        logging.getLogger("micro_engram").setLevel(logging.ERROR)
    cfg = load_config(args.config)
    t = Trainer(cfg)
    try:
        t.build()
        t.train()
    except BaseException:
        # fail fast: print now and exit hard, so torchrun stops the other ranks instead of
        # leaving them waiting in a collective this rank never reaches
        import sys
        import traceback

        rank = os.environ.get("RANK", "?")
        print(f"\n[micro_engram] rank {rank} FAILED:", file=sys.stderr, flush=True)
        traceback.print_exc()
        sys.stderr.flush()
        if torch.cuda.is_available():
            dev = torch.cuda.current_device()
            print(f"[micro_engram] rank {rank}: {torch.cuda.memory_allocated(dev) / 2**30:.2f} GiB allocated, "
                  f"{torch.cuda.memory_reserved(dev) / 2**30:.2f} GiB reserved", file=sys.stderr, flush=True)
        os._exit(1)
    if dist.is_initialized():
        dist.destroy_process_group()
