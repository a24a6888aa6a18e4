"""micro_engram.train: stage-1 engram training over a frozen Gemma-style base, one process per
GPU (torchrun), PyTorch for the plumbing and the sm_100a kernels for the work.

Where things live on each GPU:
  base model      the frozen decoder (micro_engram_fork_b200.models.gemma): replicated when it
                  fits in HBM, or row-sharded with the layer all-gather folded into the tcgen05
                  GEMMs (base_placement: sharded); per-layer activation checkpointing planned
                  against free HBM, optional offload of checkpointed layer inputs to pinned memory
  embedding/head  vocab rows split over the GPUs (head.VocabShard): peer-read embedding and the
                  fused chunked softcapped loss
  engram tables   row-sharded in peer-mapped row stores (rows.RowTables): fused fetch, row
                  gradients pushed to their owners, touched-row Adam with stochastic rounding
  engram dense    key / value / gate weights replicated; gradients averaged by the P2P kernel

The behaviour users rely on is the reference trainer's (Ready-Art/micro_engram_fork,
micro_engram/train/loop.py:1-595): YAML keys, per-token mean loss over all micro-batches and
ranks, global-norm clipping of the dense part and of the tables, LR schedules, JSONL log keys,
the checkpoint layout (train/checkpoint.py), rotation, resuming at another GPU count,
profile_step and fail-fast exit. The organisation is this framework's own: setup in stages,
the step returns device tensors (the host reads them at logging steps only), checkpoints,
reporting, timing and fault handling are separate components.
"""
import logging
import math
import os

import torch
import torch.distributed as dist

from micro_engram_fork_b200.utils.timers import PhaseTimers

from ..rows import ROWS_DIR, RowTables, _group, dist_rank_world
from ..runconfig import (CONFIG_NAME, build_config, build_slot, check_canon, engram_params, engram_requests,
                         epoch_step_scheduler, fingerprint_or_none, write_config)
from . import model as M
from .checkpoint import Checkpoints
from .data import EpochPlan, collate, prepare
from .faults import FaultHook
from .offload import ActivationOffload
from .report import Reporter, to_host

LOG = logging.getLogger("micro_engram.train")
LAZY_OPTIMIZERS = ("lazy_adam", "rowwise_adam")


def setup_dist(timeout_s=None):
    """(rank, world, local rank, device) with the process group up: NCCL on GPUs, gloo on CPU.
    A world-1 run without a launcher gets a loopback rendezvous. The group's timeout
    (MICRO_ENGRAM_PG_TIMEOUT_S) bounds how long survivors wait on a rank that died."""
    rank, world = dist_rank_world()
    if world == 1 and "MASTER_ADDR" not in os.environ:
        import socket

        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            os.environ.setdefault("MASTER_PORT", str(s.getsockname()[1]))
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    local = int(os.environ.get("LOCAL_RANK", 0))
    on_gpu = torch.cuda.is_available() and os.environ.get("MICRO_ENGRAM_CPU") != "1"
    device = torch.device("cuda", local) if on_gpu else torch.device("cpu")
    if on_gpu:
        torch.cuda.set_device(local)
    if not dist.is_initialized():
        import datetime

        kw = {"device_id": device} if on_gpu else {}
        timeout_s = timeout_s or float(os.environ.get("MICRO_ENGRAM_PG_TIMEOUT_S", "0") or 0)
        if timeout_s:
            kw["timeout"] = datetime.timedelta(seconds=timeout_s)
        dist.init_process_group("nccl" if on_gpu else "gloo", rank=rank, world_size=world, **kw)
    return rank, world, local, device


class Trainer:
    def __init__(self, cfg):
        self.cfg = cfg
        self.rank, self.world, self.local, self.device = setup_dist()
        self.ctx = {"ids": None, "pos": None}   # the micro-batch's ids/positions, read by the engram hooks
        self.global_step = self.epoch = self.step_in_epoch = 0
        self.timers = PhaseTimers(enabled=os.environ.get("MICRO_ENGRAM_PHASE_TIMES") == "1", device=self.device)
        self.faults = FaultHook(self.rank)
        self.checkpoints = Checkpoints(self)
        self.reporter = Reporter(self)
        self._p2p_ar = None
        if cfg.kernels == "reference":
            os.environ["MICRO_ENGRAM_REFERENCE_OPS"] = "1"
        if cfg.tf32 and self.device.type == "cuda":
            torch.backends.cuda.matmul.allow_tf32 = torch.backends.cudnn.allow_tf32 = True

    def log0(self, msg):
        if self.rank == 0:
            LOG.warning(msg)

    # ================================================================== setup
    def build(self, samples=None, tokenizer=None):
        """Data, base, engrams, optimizers, memory plan and schedule. `samples` / `tokenizer`
        may be handed in directly (synthetic data)."""
        torch.manual_seed(self.cfg.seed)
        self._setup_data(samples, tokenizer)
        self._setup_base()
        self._setup_engrams()
        self._setup_optimizers()
        self._setup_memory()
        self.total_steps = self._count_steps()
        self.scheduler = self._make_scheduler()
        self.offload = (ActivationOffload(self.device)
                        if self.cfg.activation_offloading and self.device.type == "cuda" else None)
        self._describe()

    def _setup_data(self, samples, tokenizer):
        cfg = self.cfg
        if samples is None:
            from transformers import AutoTokenizer

            path = cfg.tokenizer_config or cfg.base_model
            tokenizer = AutoTokenizer.from_pretrained(path)
            samples = prepare(cfg, tokenizer, path, rank=self.rank, barrier=dist.barrier if self.world > 1 else None)
        self.tokenizer, self.samples = tokenizer, samples
        self.plan = EpochPlan(samples, cfg, self.world)
        pad = getattr(tokenizer, "pad_token_id", None) if tokenizer is not None else None
        self.pad_id = 0 if pad is None else pad

    def _setup_base(self):
        cfg = self.cfg
        M.apply_kernel_patches(cfg, self.device.type == "cuda")
        self.model, _ = M.load_base(cfg, self.rank, self.local, self.device)
        self.text_name, self.text = M.text_model(self.model)
        self.placement = M.place_base(self.text, cfg, self.device, self.world)
        self.vocab = M.take_vocab(self.model, self.text, self.rank, self.world, self.device,
                                  chunk_tokens=cfg.loss_chunk_tokens)

    def _canon(self, vocab_size):
        path = self.cfg.micro_engram_canon_path
        if not path:
            return None
        canon = check_canon(torch.load(path, map_location="cpu"), vocab_size)
        self.log0(f"[micro_engram] token merging: {canon.numel():,} ids -> "
                  f"{int(torch.unique(canon).numel()):,} classes ({path})")
        return canon

    def _setup_engrams(self):
        cfg, text_cfg = self.cfg, self.text.config
        canon = self._canon(text_cfg.vocab_size)
        # one optimizer step looks up at most (bins per step, all ranks) x sequence_len rows per
        # table on any rank: the capacity of the row stores' compact gradient accumulators
        capacity = self.plan.per_step * cfg.sequence_len
        self.slots = []
        for req in engram_requests(cfg):
            req.spec["canon_path"] = cfg.micro_engram_canon_path
            self.slots.append(build_slot(req, self.model, text_cfg, canon, dtype=cfg.micro_engram_dtype,
                                         sharding="rows", get_ids=lambda: (self.ctx["ids"], self.ctx["pos"]),
                                         device=self.device, group=_group(self.world), row_capacity=capacity))
        for slot in self.slots:
            if slot.frozen:
                for p in engram_params(slot.engram):
                    p.requires_grad_(False)
        if not cfg.micro_engram_train_scales:
            frozen = [p for s in self.slots for n in getattr(s.engram, "DELTA_SCALES", ())
                      for p in [getattr(s.engram, n, None)] if isinstance(p, torch.nn.Parameter) and p.requires_grad]
            for p in frozen:
                p.requires_grad_(False)
            self.log0(f"[micro_engram] micro_engram_train_scales: false -> {len(frozen)} gate norm scales frozen"
                      + ("" if frozen else " (no scalar_sqrt gate in this run)"))
        for slot in self.slots:  # dense engram weights: this GPU, the same on every rank (rank 0's)
            slot.engram.to(self.device)
            if self.world > 1:
                for t in list(slot.engram.parameters()) + list(slot.engram.buffers()):
                    dist.broadcast(t.data, src=0)
        self.dense = [p for s in self.slots for p in s.engram.parameters() if p.requires_grad]
        trained = [s.layer for s in self.slots if not s.frozen]
        if not trained:
            raise ValueError("every engram is frozen: nothing to train")
        self.first_trained = min(trained)
        load_fp = self.rank == 0 and cfg.base_init == "load"
        self.base_conf = {"model_dim": text_cfg.hidden_size, "vocab_size": text_cfg.vocab_size,
                          "canon_path": cfg.micro_engram_canon_path, "base_model": cfg.base_model,
                          "base_fingerprint": fingerprint_or_none(cfg.base_model) if load_fp else None}
        self.no_grad_upto = self.first_trained if cfg.no_grad_prefix else None
        M.checkpointing(self.model, self.text, cfg, self.no_grad_upto)
        self.model.train()

    def _setup_optimizers(self):
        from ..optim import LazyAdamW

        cfg = self.cfg
        betas = (cfg.adam_beta1, cfg.adam_beta2)
        sr = cfg.micro_engram_stochastic_rounding is not False
        self.dense_lr = cfg.micro_engram_dense_lr if cfg.micro_engram_dense_lr is not None else cfg.learning_rate
        self.dense_opt = LazyAdamW([{"params": self.dense, "lazy": False}], lr=self.dense_lr, betas=betas,
                                   eps=cfg.adam_epsilon, weight_decay=cfg.weight_decay, stochastic_rounding=sr)
        lazy = cfg.micro_engram_optimizer in LAZY_OPTIMIZERS
        self.rows = RowTables([(f"{s.where}.micro_engram.", s.engram) for s in self.slots], lr=cfg.learning_rate,
                              betas=betas, eps=cfg.adam_epsilon, weight_decay=cfg.weight_decay, lazy=lazy,
                              rowwise=cfg.micro_engram_optimizer == "rowwise_adam", stochastic_rounding=sr,
                              sparse_grads=bool(cfg.sparse_row_grads and lazy))
        if cfg.optimizer and not str(cfg.optimizer).startswith("adamw"):
            self.log0(f"[micro_engram] optimizer: {cfg.optimizer} is not used; the dense engram weights use AdamW")

    def _setup_memory(self):
        """Table moments to host memory when asked (or when HBM is short), and the HBM-budgeted
        activation checkpointing plan."""
        cfg = self.cfg
        ropt = self.rows.optimizer if self.device.type == "cuda" else None
        if ropt is not None:
            if cfg.table_moments_on_host is True:
                ropt.row_moments_on_host = True
            ropt.materialize_state()  # the tables' Adam state counts in the plan
        self.ckpt_plan = None
        if cfg.gradient_checkpointing and cfg.gradient_checkpointing_policy == "auto" and self.device.type == "cuda":
            self._plan_checkpointing()
            if ropt is not None and cfg.table_moments_on_host == "auto" and self.ckpt_plan["none"] < sum(
                    self.ckpt_plan.values()):
                # not every layer keeps its activations: free HBM by moving the table moments to
                # pinned host memory (the plan is the min over ranks, so every rank agrees)
                freed = ropt.move_row_moments_to_host()
                torch.cuda.empty_cache()
                self.log0(f"[micro_engram] table optimizer moments -> pinned host memory ({freed / 2 ** 30:.1f} GiB "
                          "of HBM); re-planning")
                self._plan_checkpointing()
        self.table_moments_on_host = bool(ropt is not None and ropt.row_moments_on_host)

    def _plan_checkpointing(self):
        """Free HBM after setup, less a reserve for the backward's working set, the loss chunks
        and the allocator, decides what each layer keeps (the same plan on every rank)."""
        torch.cuda.synchronize(self.device)
        free, total = torch.cuda.mem_get_info(self.device)
        cached = torch.cuda.memory_reserved(self.device) - torch.cuda.memory_allocated(self.device)
        reserve = float(self.cfg.gradient_checkpointing_reserve_gib) * 2 ** 30 + 0.04 * total
        budget = torch.tensor([float(free + cached - reserve)], device=self.device)
        if self.world > 1:
            dist.all_reduce(budget, op=dist.ReduceOp.MIN)
        tokens = self.cfg.micro_batch_size * self.cfg.sequence_len
        plan = self.text.plan_checkpointing(tokens, max(0.0, float(budget)), upto=self.no_grad_upto)
        self.ckpt_plan = {m: sum(1 for v in plan.values() if v == m) for m in ("none", "selective", "full")}
        self.log0(f"[micro_engram] activation checkpointing plan ({float(budget) / 2 ** 30:.1f} GiB): "
                  f"{self.ckpt_plan['none']} layers keep everything, {self.ckpt_plan['selective']} keep the "
                  f"attention half, {self.ckpt_plan['full']} keep only their input")

    def _count_steps(self):
        cfg = self.cfg
        if cfg.max_steps:
            return int(cfg.max_steps)
        whole = int(math.floor(cfg.num_epochs))
        steps = sum(self.plan.steps_per_epoch(e) for e in range(whole))
        part = cfg.num_epochs - whole
        if part > 0:
            steps += int(self.plan.steps_per_epoch(whole) * part)
        if steps <= 0:
            raise ValueError(f"no optimizer steps: {len(self.samples):,} samples pack into "
                             f"{len(self.plan.bins(0)):,} bins, fewer than one step needs ({self.plan.per_step})")
        return steps

    def _make_scheduler(self):
        cfg = self.cfg
        if cfg.warmup_steps is not None:
            warm = cfg.warmup_steps
        else:
            warm = math.ceil(cfg.warmup_ratio * self.total_steps) if cfg.warmup_ratio else 0
        self.warmup = warm
        if cfg.micro_engram_lr_epoch_decay:
            return epoch_step_scheduler(self.dense_opt, self.total_steps, warm, float(cfg.num_epochs),
                                        cfg.micro_engram_lr_epoch_decay)
        from transformers import get_scheduler

        name, kwargs = cfg.lr_scheduler, dict(cfg.lr_scheduler_kwargs or {})
        if name == "cosine" and cfg.cosine_min_lr_ratio is not None:
            name, kwargs = "cosine_with_min_lr", {**kwargs, "min_lr_rate": cfg.cosine_min_lr_ratio}
        return get_scheduler(name, self.dense_opt, num_warmup_steps=0 if name == "constant" else warm,
                             num_training_steps=self.total_steps, scheduler_specific_kwargs=kwargs or None)

    def _describe(self):
        n_dense = sum(p.numel() for p in self.dense)
        n_rows = sum(p.numel() for p in self.rows.params() if p.requires_grad)
        stray = sum(p.numel() for p in self.text.parameters() if p.requires_grad) - n_dense
        if stray:
            raise RuntimeError(f"{stray} base parameters are trainable")
        per = "; ".join(f"layer {s.layer}{' (frozen)' if s.frozen else ''}: "
                        f"{sum(p.numel() for p in s.engram.row_shards) / 1e6:.1f}M table params on this GPU, "
                        f"{sum(p.numel() for p in s.engram.parameters()) / 1e6:.1f}M dense" for s in self.slots)
        self.log0(f"[micro_engram] trainable: engram only ({n_rows / 1e6:.1f}M table params on this GPU + "
                  f"{n_dense / 1e6:.1f}M dense); base: frozen, {self.placement}; {per}")
        self.log0(f"[micro_engram] {len(self.samples):,} samples, {len(self.plan.bins(0)):,} bins of "
                  f"{self.cfg.sequence_len} tokens, {self.plan.per_step} bins per step, {self.total_steps} steps; "
                  f"no-grad prefix through layer {self.first_trained if self.cfg.no_grad_prefix else '-'}; "
                  f"vocab rows {self.vocab.rows:,} of {self.vocab.V:,} on this GPU (loss chunk {self.vocab.chunk} "
                  f"tokens); table gradients: {'sparse (touched rows only)' if self.rows.sparse else 'dense'}")
        if self.device.type == "cuda":
            self.log0(f"[micro_engram] after setup: {torch.cuda.memory_allocated(self.device) / 2 ** 30:.2f} GiB "
                      f"allocated on GPU {self.local}")

    # ================================================================== one step
    def _micro_batch(self, bins):
        batch = collate(self.samples, bins, self.cfg.sequence_len, self.pad_id, pin=self.device.type == "cuda")
        return {k: v.to(self.device, non_blocking=True) for k, v in batch.items()}

    def forward_loss(self, batch, scale):
        """Sum of this GPU's token losses of one micro-batch (a device scalar); runs the
        backward of loss * scale."""
        ids, pos, labels = (batch[k].reshape(1, -1) for k in ("input_ids", "position_ids", "labels"))  # one row
        self.ctx["ids"], self.ctx["pos"] = ids, pos
        with self.timers.phase("embed"):
            emb = self.vocab.embed(ids)
        offload = self.offload.context() if self.offload else _Nothing()
        with self.timers.phase("forward"), offload, M.grad_from_layer(self.text, self.first_trained,
                                                                      self.cfg.no_grad_prefix):
            h = self.text(emb, pos)
        with self.timers.phase("loss"):
            total, _ = self.vocab.loss_sum(h.reshape(-1, h.shape[-1]), labels.reshape(-1))
        with self.timers.phase("backward"):
            (total * scale).backward()
        if self.offload:
            self.offload.end_step()
        self.ctx["ids"] = self.ctx["pos"] = None
        return total.detach()

    def train_step(self, micro, batches=None, sync=True):
        """One optimizer step over the gradient_accumulation_steps micro-batches `micro` (bin
        lists) or their already collated device `batches`. Returns the step's logs: Python
        numbers with sync (the public API), device tensors without (the training loop, which
        reads them at logging steps only)."""
        if batches is None:
            batches = [self._micro_batch(b) for b in micro]
        tokens = torch.stack([(b["labels"] != -100).sum() for b in batches]).sum()
        if self.world > 1:
            dist.all_reduce(tokens)
        count = tokens.clamp_min(1).float()
        scale = self.world / count   # per-token mean over every micro-batch and rank (loss * world / N)
        loss = torch.zeros((), device=self.device)
        for b in batches:
            loss += self.forward_loss(b, scale)
        with self.timers.phase("reduce"):
            if self.world > 1:
                dist.all_reduce(loss)
                self._reduce_dense()
        with self.timers.phase("optimizer"):
            dense_norm = torch.nn.utils.clip_grad_norm_(self.dense, self.cfg.max_grad_norm or float("inf"))
            table_norm = self.rows.clip(self.cfg.max_grad_norm)
            lr = self.cfg.learning_rate * self.lr_factor()
            dense_lr = self.dense_opt.param_groups[0]["lr"]
            self.dense_opt.step()
            self.rows.step(lr)
            self.dense_opt.zero_grad(set_to_none=True)
            self.scheduler.step()
        logs = {"loss": loss / count, "grad_norm": dense_norm, "learning_rate": lr, "dense_lr": dense_lr,
                "tokens": tokens}
        if table_norm is not None:
            logs["table_grad_norm"] = table_norm
        return to_host(logs) if sync else logs

    def lr_factor(self):
        return self.scheduler.lr_lambdas[0](self.scheduler.last_epoch)

    _lr_factor = lr_factor

    def _reduce_dense(self):
        """Average the replicated dense engram gradients over ranks in fp32: the fused P2P
        kernel over peer memory on CUDA (dense_allreduce: p2p; one node, up to 16 ranks), else
        one flat NCCL / gloo all_reduce."""
        if not self.dense:
            return
        if self.device.type == "cuda" and self.cfg.dense_allreduce == "p2p" and 1 < self.world <= 16:
            if self._p2p_ar is None:
                from micro_engram_fork_b200.parallel.allreduce import P2PAllReduce

                self._p2p_ar = P2PAllReduce(sum(p.numel() for p in self.dense), self.device)
            # every rank contributes every parameter (zeros where it has no gradient)
            mean = self._p2p_ar([p.grad if p.grad is not None else torch.zeros_like(p) for p in self.dense])
            offset = 0
            for p in self.dense:
                if p.grad is not None:
                    p.grad.copy_(mean[offset:offset + p.numel()].view_as(p.grad))
                offset += p.numel()
            return
        grads = [p.grad for p in self.dense if p.grad is not None]
        if grads:
            flat = torch.cat([g.reshape(-1).float() for g in grads])
            dist.all_reduce(flat)
            flat /= self.world
            for g, part in zip(grads, flat.split([g.numel() for g in grads])):
                g.copy_(part.view_as(g))

    # ================================================================== the run
    def _publish_config(self, rows_dir):
        """Rank 0 writes the run's engram config into output_dir: with no weights while the run
        trains, pointing at the saved row folder once it is done."""
        if self.rank != 0:
            return
        os.makedirs(self.cfg.output_dir, exist_ok=True)
        write_config(build_config(self.base_conf, self.slots, lambda _slot: rows_dir), self.cfg.output_dir)

    def train(self):
        cfg = self.cfg
        self._maybe_resume()
        self._publish_config(None)
        self.reporter.open()
        snapshot_at = cfg.micro_engram_memory_snapshot
        if snapshot_at and self.device.type == "cuda":
            torch.cuda.memory._record_memory_history(max_entries=200_000)
        while self.global_step < self.total_steps:
            in_epoch = self.plan.steps_per_epoch(self.epoch)
            if self.step_in_epoch >= in_epoch:
                self.epoch, self.step_in_epoch = self.epoch + 1, 0
                continue
            self.faults.before_step(self.global_step + 1)
            if self.device.type == "cuda":
                torch.cuda.reset_peak_memory_stats(self.device)
            micro = self.plan.micro_batches(self.epoch, self.step_in_epoch, self.rank)
            if cfg.profile_step and self.global_step + 1 == cfg.profile_step:
                logs = self.reporter.profiled(lambda: self.train_step(micro, sync=False))
            else:
                logs = self.train_step(micro, sync=False)
            self.global_step += 1
            self.step_in_epoch += 1
            if snapshot_at and self.device.type == "cuda" and self.global_step == snapshot_at:
                self.reporter.memory_snapshot()
            self.reporter.step_done(logs, in_epoch)
            if cfg.save_steps and self.global_step % cfg.save_steps == 0:
                self.save_checkpoint()
        self.reporter.close()
        if not cfg.save_steps or self.global_step % cfg.save_steps:
            self.save_checkpoint()
        self.rows.save(os.path.join(cfg.output_dir, ROWS_DIR))
        self._publish_config(ROWS_DIR)
        if self.rank == 0:
            self.log0(f"[micro_engram] done: {cfg.output_dir}/{ROWS_DIR} holds the engram; serve it with "
                      f"--additional-config '{{\"micro_engram\": \"{cfg.output_dir}/{CONFIG_NAME}\"}}'")

    def save_checkpoint(self):
        folder = self.checkpoints.save()
        self.log0(f"[micro_engram] saved {folder}")
        return folder

    def _maybe_resume(self):
        return self.checkpoints.resume()


class _Nothing:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


def _fail_fast():
    """Print this rank's failure and leave at once (exit 1): torchrun then stops the other ranks,
    and ranks already waiting in a collective get a closed connection or the group's timeout
    instead of waiting on a rank that will never arrive."""
    import sys
    import traceback

    who = f"[micro_engram] rank {os.environ.get('RANK', '?')}"
    lines = [f"\n{who} FAILED:\n{traceback.format_exc()}"]
    if torch.cuda.is_available() and torch.cuda.is_initialized():
        dev = torch.cuda.current_device()
        gib = [torch.cuda.memory_allocated(dev) / 2 ** 30, torch.cuda.memory_reserved(dev) / 2 ** 30]
        lines.append(f"{who}: {gib[0]:.2f} GiB allocated, {gib[1]:.2f} GiB reserved\n")
    sys.stderr.write("".join(lines))
    sys.stderr.flush()
    os._exit(1)


def main(argv=None):
    import argparse

    from .config import load_config

    parser = argparse.ArgumentParser(description="Train a micro_engram on a frozen base "
                                                 "(torchrun --nproc-per-node N -m micro_engram.train cfg.yaml)")
    parser.add_argument("config")
    args = parser.parse_args(argv)
    logging.basicConfig(level=logging.WARNING, format="%(asctime)s %(message)s")
    if os.environ.get("RANK", "0") != "0":
        logging.getLogger("micro_engram").setLevel(logging.ERROR)
    try:
        trainer = Trainer(load_config(args.config))
        trainer.build()
        trainer.train()
    except BaseException:  # noqa: BLE001
        _fail_fast()
    if dist.is_initialized():
        dist.destroy_process_group()
