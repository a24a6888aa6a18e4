"""Checkpoints of micro_engram.train: writing, rotation and resuming.

Layout of output_dir/checkpoint-<step>/ (the reference trainer's, so runs resume across the
two frameworks' tools; Ready-Art/micro_engram_fork micro_engram/train/loop.py:436-534):
  micro_engram_rows/         DCP: every trained engram (tables as Shard(0) DTensors of the whole
                             table, so a run resumes at any GPU count; dense weights; buffers)
  micro_engram_rows_optim/   DCP: the tables' optimizer moments and step
  micro_engram_dense_optim.pt  dense optimizer, LR scheduler and CPU RNG state (rank 0)
  micro_engram_config.json   the run config pointing at micro_engram_rows
  trainer_state.json         written last: its presence marks the checkpoint complete
output_dir/micro_engram_config.json points at the newest checkpoint's tables.
"""
import glob
import json
import os
import re
import shutil

import torch
import torch.distributed as dist

from ..rows import ROWS_DIR, ROWS_OPTIM_DIR
from ..runconfig import build_config, write_config
from ..weights import latest_checkpoint, load_engram_weights

STATE_FILE = "trainer_state.json"
DENSE_FILE = "micro_engram_dense_optim.pt"
TRAINER_TAG = "micro_engram.train"
_STEP_DIR = re.compile(r"checkpoint-(\d+)$")


class Checkpoints:
    def __init__(self, trainer):
        self.t = trainer

    # ------------------------------------------------------------------ write
    def save(self):
        """Collective: every rank writes its table shards; rank 0 writes the rest, then the
        completion marker, then rotates."""
        t, cfg = self.t, self.t.cfg
        step = t.global_step
        folder = os.path.join(cfg.output_dir, f"checkpoint-{step}")
        t.rows.save(os.path.join(folder, ROWS_DIR), os.path.join(folder, ROWS_OPTIM_DIR))
        if t.rank == 0:
            os.makedirs(folder, exist_ok=True)
            torch.save({"dense_optimizer": t.dense_opt.state_dict(), "scheduler": t.scheduler.state_dict(),
                        "rng": torch.get_rng_state()}, os.path.join(folder, DENSE_FILE))
            write_config(build_config(t.base_conf, t.slots, lambda s: ROWS_DIR), folder)
            write_config(build_config(t.base_conf, t.slots, lambda s: f"checkpoint-{step}/{ROWS_DIR}"),
                         cfg.output_dir)
            marker = {"global_step": step, "epoch": t.epoch, "step_in_epoch": t.step_in_epoch,
                      "total_steps": t.total_steps, "trainer": TRAINER_TAG}
            with open(os.path.join(folder, STATE_FILE), "w") as f:
                json.dump(marker, f, indent=2)
            self.rotate()
        if t.world > 1:
            dist.barrier()
        return folder

    def complete(self):
        """[(step, folder)] of the complete checkpoints, oldest first."""
        found = []
        for c in glob.glob(os.path.join(self.t.cfg.output_dir, "checkpoint-*")):
            hit = _STEP_DIR.search(c)
            if hit and os.path.isfile(os.path.join(c, STATE_FILE)):
                found.append((int(hit.group(1)), c))
        return sorted(found)

    def rotate(self):
        """Keep the newest save_total_limit complete checkpoints (incomplete ones are left for
        inspection; they are never resumed from)."""
        keep = self.t.cfg.save_total_limit
        if keep:
            for _, folder in self.complete()[:-keep]:
                shutil.rmtree(folder, ignore_errors=True)

    # ------------------------------------------------------------------ resume
    def source(self):
        """The checkpoint to resume from: resume_from_checkpoint, else (auto resume) the newest
        complete checkpoint in output_dir, else None."""
        cfg = self.t.cfg
        if cfg.resume_from_checkpoint is not None:
            return cfg.resume_from_checkpoint
        if cfg.auto_resume_from_checkpoints and os.path.isdir(cfg.output_dir):
            return latest_checkpoint(cfg.output_dir)
        return None

    def resume(self):
        """Restore tables, dense weights, optimizers, scheduler and position; returns the
        folder resumed from, or None."""
        t = self.t
        folder = self.source()
        if not folder:
            return None
        with open(os.path.join(folder, STATE_FILE)) as f:
            state = json.load(f)
        if state.get("trainer") != TRAINER_TAG:
            raise ValueError(f"{folder} comes from another trainer; start a new run from it with "
                             "micro_engram_init_from rather than resuming")
        tables, with_moments = t.rows.load(os.path.join(folder, ROWS_DIR), os.path.join(folder, ROWS_OPTIM_DIR))
        self._load_dense_weights(os.path.join(folder, ROWS_DIR))
        blob = torch.load(os.path.join(folder, DENSE_FILE), map_location="cpu", weights_only=False)
        t.dense_opt.load_state_dict(blob["dense_optimizer"])
        t.scheduler.load_state_dict(blob["scheduler"])
        # the schedule continues from the saved position with this run's dense LR
        t.scheduler.base_lrs = [t.dense_lr]
        factor = t.lr_factor()
        for group in t.dense_opt.param_groups:
            group["initial_lr"] = t.dense_lr
            group["lr"] = t.dense_lr * factor
        t.global_step, t.epoch, t.step_in_epoch = state["global_step"], state["epoch"], state["step_in_epoch"]
        if state.get("total_steps") not in (None, t.total_steps):
            t.log0(f"[micro_engram] resume: {t.total_steps} steps in this run (the checkpoint planned "
                   f"{state['total_steps']}); the LR schedule follows the new count")
        t.log0(f"[micro_engram] resumed from {folder} at step {t.global_step} (epoch {t.epoch}, "
               f"{t.step_in_epoch} steps in), {tables} tables"
               + ("" if with_moments else "; no table optimizer state found"))
        return folder

    def _load_dense_weights(self, folder):
        for slot in self.t.slots:
            if slot.frozen:
                continue
            dense = {k: v for k, v in load_engram_weights(folder, layer=slot.layer).items()
                     if not k.startswith("tables.")}
            res = slot.engram.load_state_dict(dense, strict=False)
            tables = {f"tables.{k}.weight" for k in range(len(slot.engram.row_shards))}
            wrong = [k for k in res.missing_keys if k not in tables and k != "mults"] + list(res.unexpected_keys)
            if wrong:
                raise ValueError(f"[micro_engram] resume: the engram at layer {slot.layer} does not match {folder}: "
                                 f"{wrong[:10]}")
