"""What a training run reports: the JSONL log (output_dir/train_log.jsonl, one line per logging
step, the reference's keys: loss, ppl, grad_norm, table_grad_norm, learning_rate, dense_lr,
epoch, step, s_per_step, trained_tokens_per_s, mem_peak_*, engram/* stats), the progress bar,
wandb, the one-step profile (profile_step) and the CUDA memory snapshot.

Step results arrive as device tensors; they become Python numbers here, at logging steps
only, so steps between logs never wait on the host.
"""
import json
import logging
import math
import os
import time

import torch
import torch.distributed as dist

from ..stats import module_stats

LOG = logging.getLogger("micro_engram.train")


def to_host(logs):
    """Step logs with every tensor turned into a Python number (one device read for all)."""
    keys = [k for k, v in logs.items() if torch.is_tensor(v)]
    if not keys:
        return dict(logs)
    vals = torch.stack([logs[k].detach().double().reshape(()).to(logs[keys[0]].device) for k in keys]).tolist()
    out = dict(logs)
    out.update(zip(keys, vals))
    for k in ("tokens", "step"):
        if k in out and isinstance(out[k], float):
            out[k] = int(out[k])
    if "loss" in out:
        out["ppl"] = math.exp(min(out["loss"], 50.0))
    return out


class Reporter:
    def __init__(self, trainer):
        self.t = trainer
        self.pbar = None
        self.wandb = None
        self.window_start = time.time()
        self.window_tokens = 0

    # ------------------------------------------------------------------ lifecycle
    def open(self):
        t, cfg = self.t, self.t.cfg
        if t.rank != 0:
            return
        os.makedirs(cfg.output_dir, exist_ok=True)
        if cfg.wandb_project and cfg.wandb_mode != "disabled":
            import wandb

            self.wandb = wandb
            wandb.init(project=cfg.wandb_project, name=cfg.wandb_name, entity=cfg.wandb_entity, mode=cfg.wandb_mode,
                       config=cfg.model_dump(), resume="allow")
        try:
            from tqdm import tqdm
        except ImportError:
            return
        self.pbar = tqdm(total=t.total_steps, initial=t.global_step, dynamic_ncols=True, unit="step",
                         bar_format=self._bar(""))

    def close(self):
        if self.pbar is not None:
            self.pbar.close()
            self.pbar = None
        if self.wandb is not None and self.t.rank == 0:
            self.wandb.finish()

    @staticmethod
    def _bar(tail):
        return "{percentage:3.0f}%|{bar}| {n}/{total} [{elapsed}<{remaining}, {rate_inv_fmt}]" + tail

    # ------------------------------------------------------------------ per step
    def step_done(self, logs, steps_in_epoch):
        """Count the step; at logging steps turn its results into a log line."""
        t, cfg = self.t, self.t.cfg
        self.window_tokens += logs["tokens"]
        last = t.global_step == t.total_steps
        logging_step = t.global_step % cfg.logging_steps == 0 or last
        if self.pbar is not None:
            self.pbar.update(1)
        if not logging_step:
            return
        host = to_host(logs)
        if self.pbar is not None:  # the loss shown is the last logging step's (no per-step host read)
            ppl = host["ppl"]
            shown = f"{ppl:.0f}" if ppl >= 100 else f"{ppl:.2f}"
            self.pbar.bar_format = self._bar(f"  loss {host['loss']:.4f}  ppl {shown}")
            self.pbar.refresh()
        from .faults import check_device

        check_device(t)  # a kernel-side error (bounds, capacity, a bounded wait that ran out) stops the run
        elapsed = time.time() - self.window_start
        host.pop("tokens")
        window = self.window_tokens
        window = float(window.item()) if torch.is_tensor(window) else float(window)
        host.update(self.memory())
        host.update(self.engram_stats())
        host.update({"epoch": round(t.epoch + t.step_in_epoch / max(1, steps_in_epoch), 4), "step": t.global_step,
                     "s_per_step": round(elapsed / cfg.logging_steps, 2),
                     "trained_tokens_per_s": round(window / max(elapsed, 1e-9), 1)})
        if t.timers.enabled:
            host.update({f"time_ms/{k}": v for k, v in t.timers.report().items()})
        self.write(host)
        self.window_start, self.window_tokens = time.time(), 0

    def write(self, logs):
        t = self.t
        if t.rank != 0:
            return
        line = json.dumps({k: (round(v, 6) if isinstance(v, float) else v) for k, v in logs.items()})
        if self.pbar is not None:
            self.pbar.write(line)
        else:
            print(line, flush=True)
        with open(os.path.join(t.cfg.output_dir, "train_log.jsonl"), "a") as f:
            f.write(line + "\n")
        if self.wandb is not None:
            self.wandb.log({k: v for k, v in logs.items() if isinstance(v, (int, float))}, step=t.global_step)

    # ------------------------------------------------------------------ pieces of a log line
    def memory(self):
        t = self.t
        if t.device.type != "cuda":
            return {}
        mine = torch.tensor([torch.cuda.max_memory_allocated(t.device), torch.cuda.max_memory_reserved(t.device)],
                            dtype=torch.float64, device=t.device) / 2 ** 30
        every = [torch.zeros_like(mine) for _ in range(t.world)]
        if t.world > 1:
            dist.all_gather(every, mine)
        else:
            every = [mine]
        table = torch.stack(every).tolist()
        return {"mem_peak_alloc_gib": round(max(r[0] for r in table), 2),
                "mem_peak_reserved_gib": round(max(r[1] for r in table), 2),
                "mem_peak_alloc_per_gpu": [round(r[0], 2) for r in table]}

    def engram_stats(self):
        t = self.t
        every = t.cfg.micro_engram_stats_steps
        gates = [s.engram.pop_gate_stats() for s in t.slots]  # every rank drains its counters
        if t.rank != 0 or not every or t.global_step % every:
            return {}
        out = {}
        for slot, gate in zip(t.slots, gates):
            if slot.frozen:
                continue
            try:
                stats = module_stats(slot.engram)
            except Exception as e:  # noqa: BLE001 - stats never stop a run
                LOG.warning(f"[micro_engram] engram stats failed: {e}")
                continue
            if gate is not None:
                stats["engram/gate_mean"], stats["engram/gate_saturated"] = gate
            if len(t.slots) > 1:
                stats = {k.replace("engram/", f"engram_L{slot.layer}/", 1): v for k, v in stats.items()}
            out.update(stats)
        return out

    # ------------------------------------------------------------------ profile and memory snapshot
    def profiled(self, run_step):
        """run_step() under torch.profiler; rank 0 writes profile/rank0_step<N>.{txt,json}."""
        from torch.profiler import ProfilerActivity, profile

        t = self.t
        cuda = t.device.type == "cuda"
        kinds = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if cuda else [])
        with profile(activities=kinds, record_shapes=False) as prof:
            logs = run_step()
            if cuda:
                torch.cuda.synchronize(t.device)
        if t.rank == 0:
            folder = os.path.join(t.cfg.output_dir, "profile")
            os.makedirs(folder, exist_ok=True)
            stem = os.path.join(folder, f"rank0_step{t.global_step + 1}")
            try:
                prof.export_chrome_trace(stem + ".json")
                with open(stem + ".txt", "w") as f:
                    f.write(prof.key_averages().table(sort_by="cuda_time_total" if cuda else "cpu_time_total",
                                                      row_limit=40))
                LOG.warning(f"[micro_engram] profile written: {stem}.txt (top kernels), {stem}.json (timeline)")
            except Exception as e:  # noqa: BLE001
                LOG.warning(f"[micro_engram] could not write the profile (training continues): {e}")
        return logs

    def memory_snapshot(self):
        t = self.t
        folder = os.path.join(t.cfg.output_dir, "memory_snapshot")
        os.makedirs(folder, exist_ok=True)
        path = os.path.join(folder, f"rank{t.rank}_step{t.global_step}.pickle")
        try:
            torch.cuda.memory._dump_snapshot(path)
            LOG.warning(f"[micro_engram] memory snapshot written: {path}")
        finally:
            torch.cuda.memory._record_memory_history(enabled=None)
