"""Data for micro_engram.train: read JSONL, tokenize, cache, pack, collate.

Rules are the reference's (micro_engram/train/data.py:1-430), which follow Axolotl's:
  completion     text cut at sequence_len*64 tokens, EOS appended when shorter, split into
                 sequence_len chunks; every token trained
  chat_template  rendered with the chat template; the content of trained turns (default the
                 assistant's) is trained through its end-of-turn token, not the role header
Packing: per epoch the samples are shuffled with seed+epoch and packed first-fit over the
last 64 open bins of sequence_len tokens; the bins are shuffled with seed+epoch+1.
Collate: position_ids restart at 0 per document; padding continues the last document's
positions; labels are next-token targets that never cross a document.

The packed micro-batch is built as pinned host tensors so the host->device copy of each
step's inputs is one asynchronous cudaMemcpy per tensor.
"""
import hashlib
import json
import logging
import os

import numpy as np

LOG = logging.getLogger("micro_engram.train")

DATA_VERSION = 1
MAX_OPEN_BINS = 64


# ----------------------------------------------------------------------------- reading
def read_jsonl(path):
    with open(path, encoding="utf-8") as f:
        for n, line in enumerate(f, 1):
            line = line.strip()
            if not line:
                continue
            try:
                yield json.loads(line)
            except json.JSONDecodeError as e:
                raise ValueError(f"{path}:{n}: not valid JSON ({e})") from e


_DEFAULT_ROLES = {"human": "user", "user": "user", "gpt": "assistant", "assistant": "assistant",
                  "model": "assistant", "system": "system", "tool": "tool"}


def _role_map(ds):
    roles = dict(_DEFAULT_ROLES)
    for ours, names in (ds.roles or {}).items():
        for name in names:
            roles[name] = ours
    return roles


def messages_of(obj, ds):
    """[{role, content, ...}] of one chat sample (message_property_mappings applied), or None."""
    msgs = obj.get(ds.field_messages or "messages")
    if msgs is None:
        for alt in ("messages", "conversations", "conversation"):
            if isinstance(obj.get(alt), list):
                msgs = obj[alt]
                break
    if not isinstance(msgs, list) or not msgs:
        return None
    mapping = {"role": "role", "content": "content"}
    mapping.update(ds.message_property_mappings or {})
    if ds.message_property_mappings is None and "from" in msgs[0] and "role" not in msgs[0]:
        mapping.update(role="from", content="value")  # ShareGPT
    roles = _role_map(ds)
    out = []
    for m in msgs:
        msg = {ours: m[theirs] for ours, theirs in mapping.items() if theirs in m and m[theirs] is not None}
        if "role" not in msg or "content" not in msg:
            return None
        msg["role"] = roles.get(msg["role"], msg["role"])
        out.append(msg)
    return out


# ----------------------------------------------------------------------------- tokenizing
def load_template(value):
    if not value:
        return None
    if os.path.isfile(value):
        with open(value, encoding="utf-8") as f:
            return f.read()
    if "{%" in value or "{{" in value:
        return value
    raise FileNotFoundError(f"chat_template_jinja: no such file {value}")


def chat_spans(render, msgs, roles_to_train, eot=()):
    """(full rendered conversation, [(start, end)] character spans of the trained turns).

    A trained span starts after the role header (what the generation prompt adds) and ends
    at the last end-of-turn token (`eot`) inside the turn, inclusive. The template must be
    prefix-stable (rendering the first i turns is a prefix of the whole)."""
    full = render(msgs)
    spans, prev = [], ""
    for i, m in enumerate(msgs):
        cur = render(msgs[:i + 1])
        if not full.startswith(cur):
            raise ValueError("the chat template is not prefix-stable (rendering the first turns is not a prefix of "
                             "the whole conversation), so turns can't be located; check chat_template_kwargs "
                             "(e.g. preserve_thinking) or use axolotl_prepared_dataset")
        if m["role"] in roles_to_train:
            start = len(prev)
            head = render(msgs[:i], add_generation_prompt=True) if i else None
            if head and cur.startswith(head) and len(head) > start:
                start = len(head)
            end = len(cur)
            if eot:
                best = max((cur.rfind(t, start, end) + len(t) for t in eot if cur.rfind(t, start, end) >= 0),
                           default=-1)
                if best > 0:
                    end = best
            spans.append((start, end))
        prev = cur
    return full, spans


class Tokenizing:
    """Raw samples -> (token ids, trained mask or None for all trained)."""

    def __init__(self, tokenizer, cfg):
        self.tok = tokenizer
        self.cfg = cfg
        self.seq = cfg.sequence_len
        self.kwargs = dict(cfg.chat_template_kwargs or {})
        self.template = load_template(cfg.chat_template_jinja)
        self.eot = list(cfg.eot_tokens or [])

    def completion(self, text):
        if not text:
            return []
        cap = self.seq * 64
        ids = self.tok(text, truncation=True, max_length=cap, padding=False)["input_ids"]
        if not ids:
            return []
        eos = self.tok.eos_token_id
        if ids[-1] != eos and len(ids) < cap:
            ids = ids + [eos]
        return [(ids[i:i + self.seq], None) for i in range(0, len(ids), self.seq)]

    def render(self, msgs, add_generation_prompt=False):
        kw = dict(self.kwargs)
        if self.template is not None:
            kw["chat_template"] = self.template
        return self.tok.apply_chat_template(msgs, tokenize=False, add_generation_prompt=add_generation_prompt, **kw)

    def chat(self, msgs, roles_to_train):
        full, spans = chat_spans(self.render, msgs, roles_to_train, self.eot)
        enc = self.tok(full, add_special_tokens=False, return_offsets_mapping=True)
        ids, offs = enc["input_ids"], enc["offset_mapping"]
        mask = np.zeros(len(ids), dtype=bool)
        if offs:
            starts = np.array([s for s, _ in offs])
            ends = np.array([e for _, e in offs])
            for a, b in spans:
                mask |= (starts >= a) & (ends <= b) & (ends > starts)
        return ids, mask


def _tokenize_lines(t, lines, kind, ds):
    out, stats = [], {"empty": 0, "untrained": 0, "too_long": 0, "bad": 0}
    roles = set(ds.roles_to_train or ["assistant"])
    for obj in lines:
        if kind == "completion":
            text = obj.get(ds.field or "text")
            chunks = t.completion(text) if isinstance(text, str) else []
            if not chunks:
                stats["empty"] += 1
            out.extend(chunks)
            continue
        msgs = messages_of(obj, ds)
        if msgs is None:
            stats["bad"] += 1
            continue
        ids, mask = t.chat(msgs, roles)
        if len(ids) > t.seq:
            stats["too_long"] += 1
            continue
        if not mask.any():
            stats["untrained"] += 1
            continue
        out.append((ids, mask))
    return out, stats


def _tok_worker(args):
    lines, kind, cfg_dict, tok_path, ds_dict = args
    from transformers import AutoTokenizer

    from .config import DatasetConfig, TrainConfig

    t = Tokenizing(AutoTokenizer.from_pretrained(tok_path), TrainConfig(**cfg_dict))
    return _tokenize_lines(t, lines, kind, DatasetConfig(**ds_dict))


# ----------------------------------------------------------------------------- cache
class Samples:
    """Flat token storage: tokens int32, trained bool, offsets int64 (sample i = [o_i, o_i+1))."""

    def __init__(self, tokens, trained, offsets):
        self.tokens, self.trained, self.offsets = tokens, trained, offsets

    def __len__(self):
        return len(self.offsets) - 1

    def lengths(self):
        return np.diff(self.offsets)

    def get(self, i):
        a, b = self.offsets[i], self.offsets[i + 1]
        return self.tokens[a:b], self.trained[a:b]

    def save(self, folder):
        os.makedirs(folder, exist_ok=True)
        tmp = os.path.join(folder, "samples.tmp.npz")
        np.savez(tmp, tokens=self.tokens, trained=self.trained, offsets=self.offsets)
        os.replace(tmp, os.path.join(folder, "samples.npz"))

    @classmethod
    def load(cls, folder):
        z = np.load(os.path.join(folder, "samples.npz"))
        return cls(z["tokens"], z["trained"], z["offsets"])

    @classmethod
    def from_list(cls, items):
        offsets = np.zeros(len(items) + 1, dtype=np.int64)
        np.cumsum([len(ids) for ids, _ in items], out=offsets[1:])
        tokens = np.empty(offsets[-1], dtype=np.int32)
        trained = np.empty(offsets[-1], dtype=bool)
        for k, (ids, mask) in enumerate(items):
            a, b = offsets[k], offsets[k + 1]
            tokens[a:b] = ids
            trained[a:b] = True if mask is None else mask
        return cls(tokens, trained, offsets)


def _file_sig(path):
    st = os.stat(path)
    return [os.path.abspath(path), st.st_size, int(st.st_mtime)]


def data_hash(cfg, tok_path):
    h = {
        "v": DATA_VERSION,
        "datasets": [{**d.model_dump(), "_file": _file_sig(d.path)} for d in cfg.datasets],
        "tokenizer": os.path.abspath(tok_path),
        "seq": cfg.sequence_len,
        "template": load_template(cfg.chat_template_jinja),
        "kwargs": cfg.chat_template_kwargs,
        "eot": cfg.eot_tokens,
    }
    return hashlib.sha256(json.dumps(h, sort_keys=True, default=str).encode()).hexdigest()[:16]


def tokenize_all(cfg, tokenizer, tok_path):
    items, total = [], {}
    nproc = max(1, int(cfg.dataset_num_proc or 1))
    for ds in cfg.datasets:
        rows = list(read_jsonl(ds.path))
        if nproc > 1 and len(rows) > 64:
            from multiprocessing import get_context

            chunk = -(-len(rows) // (nproc * 4))
            jobs = [(rows[i:i + chunk], ds.type, cfg.model_dump(), tok_path, ds.model_dump())
                    for i in range(0, len(rows), chunk)]
            with get_context("spawn").Pool(nproc) as pool:
                results = pool.map(_tok_worker, jobs)
        else:
            results = [_tokenize_lines(Tokenizing(tokenizer, cfg), rows, ds.type, ds)]
        before = len(items)
        for got, stats in results:
            items.extend(got)
            for k, v in stats.items():
                total[k] = total.get(k, 0) + v
        LOG.warning(f"[micro_engram] {ds.path}: {len(rows):,} rows -> {len(items) - before:,} samples ({ds.type})")
    dropped = {k: v for k, v in total.items() if v}
    if dropped:
        LOG.warning(f"[micro_engram] dropped rows: {dropped}")
    if not items:
        raise ValueError("no training samples")
    return Samples.from_list(items)


def read_axolotl_prepared(path):
    from datasets import load_from_disk

    ds = load_from_disk(path)
    if hasattr(ds, "keys") and "train" in ds:
        ds = ds["train"]
    items = [(row["input_ids"], np.asarray(row["labels"]) != -100)
             for row in ds.select_columns(["input_ids", "labels"])]
    LOG.warning(f"[micro_engram] read {len(items):,} samples from the Axolotl prepared dataset {path}")
    return Samples.from_list(items)


def prepare(cfg, tokenizer, tok_path, rank=0, barrier=None):
    """The run's samples: from the cache, else tokenized on rank 0 and cached."""
    if cfg.axolotl_prepared_dataset:
        return read_axolotl_prepared(cfg.axolotl_prepared_dataset)
    folder = None
    if cfg.dataset_prepared_path:
        folder = os.path.join(cfg.dataset_prepared_path, "micro_engram-" + data_hash(cfg, tok_path))
    if folder and os.path.isfile(os.path.join(folder, "samples.npz")):
        LOG.warning(f"[micro_engram] tokenized data from cache {folder}")
        return Samples.load(folder)
    if folder is None:
        return tokenize_all(cfg, tokenizer, tok_path)
    if rank == 0:
        tokenize_all(cfg, tokenizer, tok_path).save(folder)
        LOG.warning(f"[micro_engram] tokenized data cached in {folder}")
    if barrier is not None:
        barrier()
    return Samples.load(folder)


# ----------------------------------------------------------------------------- packing
def pack(lengths, capacity, seed, shuffle=True):
    """Bins (lists of sample indices) of <= capacity tokens, first-fit over the last
    MAX_OPEN_BINS open bins, samples in a seeded random order; empty/too-long samples skipped."""
    order = np.arange(len(lengths))
    if shuffle:
        np.random.default_rng(seed).shuffle(order)
    bins, room, open_bins = [], [], []
    for i in order:
        n = int(lengths[i])
        if n == 0 or n > capacity:
            continue
        placed = False
        for b in open_bins:
            if room[b] >= n:
                bins[b].append(int(i))
                room[b] -= n
                if room[b] == 0:
                    open_bins.remove(b)
                placed = True
                break
        if not placed:
            bins.append([int(i)])
            room.append(capacity - n)
            if room[-1] > 0:
                open_bins.append(len(bins) - 1)
                if len(open_bins) > MAX_OPEN_BINS:
                    open_bins.pop(0)
    if shuffle:
        perm = np.random.default_rng(seed + 1).permutation(len(bins))
        bins = [bins[k] for k in perm]
    return bins


def collate(samples, bins, seq_len, pad_id, pin=False):
    """{input_ids, labels, position_ids} [B, seq_len] int64 for a micro-batch of bins."""
    import torch

    B = len(bins)
    ids = np.full((B, seq_len), pad_id, dtype=np.int64)
    lab = np.full((B, seq_len), -100, dtype=np.int64)
    pos = np.zeros((B, seq_len), dtype=np.int64)
    for r, b in enumerate(bins):
        t, last = 0, 0
        for i in b:
            tok, tr = samples.get(i)
            n = len(tok)
            ids[r, t:t + n] = tok
            lab[r, t:t + n] = np.where(tr, tok, -100)
            pos[r, t:t + n] = np.arange(n)
            t += n
            last = n
        if t < seq_len:
            pos[r, t:] = np.arange(last, last + seq_len - t)
    shifted = np.full_like(lab, -100)
    shifted[:, :-1] = lab[:, 1:]
    shifted[:, :-1][pos[:, 1:] == 0] = -100
    out = {"input_ids": torch.from_numpy(ids), "labels": torch.from_numpy(shifted), "position_ids": torch.from_numpy(pos)}
    if pin:
        out = {k: v.pin_memory() for k, v in out.items()}
    return out


class EpochPlan:
    """Which bins each rank gets for each step of an epoch."""

    def __init__(self, samples, cfg, world):
        self.samples, self.cfg, self.world = samples, cfg, world
        self.per_step = world * cfg.micro_batch_size * cfg.gradient_accumulation_steps
        self._cache = {}

    def bins(self, epoch):
        if epoch not in self._cache:
            self._cache = {epoch: pack(self.samples.lengths(), self.cfg.sequence_len, self.cfg.seed + epoch,
                                       shuffle=self.cfg.shuffle_each_epoch or epoch == 0)}
        return self._cache[epoch]

    def steps_per_epoch(self, epoch=0):
        return len(self.bins(epoch)) // self.per_step

    def micro_batches(self, epoch, step, rank):
        b = self.bins(epoch)
        base = step * self.per_step
        mbs, ga = self.cfg.micro_batch_size, self.cfg.gradient_accumulation_steps
        return [b[base + (a * self.world + rank) * mbs: base + (a * self.world + rank) * mbs + mbs] for a in range(ga)]
