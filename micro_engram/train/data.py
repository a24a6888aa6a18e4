"""Training data of micro_engram.train: JSONL -> token samples -> packed bins -> micro-batches.

The rules are the public behaviour of the reference trainer (Ready-Art/micro_engram_fork,
micro_engram/train/data.py:1-430), which follows Axolotl, because a resumed or compared run
must see the same tokens in the same order:
  completion     tokens cut at sequence_len * 64, EOS appended when the text ends before the
                 cut, split into sequence_len pieces; every token trained
  chat_template  the conversation rendered with the chat template; a trained turn (default:
                 the assistant's) is trained from after its role header through its last
                 end-of-turn token
  packing        per epoch the samples are visited in a seed+epoch order and placed first-fit
                 into the newest 64 open bins of sequence_len tokens; the bins are then put in
                 a seed+epoch+1 order
  collate        positions restart at 0 per document; padding continues the last document's
                 positions; labels are next-token targets that never cross a document
The implementation is this framework's: a columnar sample store, vectorised collation into
pinned host tensors (one asynchronous copy per tensor and step), and a step plan built by
reshaping an index range.
"""
import hashlib
import json
import logging
import os

import numpy as np

LOG = logging.getLogger("micro_engram.train")

CACHE_FORMAT = 2
MAX_OPEN_BINS = 64
IGNORE = -100


# ============================================================================ reading
def read_jsonl(path):
    """The objects of a JSON-lines file (blank lines skipped; a bad line names its number)."""
    with open(path, encoding="utf-8") as f:
        for number, line in enumerate(f, 1):
            if line.strip():
                try:
                    yield json.loads(line)
                except json.JSONDecodeError as e:
                    raise ValueError(f"{path}:{number}: not valid JSON ({e})") from e


ROLE_ALIASES = {"human": "user", "user": "user", "gpt": "assistant", "assistant": "assistant",
                "model": "assistant", "system": "system", "tool": "tool"}
MESSAGE_FIELDS = ("messages", "conversations", "conversation")


def messages_of(obj, ds):
    """[{role, content, ...}] of one chat sample, with the dataset's field and role mappings
    applied (ShareGPT's from/value is recognised); None when the sample has no usable turns."""
    turns = obj.get(ds.field_messages or "messages")
    if turns is None:
        turns = next((obj[k] for k in MESSAGE_FIELDS if isinstance(obj.get(k), list)), None)
    if not isinstance(turns, list) or not turns:
        return None
    fields = {"role": "role", "content": "content"}
    if ds.message_property_mappings is not None:
        fields.update(ds.message_property_mappings)
    elif "from" in turns[0] and "role" not in turns[0]:
        fields.update(role="from", content="value")
    aliases = dict(ROLE_ALIASES)
    for role, names in (ds.roles or {}).items():
        aliases.update({name: role for name in names})
    out = []
    for turn in turns:
        msg = {mine: turn[theirs] for mine, theirs in fields.items() if turn.get(theirs) is not None}
        if "role" not in msg or "content" not in msg:
            return None
        msg["role"] = aliases.get(msg["role"], msg["role"])
        out.append(msg)
    return out


# ============================================================================ tokenizing
_JINJA_TAGS = ("{%", "{{")


def load_template(value):
    """chat_template_jinja as template text. The key names a template file or holds the template
    itself; a value that opens no file and carries no Jinja tag is a missing file."""
    if not value:
        return None
    try:
        with open(value, encoding="utf-8") as f:
            return f.read()
    except OSError:  # no such file, a folder, or template text too long to be a path
        if any(tag in value for tag in _JINJA_TAGS):
            return value
        raise FileNotFoundError(f"chat_template_jinja: no such file {value}") from None


def _turn_end(text, start, end, eot):
    """End of a trained turn: just past the last end-of-turn marker inside [start, end), or end."""
    found = [text.rfind(t, start, end) + len(t) for t in eot if text.rfind(t, start, end) >= 0]
    best = max(found, default=-1)
    return best if best > 0 else end


def chat_spans(render, msgs, roles_to_train, eot=()):
    """(rendered conversation, character spans of its trained turns). The template must be
    prefix-stable: rendering the first i turns gives a prefix of the whole conversation."""
    full = render(msgs)
    spans = []
    before = ""  # the rendering of the turns so far
    for i, msg in enumerate(msgs):
        upto = render(msgs[:i + 1])
        if not full.startswith(upto):
            raise ValueError("the chat template is not prefix-stable (the first turns do not render as a prefix of "
                             "the whole conversation), so trained turns cannot be located; check "
                             "chat_template_kwargs (e.g. preserve_thinking) or use axolotl_prepared_dataset")
        if msg["role"] in roles_to_train:
            start = len(before)
            if i:  # skip the role header: it is what the generation prompt adds
                header = render(msgs[:i], add_generation_prompt=True)
                if upto.startswith(header):
                    start = max(start, len(header))
            spans.append((start, _turn_end(upto, start, len(upto), eot) if eot else len(upto)))
        before = upto
    return full, spans


class Tokenizing:
    """Turns raw samples into (token ids, trained mask or None when every token trains)."""

    def __init__(self, tokenizer, cfg):
        self.tok = tokenizer
        self.seq = cfg.sequence_len
        self.template_kwargs = dict(cfg.chat_template_kwargs or {})
        template = load_template(cfg.chat_template_jinja)
        if template is not None:
            self.template_kwargs["chat_template"] = template
        self.eot = list(cfg.eot_tokens or [])

    def completion(self, text):
        """[(ids, None)] pieces of sequence_len tokens of one text."""
        if not text:
            return []
        cap = 64 * self.seq
        ids = list(self.tok(text, truncation=True, max_length=cap, padding=False)["input_ids"])
        if not ids:
            return []
        if len(ids) < cap and ids[-1] != self.tok.eos_token_id:
            ids.append(self.tok.eos_token_id)
        return [(ids[a:a + self.seq], None) for a in range(0, len(ids), self.seq)]

    def render(self, msgs, add_generation_prompt=False):
        return self.tok.apply_chat_template(msgs, tokenize=False, add_generation_prompt=add_generation_prompt,
                                            **self.template_kwargs)

    def chat(self, msgs, roles_to_train):
        """(ids, trained mask) of one conversation: a token trains when its characters lie
        inside a trained span."""
        text, spans = chat_spans(self.render, msgs, roles_to_train, self.eot)
        enc = self.tok(text, add_special_tokens=False, return_offsets_mapping=True)
        ids = enc["input_ids"]
        mask = np.zeros(len(ids), dtype=bool)
        if enc["offset_mapping"]:
            where = np.asarray(enc["offset_mapping"], dtype=np.int64).reshape(-1, 2)
            lo, hi = where[:, 0], where[:, 1]
            for a, b in spans:
                mask |= (lo >= a) & (hi <= b) & (hi > lo)
        return ids, mask


def _tokenize_rows(t, rows, kind, ds):
    """(samples, counts of dropped rows by reason) for one dataset's rows."""
    samples, dropped = [], dict.fromkeys(("empty", "untrained", "too_long", "bad"), 0)
    train_roles = set(ds.roles_to_train or ["assistant"])
    for obj in rows:
        if kind == "completion":
            text = obj.get(ds.field or "text")
            pieces = t.completion(text) if isinstance(text, str) else []
            dropped["empty"] += not pieces
            samples += pieces
            continue
        msgs = messages_of(obj, ds)
        if msgs is None:
            dropped["bad"] += 1
            continue
        ids, mask = t.chat(msgs, train_roles)
        reason = "too_long" if len(ids) > t.seq else ("untrained" if not mask.any() else None)
        if reason:
            dropped[reason] += 1
        else:
            samples.append((ids, mask))
    return samples, dropped


def _tokenize_job(job):
    """Worker of the multi-process tokenizer: (rows, kind, config dict, tokenizer path, dataset dict)."""
    rows, kind, cfg_dict, tok_path, ds_dict = job
    from transformers import AutoTokenizer

    from .config import DatasetConfig, TrainConfig

    t = Tokenizing(AutoTokenizer.from_pretrained(tok_path), TrainConfig(**cfg_dict))
    return _tokenize_rows(t, rows, kind, DatasetConfig(**ds_dict))


# ============================================================================ samples
class Samples:
    """Every sample's tokens in one int32 column, a bool trained column beside it, and int64
    offsets (sample i is rows offsets[i]:offsets[i+1])."""

    def __init__(self, tokens, trained, offsets):
        self.tokens, self.trained, self.offsets = tokens, trained, offsets

    def __len__(self):
        return len(self.offsets) - 1

    def lengths(self):
        return np.diff(self.offsets)

    def get(self, i):
        lo, hi = self.offsets[i], self.offsets[i + 1]
        return self.tokens[lo:hi], self.trained[lo:hi]

    @classmethod
    def from_list(cls, items):
        """From [(ids, trained mask or None)]."""
        lens = np.fromiter((len(ids) for ids, _ in items), dtype=np.int64, count=len(items))
        offsets = np.zeros(len(items) + 1, dtype=np.int64)
        np.cumsum(lens, out=offsets[1:])
        if not items:
            return cls(np.zeros(0, np.int32), np.zeros(0, bool), offsets)
        tokens = np.concatenate([np.asarray(ids, dtype=np.int32).reshape(-1) for ids, _ in items])
        trained = np.concatenate([np.ones(n, dtype=bool) if m is None else np.asarray(m, dtype=bool).reshape(-1)
                                  for n, (_, m) in zip(lens, items)])
        return cls(tokens, trained, offsets)

    def save(self, folder):
        """Atomically (write, then rename) as folder/samples.npz."""
        os.makedirs(folder, exist_ok=True)
        partial = os.path.join(folder, "samples.partial.npz")
        np.savez(partial, tokens=self.tokens, trained=self.trained, offsets=self.offsets)
        os.replace(partial, os.path.join(folder, "samples.npz"))

    @classmethod
    def load(cls, folder):
        with np.load(os.path.join(folder, "samples.npz")) as z:
            return cls(z["tokens"], z["trained"], z["offsets"])


def cache_key(cfg, tok_path):
    """16 hex digits naming a tokenized-data cache: changes with the data files (path, size,
    mtime), the dataset settings, the tokenizer, sequence_len and the chat-template settings."""
    digest = hashlib.sha256(f"micro_engram data cache v{CACHE_FORMAT}".encode())

    def add(label, value):
        digest.update(f"|{label}=".encode())
        digest.update(json.dumps(value, sort_keys=True, default=str).encode())

    for ds in cfg.datasets:
        st = os.stat(ds.path)
        add("dataset", ds.model_dump())
        add("file", [os.path.abspath(ds.path), st.st_size, int(st.st_mtime)])
    add("tokenizer", os.path.abspath(tok_path))
    add("sequence_len", cfg.sequence_len)
    add("template", load_template(cfg.chat_template_jinja))
    add("template_kwargs", cfg.chat_template_kwargs)
    add("eot", cfg.eot_tokens)
    return digest.hexdigest()[:16]


data_hash = cache_key  # the name the tools use


def _tokenize_dataset(cfg, tokenizer, tok_path, ds, nproc):
    rows = list(read_jsonl(ds.path))
    if nproc > 1 and len(rows) > 64:
        from multiprocessing import get_context

        size = -(-len(rows) // (4 * nproc))
        jobs = [(rows[a:a + size], ds.type, cfg.model_dump(), tok_path, ds.model_dump())
                for a in range(0, len(rows), size)]
        with get_context("spawn").Pool(nproc) as pool:
            parts = pool.map(_tokenize_job, jobs)
    else:
        parts = [_tokenize_rows(Tokenizing(tokenizer, cfg), rows, ds.type, ds)]
    samples = [s for got, _ in parts for s in got]
    dropped = {}
    for _, counts in parts:
        for reason, n in counts.items():
            dropped[reason] = dropped.get(reason, 0) + n
    LOG.warning(f"[micro_engram] {ds.path}: {len(rows):,} rows -> {len(samples):,} samples ({ds.type})")
    return samples, dropped


def tokenize_all(cfg, tokenizer, tok_path):
    """Every dataset of the config tokenized (dataset_num_proc processes when set)."""
    nproc = max(1, int(cfg.dataset_num_proc or 1))
    items, dropped = [], {}
    for ds in cfg.datasets:
        got, counts = _tokenize_dataset(cfg, tokenizer, tok_path, ds, nproc)
        items += got
        for reason, n in counts.items():
            dropped[reason] = dropped.get(reason, 0) + n
    if any(dropped.values()):
        LOG.warning(f"[micro_engram] dropped rows: {({k: v for k, v in dropped.items() if v})}")
    if not items:
        raise ValueError("no training samples")
    return Samples.from_list(items)


def read_axolotl_prepared(path):
    """Samples from an Axolotl prepared dataset: a datasets.save_to_disk folder (a Dataset, or a
    DatasetDict whose "train" split is used) with input_ids and labels, where a label of -100
    marks a token that is not trained."""
    from datasets import load_from_disk

    loaded = load_from_disk(path)
    split = loaded["train"] if isinstance(loaded, dict) and "train" in loaded else loaded  # DatasetDict is a dict
    ids = split["input_ids"]
    trained = [np.not_equal(np.asarray(lab), IGNORE) for lab in split["labels"]]
    LOG.warning(f"[micro_engram] {len(ids):,} samples from the Axolotl prepared dataset {path}")
    return Samples.from_list(list(zip(ids, trained)))


def prepare(cfg, tokenizer, tok_path, rank=0, barrier=None):
    """The run's samples: an Axolotl prepared dataset, else the tokenized-data cache under
    dataset_prepared_path (rank 0 builds it, the others wait at `barrier`), else tokenized now."""
    if cfg.axolotl_prepared_dataset:
        return read_axolotl_prepared(cfg.axolotl_prepared_dataset)
    if not cfg.dataset_prepared_path:
        return tokenize_all(cfg, tokenizer, tok_path)
    folder = os.path.join(cfg.dataset_prepared_path, "micro_engram-" + cache_key(cfg, tok_path))
    if os.path.isfile(os.path.join(folder, "samples.npz")):
        LOG.warning(f"[micro_engram] tokenized data from the cache {folder}")
        return Samples.load(folder)
    if rank == 0:
        tokenize_all(cfg, tokenizer, tok_path).save(folder)
        LOG.warning(f"[micro_engram] tokenized data cached in {folder}")
    if barrier is not None:
        barrier()
    return Samples.load(folder)


# ============================================================================ packing
def pack(lengths, capacity, seed, shuffle=True):
    """Bins (lists of sample indices) of at most `capacity` tokens. Samples are visited in a
    seeded random order and go into the first of the newest MAX_OPEN_BINS bins with room; empty
    and over-long samples are skipped; the bins come back in a second seeded random order."""
    visit = np.arange(len(lengths))
    if shuffle:
        np.random.default_rng(seed).shuffle(visit)
    members, free = [], []
    window = []  # bins still open, oldest first
    for i in visit.tolist():
        need = int(lengths[i])
        if need <= 0 or need > capacity:
            continue
        target = next((b for b in window if free[b] >= need), -1)
        if target < 0:
            members.append([i])
            free.append(capacity - need)
            if free[-1] > 0:
                window.append(len(members) - 1)
                if len(window) > MAX_OPEN_BINS:
                    window.pop(0)
            continue
        members[target].append(i)
        free[target] -= need
        if free[target] == 0:
            window.remove(target)
    if shuffle:
        order = np.random.default_rng(seed + 1).permutation(len(members))
        members = [members[k] for k in order]
    return members


def collate(samples, bins, seq_len, pad_id, pin=False):
    """{input_ids, labels, position_ids}: int64 [len(bins), seq_len] tensors of one micro-batch
    (pinned host memory with pin)."""
    import torch

    rows = len(bins)
    ids = np.full((rows, seq_len), pad_id, dtype=np.int64)
    labels = np.full((rows, seq_len), IGNORE, dtype=np.int64)
    pos = np.zeros((rows, seq_len), dtype=np.int64)
    for r, members in enumerate(bins):
        docs = [samples.get(i) for i in members]
        lens = np.array([len(t) for t, _ in docs], dtype=np.int64)
        n = int(lens.sum())
        if n:
            toks = np.concatenate([t for t, _ in docs])
            trained = np.concatenate([m for _, m in docs])
            ids[r, :n] = toks
            labels[r, :n] = np.where(trained, toks, IGNORE)
            first = np.repeat(np.cumsum(lens) - lens, lens)
            pos[r, :n] = np.arange(n) - first
        tail_from = int(lens[-1]) if len(lens) else 0
        pos[r, n:] = tail_from + np.arange(seq_len - n)
    targets = np.full_like(labels, IGNORE)
    targets[:, :-1] = np.where(pos[:, 1:] == 0, IGNORE, labels[:, 1:])  # never across a document start
    out = {"input_ids": torch.from_numpy(ids), "labels": torch.from_numpy(targets),
           "position_ids": torch.from_numpy(pos)}
    return {k: v.pin_memory() for k, v in out.items()} if pin else out


class EpochPlan:
    """Which bins every rank trains at every step of an epoch: a step takes world x
    micro_batch_size x gradient_accumulation_steps consecutive bins; micro-batch a of rank r is
    the r-th of the world groups in the a-th slice."""

    def __init__(self, samples, cfg, world):
        self.samples, self.cfg, self.world = samples, cfg, world
        self.mbs, self.ga = cfg.micro_batch_size, cfg.gradient_accumulation_steps
        self.per_step = world * self.mbs * self.ga
        self._epoch, self._bins = None, None

    def bins(self, epoch):
        if self._epoch != epoch:
            cfg = self.cfg
            self._bins = pack(self.samples.lengths(), cfg.sequence_len, cfg.seed + epoch,
                              shuffle=cfg.shuffle_each_epoch or epoch == 0)
            self._epoch = epoch
        return self._bins

    def steps_per_epoch(self, epoch=0):
        return len(self.bins(epoch)) // self.per_step

    def micro_batches(self, epoch, step, rank):
        """[micro-batch][bin] of `rank` at `step`."""
        bins = self.bins(epoch)
        index = step * self.per_step + np.arange(self.per_step).reshape(self.ga, self.world, self.mbs)[:, rank, :]
        return [[bins[k] for k in row] for row in index.tolist()]
