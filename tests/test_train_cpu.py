"""The trainer end to end on CPU (2 gloo processes, a tiny random Gemma 4 saved by HF, a
word-level tokenizer, completion data): the first-step loss against a plain HF forward
(per-token mean over micro-batches and ranks), the no-grad prefix, save -> resume -> next
step against the uninterrupted run, micro_batch_size 2, the dense LR schedule (and a new value
on resume), micro_engram_train_scales, sparse vs dense row gradients, cpu_ram_efficient_loading,
and a whole Trainer.train() run (checkpoint rotation, the final engram config and weights,
profile_step outputs, the JSONL log). Reference counterpart: test_train.py."""
import json
import os

import pytest
import torch

from helpers import run_dist

SPECIAL = ["<pad>", "<eos>", "<bos>", "<|turn>", "<turn|>"]
WORDS = [f"w{i}" for i in range(123)]
V = len(SPECIAL) + len(WORDS)


def _tokenizer():
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast

    vocab = {t: i for i, t in enumerate(SPECIAL + WORDS)}
    core = Tokenizer(models.WordLevel(vocab, unk_token="<pad>"))
    core.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    return PreTrainedTokenizerFast(tokenizer_object=core, pad_token="<pad>", eos_token="<eos>", bos_token="<bos>")


def _tiny_gemma():
    """4 layers (2 sliding, 2 global), d 64, norm weights moved off 1 so that they matter."""
    from transformers import Gemma4ForCausalLM
    from transformers.models.gemma4.configuration_gemma4 import Gemma4TextConfig

    layer_types = ["sliding_attention"] * 2 + ["full_attention"] * 2
    cfg = Gemma4TextConfig(vocab_size=V, hidden_size=64, intermediate_size=128, num_hidden_layers=4,
                           num_attention_heads=4, num_key_value_heads=2, head_dim=16, global_head_dim=32,
                           layer_types=layer_types, sliding_window=8, hidden_size_per_layer_input=0,
                           max_position_embeddings=1024, final_logit_softcapping=30.0, pad_token_id=0,
                           eos_token_id=1, bos_token_id=2)
    cfg.architectures = ["Gemma4ForCausalLM"]
    torch.manual_seed(0)
    model = Gemma4ForCausalLM(cfg)
    norms = [p for p in model.parameters() if p.dim() == 1]
    with torch.no_grad():
        for p in norms:
            p.copy_(1 + 0.2 * torch.randn_like(p))
    return model


def _corpus(path, docs=40):
    g = torch.Generator().manual_seed(1)
    lines = []
    for _ in range(docs):
        length = int(torch.randint(5, 60, (1,), generator=g))
        words = [WORDS[int(i)] for i in torch.randint(0, len(WORDS), (length,), generator=g)]
        lines.append(json.dumps({"text": "<bos> " + " ".join(words)}))
    with open(path, "w") as f:
        f.write("\n".join(lines))
    return path


def make_assets(root):
    """(model folder with tokenizer, completion JSONL); also canon.pt merging every even/odd id pair."""
    model_dir = os.path.join(root, "base")
    _tiny_gemma().to(torch.bfloat16).save_pretrained(model_dir)
    _tokenizer().save_pretrained(model_dir)
    torch.save(torch.arange(V) & ~1, os.path.join(root, "canon.pt"))
    return model_dir, _corpus(os.path.join(root, "cpt.jsonl"))


def base_cfg(root, model_dir, data, out, **over):
    engram = {"micro_engram_layer": 1, "micro_engram_table_size": 97, "micro_engram_dim": 8, "micro_engram_heads": 2,
              "micro_engram_gate": "scalar_sqrt", "micro_engram_extra": [{"layer": 3}],
              "micro_engram_optimizer": "rowwise_adam", "micro_engram_dtype": "fp32",
              "micro_engram_canon_path": os.path.join(root, "canon.pt"), "micro_engram_stats_steps": 1}
    run = {"base_model": model_dir, "datasets": [{"path": data, "type": "completion"}], "sequence_len": 32,
           "output_dir": out, "micro_batch_size": 1, "gradient_accumulation_steps": 2, "num_epochs": 1,
           "learning_rate": 5e-3, "lr_scheduler": "constant", "max_grad_norm": 2.0, "seed": 7,
           "gradient_checkpointing": True, "loss_chunk_tokens": 16, "save_steps": None}
    return {**run, **engram, **over}


def _trainer(cfg):
    from micro_engram.train.config import load_config
    from micro_engram.train.loop import Trainer

    t = Trainer(load_config(cfg))
    t.build()
    return t


def _randomize_dense(t):
    g = torch.Generator().manual_seed(5)
    with torch.no_grad():
        for p in (p for s in t.slots for p in s.engram.parameters()):
            p.copy_(torch.randn(p.shape, generator=g) * 0.05)


def snapshot(t):
    """Every engram weight of the trainer (dense parameters and table row shards), cloned."""
    named = {}
    for s in t.slots:
        named.update({f"{s.layer}.{n}": p for n, p in s.engram.named_parameters()})
        named.update({f"{s.layer}.rows{k}": p for k, p in enumerate(s.engram.row_shards)})
    return {k: p.detach().clone() for k, p in named.items()}


def grad_as_dense(p):
    """A table shard's gradient as a dense fp32 tensor, whether it is sparse (rows, values) or not."""
    sparse = getattr(p, "sparse_grad", None)
    if sparse is None:
        return None if p.grad is None else p.grad.float().clone()
    rows, vals = sparse
    return torch.zeros(p.shape, dtype=torch.float32).index_add_(0, rows, vals.float())


def hf_token_mean_loss(ref, batches):
    """Cross-entropy of the HF model, summed over every rank's batches and divided by the trained tokens."""
    import torch.distributed as dist

    tot = torch.zeros(2)
    with torch.no_grad():
        for b in batches:
            logits = ref(input_ids=b["input_ids"], position_ids=b["position_ids"]).logits.float().reshape(-1, V)
            labels = b["labels"].reshape(-1)
            tot[0] += torch.nn.functional.cross_entropy(logits, labels, ignore_index=-100, reduction="sum")
            tot[1] += (labels != -100).sum()
    dist.all_reduce(tot)
    return float(tot[0] / tot[1])


def _clear_grads(t):
    for p in t.dense:
        p.grad = None
    t.rows.zero_grad()


def check_first_step(t, ref, rank):
    micro = t.plan.micro_batches(0, 0, rank)
    return {"ref_loss": hf_token_mean_loss(ref, [t._micro_batch(b) for b in micro]),
            "loss": t.train_step(micro)["loss"]}


def check_prefix(t, rank):
    """The no-grad prefix (layers before the first engram run without autograd) leaves every engram
    gradient as a full backward gives it."""
    _randomize_dense(t)
    batch = t._micro_batch(t.plan.micro_batches(0, 1, rank)[0])
    runs = {}
    for prefix in (True, False):
        t.cfg.no_grad_prefix = prefix
        _clear_grads(t)
        t.forward_loss(batch, 1.0)
        runs[prefix] = [None if p.grad is None else p.grad.clone() for p in t.dense] + \
            [grad_as_dense(p) for p in t.rows.params()]

    def same(a, c):
        return (a is None) == (c is None) and (a is None or torch.allclose(a, c, atol=1e-6))

    t.cfg.no_grad_prefix = True
    _clear_grads(t)
    return {"prefix_same": all(same(a, c) for a, c in zip(runs[True], runs[False])),
            "prefix_nonzero": any(a is not None and bool(a.abs().sum() > 0) for a in runs[True])}


def check_resume(t, cfg, out, rank):
    """save -> resume -> next step gives what the uninterrupted run gives."""
    t.global_step, t.step_in_epoch = 1, 1
    t.save_checkpoint()
    t.train_step(t.plan.micro_batches(0, 1, rank))
    straight = snapshot(t)
    again = _trainer({**cfg, "resume_from_checkpoint": os.path.join(out, "checkpoint-1")})
    again._maybe_resume()
    again.train_step(again.plan.micro_batches(0, again.step_in_epoch, rank))
    resumed = snapshot(again)
    return {"resume_same": all(torch.allclose(straight[k], resumed[k], atol=1e-6) for k in straight),
            "resume_step": again.global_step}


def check_meta_loading(cfg, root, rank):
    """cpu_ram_efficient_loading: rank 0 reads the weights, the other ranks get a broadcast."""
    t = _trainer({**cfg, "output_dir": os.path.join(root, "run_b"), "fsdp_config": {"cpu_ram_efficient_loading": True}})
    return {"meta_loss": t.train_step(t.plan.micro_batches(0, 0, rank))["loss"]}


def check_sparse(cfg, root, rank):
    """Sparse (touched rows only) and dense table gradients give the same 3 clipped steps."""
    runs = []
    for sparse in (True, False):
        t = _trainer({**cfg, "output_dir": os.path.join(root, f"run_sp{int(sparse)}"), "sparse_row_grads": sparse,
                      "max_grad_norm": 0.05})
        _randomize_dense(t)
        norms = [t.train_step(t.plan.micro_batches(0, k, rank))["table_grad_norm"] for k in range(3)]
        runs.append((snapshot(t), norms))
    (wa, na), (wb, nb) = runs
    same_w = all(torch.allclose(wa[k], wb[k], atol=1e-6) for k in wa)
    same_n = all(abs(x - y) < 1e-5 * max(1, abs(y)) for x, y in zip(na, nb))
    return {"sparse_same": same_w and same_n, "sparse_norms": na}


def check_mb2(cfg, root, ref, rank):
    """micro_batch_size 2 packs both rows into one; the loss still matches HF on both rows."""
    t = _trainer({**cfg, "output_dir": os.path.join(root, "run_mb2"), "micro_batch_size": 2,
                  "gradient_accumulation_steps": 1})
    micro = t.plan.micro_batches(0, 0, rank)
    return {"mb2": (t.train_step(micro)["loss"], hf_token_mean_loss(ref, [t._micro_batch(x) for x in micro]))}


def check_dense_lr(cfg, root, rank):
    """micro_engram_dense_lr follows the tables' schedule; a new value takes effect on resume."""
    lc = {**cfg, "output_dir": os.path.join(root, "run_lr"), "learning_rate": 5e-3, "micro_engram_dense_lr": 1e-3,
          "lr_scheduler": "cosine", "warmup_steps": 2}
    t = _trainer(lc)
    logs = [t.train_step(t.plan.micro_batches(0, k, rank)) for k in range(3)]
    t.global_step = t.step_in_epoch = 3
    t.save_checkpoint()
    t = _trainer({**lc, "micro_engram_dense_lr": 2e-4, "resume_from_checkpoint": os.path.join(root, "run_lr",
                                                                                               "checkpoint-3")})
    t._maybe_resume()
    logs.append(t.train_step(t.plan.micro_batches(0, 3, rank)))
    return {"lr_ratio": [x["learning_rate"] / x["dense_lr"] if x["dense_lr"] else None for x in logs],
            "lr_seq": [x["learning_rate"] for x in logs]}


def check_train_scales(cfg, root, rank):
    """micro_engram_train_scales: false freezes the scalar_sqrt gate's norm scales."""
    res = {}
    for train in (False, True):
        t = _trainer({**cfg, "output_dir": os.path.join(root, f"run_sc{int(train)}"),
                      "micro_engram_train_scales": train})
        _randomize_dense(t)
        start = {s.layer: s.engram.q_scale.detach().clone() for s in t.slots}
        for k in range(2):
            t.train_step(t.plan.micro_batches(0, k, rank))
        res[f"scales_moved{int(train)}"] = any(not torch.equal(start[s.layer], s.engram.q_scale) for s in t.slots)
        res[f"scales_grad{int(train)}"] = all(s.engram.q_scale.requires_grad == train for s in t.slots)
    return res


def _worker(rank, world, root, model_dir, data):
    from transformers import Gemma4ForCausalLM

    out = os.path.join(root, "run_a")
    cfg = base_cfg(root, model_dir, data, out)
    t = _trainer(cfg)
    ref = Gemma4ForCausalLM.from_pretrained(model_dir, dtype=torch.bfloat16, attn_implementation="eager")
    res = check_first_step(t, ref, rank)
    res.update(check_prefix(t, rank))
    res.update(check_resume(t, cfg, out, rank))
    del t
    res.update(check_meta_loading(cfg, root, rank))
    res.update(check_sparse(cfg, root, rank))
    res.update(check_mb2(cfg, root, ref, rank))
    res.update(check_dense_lr(cfg, root, rank))
    res.update(check_train_scales(cfg, root, rank))
    return res


def _worker_full(rank, world, root, model_dir, data):
    cfg = base_cfg(root, model_dir, data, os.path.join(root, "run_full"), save_steps=2, save_total_limit=2,
                   num_epochs=2, lr_scheduler="cosine", warmup_ratio=0.2, profile_step=2)
    t = _trainer(cfg)
    t.train()
    return {"steps": t.global_step}


@pytest.fixture(scope="module")
def assets(tmp_path_factory):
    root = str(tmp_path_factory.mktemp("train_cpu"))
    model_dir, data = make_assets(root)
    return root, model_dir, data


def test_trainer_two_ranks(assets):
    root, model_dir, data = assets
    res = run_dist(_worker, 2, root, model_dir, data, timeout=900)
    r0 = res[0]
    assert abs(r0["loss"] - r0["ref_loss"]) < 2e-2 * r0["ref_loss"], (r0["loss"], r0["ref_loss"])
    assert all(res[r]["prefix_same"] for r in res) and r0["prefix_nonzero"]
    assert all(res[r]["resume_same"] for r in res) and r0["resume_step"] == 1
    assert abs(r0["meta_loss"] - r0["loss"]) < 1e-4, (r0["meta_loss"], r0["loss"])
    assert all(res[r]["sparse_same"] for r in res) and all(n > 0 for n in r0["sparse_norms"]), r0["sparse_norms"]
    assert abs(r0["mb2"][0] - r0["mb2"][1]) < 2e-2 * r0["mb2"][1], r0["mb2"]
    ratios, seq = r0["lr_ratio"], r0["lr_seq"]
    assert [round(x, 6) for x in ratios[1:3]] == [5.0, 5.0] and abs(ratios[3] - 25.0) < 1e-6, ratios
    assert seq[0] == 0.0 and seq[1] > 0, seq
    assert not r0["scales_moved0"] and r0["scales_grad0"] and r0["scales_moved1"] and r0["scales_grad1"]


def test_trainer_full_run(assets):
    from micro_engram.weights import engram_specs, load_engram_weights

    root, model_dir, data = assets
    run_dist(_worker_full, 2, root, model_dir, data, timeout=900)
    out = os.path.join(root, "run_full")
    ckpts = sorted(d for d in os.listdir(out) if d.startswith("checkpoint-"))
    assert len(ckpts) == 2, ckpts
    conf_path = os.path.join(out, "micro_engram_config.json")
    with open(conf_path) as f:
        specs = engram_specs(json.load(f), conf_path)
    sds = [load_engram_weights(s["weights"], layer=s["layer"]) for s in specs]
    assert len(specs) == 2
    assert all(f"tables.{k}.weight" in sd for sd in sds for k in range(4))
    assert all(sd["tables.0.weight"].shape[0] == 97 and "value.weight" in sd for sd in sds)
    assert all(os.path.isfile(os.path.join(out, "profile", f"rank0_step2.{x}")) for x in ("txt", "json"))
    with open(os.path.join(out, "train_log.jsonl")) as f:
        lines = [json.loads(x) for x in f]
    assert lines and all("loss" in x and "table_grad_norm" in x for x in lines)
    keys = {"loss", "ppl", "grad_norm", "table_grad_norm", "learning_rate", "dense_lr", "epoch", "step", "s_per_step",
            "trained_tokens_per_s"}  # the documented JSONL keys (memory keys are CUDA-only)
    assert all(keys <= set(x) for x in lines), keys - set(lines[0])
    assert [x["step"] for x in lines] == sorted(x["step"] for x in lines)
    assert any(k.startswith("engram_L1/") for k in lines[-1])
