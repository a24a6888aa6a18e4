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


def make_assets(root):
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import Gemma4ForCausalLM, PreTrainedTokenizerFast
    from transformers.models.gemma4.configuration_gemma4 import Gemma4TextConfig

    tk = Tokenizer(models.WordLevel({t: i for i, t in enumerate(SPECIAL + WORDS)}, unk_token="<pad>"))
    tk.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    tok = PreTrainedTokenizerFast(tokenizer_object=tk, pad_token="<pad>", eos_token="<eos>", bos_token="<bos>")
    cfg = Gemma4TextConfig(vocab_size=V, hidden_size=64, intermediate_size=128, num_hidden_layers=4,
                           num_attention_heads=4, num_key_value_heads=2, head_dim=16, global_head_dim=32,
                           layer_types=["sliding_attention", "sliding_attention", "full_attention", "full_attention"],
                           sliding_window=8, hidden_size_per_layer_input=0, max_position_embeddings=1024,
                           final_logit_softcapping=30.0, pad_token_id=0, eos_token_id=1, bos_token_id=2)
    cfg.architectures = ["Gemma4ForCausalLM"]
    torch.manual_seed(0)
    m = Gemma4ForCausalLM(cfg)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if p.dim() == 1:
                p.copy_(1 + 0.2 * torch.randn_like(p))
    model_dir = os.path.join(root, "base")
    m.to(torch.bfloat16).save_pretrained(model_dir)
    tok.save_pretrained(model_dir)
    g = torch.Generator().manual_seed(1)
    rows = []
    for _ in range(40):
        n = int(torch.randint(5, 60, (1,), generator=g))
        rows.append({"text": "<bos> " + " ".join(WORDS[int(i)] for i in torch.randint(0, len(WORDS), (n,), generator=g))})
    data = os.path.join(root, "cpt.jsonl")
    with open(data, "w") as f:
        f.write("\n".join(json.dumps(r) for r in rows))
    torch.save(torch.arange(V) & ~1, os.path.join(root, "canon.pt"))
    return model_dir, data


def base_cfg(root, model_dir, data, out, **over):
    c = {"base_model": model_dir, "datasets": [{"path": data, "type": "completion"}], "sequence_len": 32,
         "output_dir": out, "micro_batch_size": 1, "gradient_accumulation_steps": 2, "num_epochs": 1,
         "learning_rate": 5e-3, "lr_scheduler": "constant", "max_grad_norm": 2.0, "seed": 7,
         "gradient_checkpointing": True, "micro_engram_layer": 1, "micro_engram_table_size": 97,
         "micro_engram_dim": 8, "micro_engram_heads": 2, "micro_engram_gate": "scalar_sqrt",
         "micro_engram_extra": [{"layer": 3}], "micro_engram_optimizer": "rowwise_adam",
         "micro_engram_dtype": "fp32", "micro_engram_canon_path": os.path.join(root, "canon.pt"),
         "micro_engram_stats_steps": 1, "loss_chunk_tokens": 16, "save_steps": None}
    c.update(over)
    return c


def _trainer(cfg):
    from micro_engram.train.config import load_config
    from micro_engram.train.loop import Trainer

    t = Trainer(load_config(cfg))
    t.build()
    return t


def _randomize_dense(t):
    g = torch.Generator().manual_seed(5)
    with torch.no_grad():
        for s in t.slots:
            for _, p in s.engram.named_parameters():
                p.copy_(torch.randn(p.shape, generator=g) * 0.05)


def _state(t):
    out = {}
    for s in t.slots:
        for n, p in s.engram.named_parameters():
            out[f"{s.layer}.{n}"] = p.detach().clone()
        for k, p in enumerate(s.engram.row_shards):
            out[f"{s.layer}.rows{k}"] = p.detach().clone()
    return out


def _dense_grad(p):
    sg = getattr(p, "sparse_grad", None)
    if sg is not None:
        g = torch.zeros(p.shape, dtype=torch.float32)
        g.index_add_(0, sg[0], sg[1].float())
        return g
    return None if p.grad is None else p.grad.float().clone()


def _hf_loss(ref, batches):
    import torch.distributed as dist

    s, c = torch.zeros(()), torch.zeros(())
    with torch.no_grad():
        for b in batches:
            logits = ref(input_ids=b["input_ids"], position_ids=b["position_ids"]).logits.float()
            s += torch.nn.functional.cross_entropy(logits.reshape(-1, V), b["labels"].reshape(-1), ignore_index=-100,
                                                   reduction="sum")
            c += (b["labels"] != -100).sum()
    dist.all_reduce(s)
    dist.all_reduce(c)
    return float(s / c)


def _worker(rank, world, root, model_dir, data):
    from transformers import Gemma4ForCausalLM

    res = {}
    out = os.path.join(root, "run_a")
    cfg = base_cfg(root, model_dir, data, out)
    t = _trainer(cfg)
    micro = t.plan.micro_batches(0, 0, rank)
    ref = Gemma4ForCausalLM.from_pretrained(model_dir, dtype=torch.bfloat16, attn_implementation="eager")
    res["ref_loss"] = _hf_loss(ref, [t._micro_batch(b) for b in micro])
    res["loss"] = t.train_step(micro)["loss"]
    # no-grad prefix: the engram gradients equal a full backward's
    _randomize_dense(t)
    b = t._micro_batch(t.plan.micro_batches(0, 1, rank)[0])

    def grads(prefix):
        t.cfg.no_grad_prefix = prefix
        for p in t.dense:
            p.grad = None
        t.rows.zero_grad()
        t.forward_loss(b, 1.0)
        return [None if p.grad is None else p.grad.clone() for p in t.dense] + [_dense_grad(p) for p in t.rows.params()]

    g1, g0 = grads(True), grads(False)
    res["prefix_same"] = all((a is None and c is None) or (a is not None and c is not None and
                                                          torch.allclose(a, c, atol=1e-6)) for a, c in zip(g1, g0))
    res["prefix_nonzero"] = any(a is not None and a.abs().sum() > 0 for a in g1)
    t.cfg.no_grad_prefix = True
    for p in t.dense:
        p.grad = None
    t.rows.zero_grad()
    # save -> resume -> next step == the uninterrupted run
    t.global_step, t.step_in_epoch = 1, 1
    t.save_checkpoint()
    t.train_step(t.plan.micro_batches(0, 1, rank))
    after = _state(t)
    del t
    t2 = _trainer({**cfg, "resume_from_checkpoint": os.path.join(out, "checkpoint-1")})
    t2._maybe_resume()
    t2.train_step(t2.plan.micro_batches(0, t2.step_in_epoch, rank))
    after2 = _state(t2)
    res["resume_same"] = all(torch.allclose(after[k], after2[k], atol=1e-6) for k in after)
    res["resume_step"] = t2.global_step
    del t2
    # cpu_ram_efficient_loading: rank 0 loads, the others receive a broadcast
    t3 = _trainer({**cfg, "output_dir": os.path.join(root, "run_b"), "fsdp_config": {"cpu_ram_efficient_loading": True}})
    res["meta_loss"] = t3.train_step(t3.plan.micro_batches(0, 0, rank))["loss"]
    del t3
    # sparse row gradients == dense ones (3 clipped steps)
    states = []
    for sparse in (True, False):
        tt = _trainer({**cfg, "output_dir": os.path.join(root, f"run_sp{int(sparse)}"), "sparse_row_grads": sparse,
                       "max_grad_norm": 0.05})
        _randomize_dense(tt)
        norms = [tt.train_step(tt.plan.micro_batches(0, k, rank))["table_grad_norm"] for k in range(3)]
        states.append((_state(tt), norms))
        del tt
    (a, na), (b2, nb) = states
    res["sparse_same"] = all(torch.allclose(a[k], b2[k], atol=1e-6) for k in a) and \
        all(abs(x - y) < 1e-5 * max(1, abs(y)) for x, y in zip(na, nb))
    res["sparse_norms"] = na
    # micro_batch_size 2: rows flattened into one packed row; same loss as HF on both rows
    tm = _trainer({**cfg, "output_dir": os.path.join(root, "run_mb2"), "micro_batch_size": 2,
                   "gradient_accumulation_steps": 1})
    mb = tm.plan.micro_batches(0, 0, rank)
    res["mb2"] = (tm.train_step(mb)["loss"], _hf_loss(ref, [tm._micro_batch(x) for x in mb]))
    del tm
    # micro_engram_dense_lr: same schedule as the tables; a new value applies on resume
    lc = {**cfg, "output_dir": os.path.join(root, "run_lr"), "learning_rate": 5e-3, "micro_engram_dense_lr": 1e-3,
          "lr_scheduler": "cosine", "warmup_steps": 2}
    tl = _trainer(lc)
    l1 = [tl.train_step(tl.plan.micro_batches(0, k, rank)) for k in range(3)]
    tl.global_step = tl.step_in_epoch = 3
    tl.save_checkpoint()
    del tl
    tl = _trainer({**lc, "micro_engram_dense_lr": 2e-4,
                   "resume_from_checkpoint": os.path.join(root, "run_lr", "checkpoint-3")})
    tl._maybe_resume()
    l2 = tl.train_step(tl.plan.micro_batches(0, 3, rank))
    res["lr_ratio"] = [x["learning_rate"] / x["dense_lr"] if x["dense_lr"] else None for x in l1] + \
        [l2["learning_rate"] / l2["dense_lr"]]
    res["lr_seq"] = [x["learning_rate"] for x in l1] + [l2["learning_rate"]]
    del tl
    # micro_engram_train_scales
    for train_scales in (False, True):
        ts = _trainer({**cfg, "output_dir": os.path.join(root, f"run_sc{int(train_scales)}"),
                       "micro_engram_train_scales": train_scales})
        _randomize_dense(ts)
        before = {s.layer: s.engram.q_scale.detach().clone() for s in ts.slots}
        for k in range(2):
            ts.train_step(ts.plan.micro_batches(0, k, rank))
        res[f"scales_moved{int(train_scales)}"] = any(not torch.equal(before[s.layer], s.engram.q_scale)
                                                     for s in ts.slots)
        res[f"scales_grad{int(train_scales)}"] = all(s.engram.q_scale.requires_grad == train_scales for s in ts.slots)
        del ts
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
    assert any(k.startswith("engram_L1/") for k in lines[-1])
