"""Data pipeline, YAML config rules and the vocab-parallel head on CPU.

Data: completion chunking (cut at sequence_len*64, EOS appended, sequence_len chunks), chat
masks (assistant content + its end-of-turn token only), ShareGPT mapping, first-fit packing,
collate (positions restart per document, padding continues the last one, labels shifted and
never across documents), the tokenized-data cache, per-epoch shuffles, distinct bins per rank.
Config: LoRA / unknown keys are errors, Axolotl-only keys are ignored, load_in_8bit refused.
Head: VocabShard's embedding and chunked softcapped loss (and its gradients, with a different
loss weight per rank) against a full-logit reference on 1 and 3 gloo processes, and the chunk
rule that keeps every rank on the same number of chunks. Reference counterparts: test_train.py
(data/config part) and test_head.py."""
import json
import os

import numpy as np
import pytest
import torch

from helpers import run_dist

SPECIAL = ["<pad>", "<eos>", "<bos>", "<|turn>", "<turn|>", "user", "assistant", "system"]
WORDS = [f"w{i}" for i in range(120)]
TEMPLATE = ("{% for m in messages %}<|turn>{{ m.role }} {{ m.content }}<turn|> {% endfor %}"
            "{% if add_generation_prompt %}<|turn>assistant {% endif %}")


@pytest.fixture(scope="module")
def assets(tmp_path_factory):
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast

    root = str(tmp_path_factory.mktemp("data"))
    tk = Tokenizer(models.WordLevel({t: i for i, t in enumerate(SPECIAL + WORDS)}, unk_token="<pad>"))
    tk.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    tok = PreTrainedTokenizerFast(tokenizer_object=tk, pad_token="<pad>", eos_token="<eos>", bos_token="<bos>",
                                  additional_special_tokens=["<|turn>", "<turn|>"])
    tok.chat_template = TEMPLATE
    model_dir = os.path.join(root, "base")
    tok.save_pretrained(model_dir)
    with open(os.path.join(model_dir, "config.json"), "w") as f:
        json.dump({"model_type": "gemma4_text", "vocab_size": len(SPECIAL) + len(WORDS)}, f)
    data = os.path.join(root, "cpt.jsonl")
    g = np.random.default_rng(0)
    with open(data, "w") as f:
        for _ in range(30):
            f.write(json.dumps({"text": "<bos> " + " ".join(g.choice(WORDS, g.integers(5, 50)))}) + "\n")
    return root, model_dir, data, tok


def _cfg(root, model_dir, data, **over):
    c = {"base_model": model_dir, "datasets": [{"path": data, "type": "completion"}], "sequence_len": 32,
         "output_dir": os.path.join(root, "out"), "micro_batch_size": 1, "gradient_accumulation_steps": 2,
         "micro_engram_layer": 1, "seed": 7}
    c.update(over)
    return c


def test_completion_and_chat(assets):
    from micro_engram.train.config import DatasetConfig, load_config
    from micro_engram.train.data import Tokenizing, messages_of

    root, model_dir, data, tok = assets
    t = Tokenizing(tok, load_config(_cfg(root, model_dir, data)))
    long = "<bos> " + " ".join(WORDS[:70])
    ch = t.completion(long)
    ids = tok(long)["input_ids"]
    assert [len(c) for c, _ in ch] == [32, 32, len(ids) + 1 - 64]
    assert ch[-1][0][-1] == tok.eos_token_id and list(ch[0][0]) == ids[:32]
    t2 = Tokenizing(tok, load_config(_cfg(root, model_dir, data, eot_tokens=["<turn|>"])))
    msgs = [{"role": "system", "content": "w1 w2"}, {"role": "user", "content": "w3 w4"},
            {"role": "assistant", "content": "w5 w6 w7"}, {"role": "user", "content": "w8"},
            {"role": "assistant", "content": "w9"}]
    ids, mask = t2.chat(msgs, {"assistant"})
    trained = [tok.convert_ids_to_tokens(int(i)) for i, m in zip(ids, mask) if m]
    assert trained == ["w5", "w6", "w7", "<turn|>", "w9", "<turn|>"], trained
    ds = DatasetConfig(path="x", type="chat_template", field_messages="conversations",
                       message_property_mappings={"role": "from", "content": "value"},
                       roles={"assistant": ["gpt"], "user": ["human"]})
    got = messages_of({"conversations": [{"from": "human", "value": "a"}, {"from": "gpt", "value": "b"}]}, ds)
    assert got == [{"role": "user", "content": "a"}, {"role": "assistant", "content": "b"}]


def test_pack_collate_cache_plan(assets):
    from micro_engram.train.config import load_config
    from micro_engram.train.data import EpochPlan, Samples, collate, pack, prepare

    root, model_dir, data, tok = assets
    s = Samples.from_list([([1, 2, 3], None), ([4, 5], np.array([False, True])), ([6] * 30, None)])
    bins = pack(s.lengths(), 32, seed=0)
    assert sorted(i for b in bins for i in b) == [0, 1, 2]
    assert all(sum(s.lengths()[i] for i in b) <= 32 for b in bins)
    b = collate(s, [[0, 1]], 8, pad_id=0)
    assert b["position_ids"][0].tolist() == [0, 1, 2, 0, 1, 2, 3, 4]
    assert b["labels"][0].tolist() == [2, 3, -100, 5, -100, -100, -100, -100]
    prep = os.path.join(root, "prep")
    c3 = load_config(_cfg(root, model_dir, data, dataset_prepared_path=prep))
    a = prepare(c3, tok, model_dir)
    a2 = prepare(c3, tok, model_dir)
    assert np.array_equal(a.tokens, a2.tokens) and np.array_equal(a.offsets, a2.offsets)
    assert len(os.listdir(prep)) == 1
    plan = EpochPlan(a, c3, world=2)
    assert plan.bins(0) != plan.bins(1)
    flat = [tuple(x) for r in (0, 1) for m in plan.micro_batches(0, 0, r) for x in m]
    assert len(flat) == len(set(flat)) == 4


def test_config_rules(assets):
    from micro_engram.train.config import load_config

    root, model_dir, data, _ = assets
    for bad in ({"adapter": "qlora"}, {"lora_r": 1}, {"unfrozen_parameters": [".+x"]}, {"no_such_key": 1},
                {"load_in_8bit": True}):
        with pytest.raises(Exception):
            load_config(_cfg(root, model_dir, data, **bad))
    c = load_config(_cfg(root, model_dir, data, plugins=["x"], strict=False, bf16="auto", fsdp_version=2,
                         fsdp_config={"offload_params": True, "state_dict_type": "SHARDED"}))
    assert c.fsdp_config.offload_params


def test_vocab_chunk_rule():
    from micro_engram.train.head import VocabShard

    W = torch.zeros(262_144, 8)
    chunks = {VocabShard(W, r, 5).chunk for r in range(5)}  # 52,429 rows on ranks 0-3, 52,428 on rank 4
    assert len(chunks) == 1, chunks


def _head_worker(rank, world):
    from micro_engram.train.head import VocabShard, reference_loss_sum

    torch.manual_seed(0)
    V, d, N = 103, 16, 37
    W = torch.randn(V, d, dtype=torch.float64)
    Hs = torch.randn(world, N, d, dtype=torch.float64)
    Ls = torch.randint(0, V, (world, N))
    Ls[:, ::5] = -100
    ok = True
    for cap in (None, 3.0):
        sh = VocabShard(W, rank, world, embed_scale=2.0, softcap=cap, chunk_tokens=8)
        h = Hs[rank].clone().requires_grad_()
        tot, cnt = sh.loss_sum(h, Ls[rank])
        (tot * (rank + 1)).backward()
        ref_h = Hs[rank].clone().requires_grad_()
        ref = reference_loss_sum(ref_h, Ls[rank], W, cap)
        (ref * (rank + 1)).backward()
        ok &= bool(torch.allclose(tot, ref)) and bool(torch.allclose(h.grad, ref_h.grad, atol=1e-5))
        ok &= int(cnt) == int((Ls[rank] != -100).sum())
    ids = torch.randint(0, V, (2, 9)) + rank
    ids = ids.clamp_max(V - 1)
    ok &= bool(torch.allclose(sh.embed(ids), W[ids] * 2.0))
    return ok


@pytest.mark.parametrize("world", [1, 3])
def test_vocab_parallel_head(world):
    res = run_dist(_head_worker, world)
    assert all(res.values()), res


def test_packing_order_is_pinned():
    """The packing order is part of the contract (a resumed run, or a run compared with the
    reference trainer, must see the same bins): a fixed input packs to a recorded result."""
    import hashlib

    from micro_engram.train.data import pack

    lens = np.random.default_rng(2024).integers(0, 600, size=500)
    bins = pack(lens, 512, 11)
    assert hashlib.sha256(json.dumps(bins).encode()).hexdigest()[:16] == "a9436382b82cb5d7"
    assert sorted(i for b in bins for i in b) == [i for i in range(500) if 0 < lens[i] <= 512]


def test_every_lr_schedule():
    """Each lr_scheduler value (and the epoch decay) builds and follows its curve over 10 steps
    with 2 warmup steps; warmup_stable_decay without its decay length is refused at load."""
    import types

    import pytest
    import torch

    from micro_engram.train.config import TrainConfig
    from micro_engram.train.loop import Trainer

    def lrs(**kw):
        base = dict(base_model="x", datasets=[{"path": "d.jsonl", "type": "completion"}], output_dir="o",
                    learning_rate=1.0, warmup_steps=2)
        cfg = TrainConfig(**{**base, **kw})
        opt = torch.optim.SGD([torch.nn.Parameter(torch.zeros(1))], lr=1.0)
        sched = Trainer._make_scheduler(types.SimpleNamespace(cfg=cfg, dense_opt=opt, total_steps=10))
        out = []
        for _ in range(10):
            out.append(round(opt.param_groups[0]["lr"], 3))
            opt.step()
            sched.step()
        return out

    assert lrs(lr_scheduler="constant") == [1.0] * 10  # never warms up
    assert lrs(lr_scheduler="constant_with_warmup") == [0.0, 0.5] + [1.0] * 8
    assert lrs(lr_scheduler="linear") == [0.0, 0.5, 1.0, 0.875, 0.75, 0.625, 0.5, 0.375, 0.25, 0.125]
    cos = lrs(lr_scheduler="cosine")
    assert cos[:3] == [0.0, 0.5, 1.0] and cos[6] == 0.5 and cos[-1] < 0.05
    assert lrs(lr_scheduler="cosine", cosine_min_lr_ratio=0.1)[-1] > cos[-1]
    assert lrs(lr_scheduler="warmup_stable_decay", lr_scheduler_kwargs={"num_decay_steps": 4})[:7] == \
        [0.0, 0.5, 1.0, 1.0, 1.0, 1.0, 1.0]
    assert lrs(micro_engram_lr_epoch_decay=0.5, num_epochs=2) == [0.0, 0.5, 1.0, 1.0, 1.0] + [0.5] * 5
    with pytest.raises(ValueError, match="num_decay_steps"):
        TrainConfig(base_model="x", datasets=[{"path": "d.jsonl", "type": "completion"}], output_dir="o",
                    lr_scheduler="warmup_stable_decay")


def test_example_configs_load():
    """The example YAMLs in examples/ pass the config rules and the engram request rules."""
    import glob
    import os

    from micro_engram.runconfig import engram_requests
    from micro_engram.train.config import load_config

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    paths = sorted(glob.glob(os.path.join(root, "examples", "*.yaml")))
    assert paths
    for path in paths:
        reqs = engram_requests(load_config(path))
        assert reqs and all(r.spec["layer"] >= 0 for r in reqs), path
