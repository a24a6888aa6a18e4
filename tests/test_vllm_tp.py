"""Engram tables split across tensor-parallel ranks for serving (micro_engram_vllm.tp and
micro_engram_vllm.model), on gloo CPU processes with small stand-ins for the vLLM classes the
plugin builds on. 3 ranks and 31-row tables give an uneven split (11/11/9). Reference
counterpart: test_vllm_tp.py."""
import json
import logging
import os
import sys
import types

import pytest
import torch
import torch.nn as nn

from helpers import run_dist

D, V, N, E, LAYER = 16, 50, 31, 4, 1


def _full(dtype=torch.float32):
    from micro_engram.module import MicroEngram

    torch.manual_seed(0)
    eng = MicroEngram(model_dim=D, table_size=N, engram_dim=E, num_heads=2, vocab_size=V, gate="scalar_sqrt")
    with torch.no_grad():
        eng.value.weight.normal_(std=0.3)
        eng.q_scale.fill_(0.25)  # delta storage: scale 1.25
    return eng.to(dtype)


def _history(seed, n=24, width=3):
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(5, V, (n, width), generator=g)
    ids[:3, 1:] = -1
    return ids


def _all_reduce(t):
    import torch.distributed as dist

    dist.all_reduce(t)
    return t


_UVA = [True]
_VIEWS = []


def _install_vllm_stand_ins():
    """Module paths and base classes the plugin imports, each as small as the test needs."""
    import torch.distributed as dist

    def mod(name, **attrs):
        m = types.ModuleType(name)
        m.__dict__.update(attrs)
        sys.modules[name] = m
        return m

    class Gemma4DecoderLayer(nn.Module):
        def __init__(self):
            super().__init__()
            self.lin = nn.Linear(D, D)

        def forward(self, positions, hidden_states, residual, per_layer_input=None, **kw):
            return torch.tanh(self.lin(hidden_states)), residual

    class Gemma4ForCausalLM(nn.Module):
        def __init__(self, *, vllm_config, prefix=""):
            super().__init__()
            torch.manual_seed(5)
            self.config = types.SimpleNamespace(hidden_size=D, vocab_size=V, pad_token_id=0)
            self.model = nn.Module()
            self.model.layers = nn.ModuleList(Gemma4DecoderLayer() for _ in range(3))

        def load_weights(self, weights):
            params, done = dict(self.named_parameters()), set()
            for name, w in weights:
                if name not in params:
                    raise KeyError(f"the stand-in loader has no parameter {name}")
                with torch.no_grad():
                    params[name].copy_(w)
                done.add(name)
            return done

    mod("vllm")
    mod("vllm.config", VllmConfig=object)
    mod("vllm.logger", init_logger=logging.getLogger)
    mod("vllm.distributed",
        get_tensor_model_parallel_rank=lambda: dist.get_rank() if dist.is_initialized() else 0,
        get_tensor_model_parallel_world_size=lambda: dist.get_world_size() if dist.is_initialized() else 1,
        get_tp_group=lambda: types.SimpleNamespace(cpu_group=None),
        tensor_model_parallel_all_reduce=_all_reduce)
    mod("vllm.model_executor")
    mod("vllm.model_executor.models")
    mod("vllm.model_executor.models.gemma4", Gemma4DecoderLayer=Gemma4DecoderLayer,
        Gemma4ForCausalLM=Gemma4ForCausalLM)
    mod("vllm.model_executor.models.gemma4_mm", Gemma4ForConditionalGeneration=nn.Module)
    mod("vllm.model_executor.models.utils", PPMissingLayer=type("PPMissingLayer", (nn.Module,), {}))
    mod("vllm.utils")
    mod("vllm.utils.platform_utils", is_uva_available=lambda: _UVA[0])
    mod("vllm.utils.torch_utils", get_accelerator_view_from_cpu_tensor=lambda t: _VIEWS.append(t) or t)


def _cfg(conf=None, model_dir="/nonexistent"):
    return types.SimpleNamespace(
        additional_config={"micro_engram": conf} if conf else {},
        model_config=types.SimpleNamespace(architecture="Gemma4ForCausalLM", model=model_dir),
        use_v2_model_runner=True,
        scheduler_config=types.SimpleNamespace(max_num_batched_tokens=64))


def _lookup_worker(rank, world):
    from micro_engram.module import MicroEngram
    from micro_engram.rows import row_range
    from micro_engram_vllm.tp import load_rows, tp_lookup

    res = {}
    start, count = row_range(N, rank, world)
    for dtype in (torch.float32, torch.bfloat16):
        full = _full(dtype)
        sh = MicroEngram(model_dim=D, table_size=N, engram_dim=E, num_heads=2, vocab_size=V, gate="scalar_sqrt",
                         build_tables=False).to(dtype)
        sh.shard_rows(rank, world, dtype=dtype, requires_grad=False, empty=True)
        sh.row_lookup_fn = tp_lookup(_all_reduce)
        load_rows(sh, full.state_dict(), "test")
        h = torch.randn(24, D).to(dtype) * 5
        idx = full.hash_prev(_history(1))
        res[f"exact {dtype}"] = torch.equal(sh.inject(h, idx), full.inject(h, idx))
        res[f"rows {dtype}"] = sh.row_shards[0].shape[0] == count
    # mixed table sizes with 4-grams: every table split on its own
    torch.manual_seed(4)
    sizes = {2: 31, 3: 47, 4: 13}
    fm = MicroEngram(model_dim=D, table_size=N, engram_dim=E, num_heads=2, vocab_size=V, gate="scalar_sqrt",
                     orders=(2, 3, 4), table_sizes=sizes)
    with torch.no_grad():
        fm.value.weight.normal_(std=0.3)
    sm = MicroEngram(model_dim=D, table_size=N, engram_dim=E, num_heads=2, vocab_size=V, gate="scalar_sqrt",
                     orders=(2, 3, 4), table_sizes=sizes, build_tables=False)
    sm.shard_rows(rank, world, requires_grad=False, empty=True)
    sm.row_lookup_fn = tp_lookup(_all_reduce)
    load_rows(sm, fm.state_dict(), "mixed")
    hm = torch.randn(24, D) * 5
    im = fm.hash_prev(_history(9, width=4))
    res["mixed exact"] = torch.equal(sm.inject(hm, im), fm.inject(hm, im))
    res["mixed split"] = [p.shape[0] for p in sm.row_shards] == [row_range(r, rank, world)[1] for r in fm.table_rows]
    # loading in two pieces; refusals
    full = _full()
    sd = full.state_dict()
    sh = MicroEngram(model_dim=D, table_size=N, engram_dim=E, num_heads=2, vocab_size=V, gate="scalar_sqrt",
                     build_tables=False)
    sh.shard_rows(rank, world, requires_grad=False, empty=True)
    first = {k: v for k, v in sd.items() if k in ("tables.0.weight", "tables.1.weight", "key.weight")}
    rest = {k: v for k, v in sd.items() if k not in first}
    got = load_rows(sh, first, "part 1", complete=False) | load_rows(sh, rest, "part 2", complete=False)
    res["two pieces"] = (got == {0, 1, 2, 3}
                         and all(torch.equal(p, full.tables[k].weight[start:start + count])
                                 for k, p in enumerate(sh.row_shards))
                         and torch.allclose(sh.q_scale, torch.full((D,), 0.25)))
    for bad, what in (({k: v for k, v in sd.items() if k != "tables.2.weight"}, "missing tables"),
                      ({**sd, "tables.0.weight": torch.zeros(N + 1, E)}, "is (32, 4)")):
        try:
            load_rows(sh, bad, "bad")
            res[f"refused {what}"] = False
        except ValueError as e:
            res[f"refused {what}"] = what in str(e)
    return res


def _model_worker(rank, world, tmp):
    import torch.distributed as dist

    _install_vllm_stand_ins()
    from micro_engram_vllm.model import EngramGemma4ForCausalLM

    res = {}
    start, count = __import__("micro_engram.rows", fromlist=["row_range"]).row_range(N, rank, world)
    full = _full()
    ids = _history(2)
    h = torch.randn(24, D)
    conf = {"layer": LAYER, "table_size": N, "engram_dim": E, "num_heads": 2, "gate": "scalar_sqrt", "seed": 0,
            "orders": [2, 3], "pad_id": 0, "model_dim": D, "vocab_size": V}
    engram_sd = {f"model.layers.{LAYER}.micro_engram.{k}": v for k, v in full.state_dict().items()}
    for mode in ("file", "checkpoint"):
        if mode == "file":
            folder = os.path.join(tmp, "file")
            if rank == 0:
                os.makedirs(folder, exist_ok=True)
                torch.save(engram_sd, os.path.join(folder, "engram.pt"))
                with open(os.path.join(folder, "micro_engram_config.json"), "w") as f:
                    json.dump({**conf, "weights": "engram.pt"}, f)
            dist.barrier()
            model = EngramGemma4ForCausalLM(vllm_config=_cfg(os.path.join(folder, "micro_engram_config.json")))
            base_sd = {k: v + 1 for k, v in model.state_dict().items() if ".micro_engram." not in k}
            stale = {f"model.layers.{LAYER}.micro_engram.tables.0.weight": torch.zeros(N, E)}
            loaded = model.load_weights(iter([*base_sd.items(), *stale.items()]))
        else:
            folder = os.path.join(tmp, "assembled")
            if rank == 0:
                os.makedirs(folder, exist_ok=True)
                with open(os.path.join(folder, "micro_engram_config.json"), "w") as f:
                    json.dump(conf, f)
            dist.barrier()
            model = EngramGemma4ForCausalLM(vllm_config=_cfg(model_dir=folder))
            base_sd = {k: v + 1 for k, v in model.state_dict().items() if ".micro_engram." not in k}
            stream = list(base_sd.items()) + list(engram_sd.items())
            half = len(stream) // 2
            loaded = model.load_weights(iter(stream[:half])) | model.load_weights(iter(stream[half:]))
        layer = model.model.layers[LAYER]
        eng = layer.micro_engram
        res[f"{mode}: tables hidden from the loader, 1/TP rows"] = (
            not any(".tables." in n for n, _ in model.named_parameters())
            and sum(p.numel() for p in eng.row_shards) == 4 * count * E)
        want = {f"model.layers.{LAYER}.micro_engram.{n}" for n in ("key.weight", "value.weight", "q_scale", "k_scale")}
        res[f"{mode}: loaded names reported"] = want <= loaded and set(base_sd) <= loaded
        layer.micro_engram_ids.copy_(torch.cat([ids, torch.full((64 - 24, 3), -1)]).to(torch.int32))
        out, _ = layer(None, h, None)
        ref = full.inject(torch.tanh(layer.lin(h)), full.hash_prev(ids))
        res[f"{mode}: layer == base + full-table engram"] = torch.allclose(out, ref, atol=1e-6)
    # host offload through (stand-in) UVA views
    folder = os.path.join(tmp, "file")
    cfg = _cfg(os.path.join(folder, "micro_engram_config.json"))
    cfg.additional_config["micro_engram_offload"] = True
    _VIEWS.clear()
    model = EngramGemma4ForCausalLM(vllm_config=cfg)
    model.load_weights(iter({k: v + 1 for k, v in model.state_dict().items() if ".micro_engram." not in k}.items()))
    layer = model.model.layers[LAYER]
    eng = layer.micro_engram
    res["offload: rows on the host, one view per table"] = (
        all(p.device.type == "cpu" for p in eng.row_shards) and len(_VIEWS) == len(eng.row_shards)
        and all(v.data_ptr() == p.data_ptr() for v, p in zip(eng.row_views, eng.row_shards)))
    layer.micro_engram_ids.copy_(torch.cat([ids, torch.full((64 - 24, 3), -1)]).to(torch.int32))
    out, _ = layer(None, h, None)
    res["offload: layer == full-table engram"] = torch.allclose(
        out, full.inject(torch.tanh(layer.lin(h)), full.hash_prev(ids)), atol=1e-6)
    _UVA[0] = False
    try:
        EngramGemma4ForCausalLM(vllm_config=cfg)
        res["offload refused without UVA"] = False
    except RuntimeError as e:
        res["offload refused without UVA"] = "UVA" in str(e)
    _UVA[0] = True
    os.environ["MICRO_ENGRAM_OFFLOAD"] = "1"
    m_env = EngramGemma4ForCausalLM(vllm_config=_cfg(os.path.join(folder, "micro_engram_config.json")))
    del os.environ["MICRO_ENGRAM_OFFLOAD"]
    res["MICRO_ENGRAM_OFFLOAD=1"] = m_env.model.layers[LAYER].micro_engram.__dict__.get("row_views") is not None
    os.environ["MICRO_ENGRAM_OFF"] = "1"
    m_off = EngramGemma4ForCausalLM(vllm_config=_cfg(os.path.join(folder, "micro_engram_config.json")))
    del os.environ["MICRO_ENGRAM_OFF"]
    lo = m_off.model.layers[LAYER]
    res["MICRO_ENGRAM_OFF=1 skips the engram"] = torch.equal(lo(None, h, None)[0], torch.tanh(lo.lin(h)))
    plain = EngramGemma4ForCausalLM(vllm_config=_cfg())
    res["no config: plain model"] = plain.micro_engram_ids is None and not plain.micro_engram_slots
    return res


@pytest.mark.parametrize("world", [3, 1])
def test_tp_lookup_and_loading(world):
    for rank, res in run_dist(_lookup_worker, world).items():
        bad = [k for k, ok in res.items() if not ok]
        assert not bad, f"rank {rank}: {bad}"


@pytest.mark.parametrize("world", [3, 1])
def test_plugin_model_with_stand_ins(world, tmp_path):
    for rank, res in run_dist(_model_worker, world, str(tmp_path)).items():
        bad = [k for k, ok in res.items() if not ok]
        assert not bad, f"rank {rank}: {bad}"


def test_model_state_attach_fills_history():
    """The state wrapper installed by register(): any built model state gets the fill."""
    from micro_engram_vllm.model_state import attach

    class State:
        max_num_tokens = 8

        def prepare_inputs(self, batch, req):
            return {"x": 1}

    model = types.SimpleNamespace(micro_engram_ids=torch.full((8, 3), 5, dtype=torch.int32))
    st = attach(State(), model)
    batch = types.SimpleNamespace(input_ids=torch.tensor([7, 8, 9, 0], dtype=torch.int32),
                                  positions=torch.tensor([0, 1, 2, 0]), idx_mapping=torch.tensor([0], dtype=torch.int32),
                                  query_start_loc=torch.tensor([0, 3], dtype=torch.int32), num_reqs=1, num_tokens=3,
                                  num_tokens_after_padding=4)
    req = types.SimpleNamespace(all_token_ids=types.SimpleNamespace(gpu=torch.zeros(1, 16, dtype=torch.int32)))
    assert st.prepare_inputs(batch, req) == {"x": 1}
    want = torch.tensor([[7, -1, -1], [8, 7, -1], [9, 8, 7], [-1, -1, -1]], dtype=torch.int32)
    assert torch.equal(model.micro_engram_ids[:4], want) and bool((model.micro_engram_ids[4:] == 5).all())
    assert attach(st, model) is st
    plain = State()
    assert attach(plain, types.SimpleNamespace()) is plain
