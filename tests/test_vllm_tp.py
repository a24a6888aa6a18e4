"""Serving with engram tables split over tensor-parallel ranks (micro_engram_vllm.tp and
micro_engram_vllm.model), on gloo CPU processes.

vLLM itself cannot run here, so the plugin is imported against a minimal fake of the vLLM
modules it uses (`fake_vllm`): a decoder layer that is a tanh(Linear), a causal-LM shell with
a name-checking weight loader, and the TP helpers backed by the test's process group. 3 ranks
with 31-row tables give an uneven row split (11/11/9); world 1 is the degenerate case."""
import contextlib
import json
import logging
import os
import sys
import types
from unittest import mock

import pytest
import torch
import torch.nn as nn

from helpers import run_dist

DIM, VOCAB, ROWS, EDIM, LAYER = 16, 50, 31, 4, 1
UVA = {"available": True, "views": []}


def trained_engram(dtype=torch.float32, **kw):
    """A small trained-looking engram: random tables, a non-zero output projection, q scale 1.25."""
    from micro_engram.module import MicroEngram

    torch.manual_seed(0)
    e = MicroEngram(model_dim=DIM, table_size=ROWS, engram_dim=EDIM, num_heads=2, vocab_size=VOCAB,
                    gate="scalar_sqrt", **kw)
    with torch.no_grad():
        e.value.weight.normal_(std=0.3)
        e.q_scale.fill_(0.25)  # stored as a delta: scale 1.25
    return e.to(dtype)


def empty_shards(rank, world, dtype=torch.float32, **kw):
    from micro_engram.module import MicroEngram

    e = MicroEngram(model_dim=DIM, table_size=ROWS, engram_dim=EDIM, num_heads=2, vocab_size=VOCAB,
                    gate="scalar_sqrt", build_tables=False, **kw).to(dtype)
    e.shard_rows(rank, world, dtype=dtype, requires_grad=False, empty=True)
    return e


def histories(seed, n=24, width=3):
    """[n, width] previous-token ids; the first rows lack older history (-1)."""
    ids = torch.randint(5, VOCAB, (n, width), generator=torch.Generator().manual_seed(seed))
    ids[:3, 1:] = -1
    return ids


def summed(t):
    import torch.distributed as dist

    dist.all_reduce(t)
    return t


# ---------------------------------------------------------------------------- fake vLLM
class FakeDecoderLayer(nn.Module):
    def __init__(self):
        super().__init__()
        self.lin = nn.Linear(DIM, DIM)

    def forward(self, positions, hidden_states, residual, per_layer_input=None, **kw):
        return torch.tanh(self.lin(hidden_states)), residual


class FakeCausalLM(nn.Module):
    def __init__(self, *, vllm_config, prefix=""):
        super().__init__()
        torch.manual_seed(5)
        self.config = types.SimpleNamespace(hidden_size=DIM, vocab_size=VOCAB, pad_token_id=0)
        self.model = nn.Module()
        self.model.layers = nn.ModuleList([FakeDecoderLayer() for _ in range(3)])

    def load_weights(self, weights):
        named = dict(self.named_parameters())
        loaded = set()
        for name, tensor in weights:
            assert name in named, f"the fake loader got an unknown tensor {name}"
            with torch.no_grad():
                named[name].copy_(tensor)
            loaded.add(name)
        return loaded


def fake_vllm():
    """sys.modules entries for every vLLM module path the plugin imports."""
    import torch.distributed as dist

    def module(name, **members):
        m = types.ModuleType(name)
        for k, v in members.items():
            setattr(m, k, v)
        return m

    def tp_rank():
        return dist.get_rank() if dist.is_initialized() else 0

    def tp_size():
        return dist.get_world_size() if dist.is_initialized() else 1

    def uva_view(t):
        UVA["views"].append(t)
        return t

    tree = {
        "vllm": {}, "vllm.model_executor": {}, "vllm.model_executor.models": {}, "vllm.utils": {},
        "vllm.config": {"VllmConfig": object},
        "vllm.logger": {"init_logger": logging.getLogger},
        "vllm.distributed": {"get_tensor_model_parallel_rank": tp_rank, "get_tensor_model_parallel_world_size": tp_size,
                             "get_tp_group": lambda: types.SimpleNamespace(cpu_group=None),
                             "tensor_model_parallel_all_reduce": summed},
        "vllm.model_executor.models.gemma4": {"Gemma4DecoderLayer": FakeDecoderLayer,
                                              "Gemma4ForCausalLM": FakeCausalLM},
        "vllm.model_executor.models.gemma4_mm": {"Gemma4ForConditionalGeneration": nn.Module},
        "vllm.model_executor.models.utils": {"PPMissingLayer": type("PPMissingLayer", (nn.Module,), {})},
        "vllm.utils.platform_utils": {"is_uva_available": lambda: UVA["available"]},
        "vllm.utils.torch_utils": {"get_accelerator_view_from_cpu_tensor": uva_view},
    }
    return {name: module(name, **members) for name, members in tree.items()}


@contextlib.contextmanager
def vllm_faked():
    """The fake vLLM modules in sys.modules for the duration; afterwards the real entries (or
    none) come back and the plugin modules that bound the fakes are dropped. Everything else
    imported meanwhile stays imported: dropping it too (mock.patch.dict(sys.modules) would) makes
    the next import re-run modules that register torch libraries, which torch refuses."""
    fakes = fake_vllm()
    saved = {name: sys.modules.get(name) for name in fakes}
    sys.modules.update(fakes)
    try:
        yield
    finally:
        for name, mod in saved.items():
            if mod is None:
                sys.modules.pop(name, None)
            else:
                sys.modules[name] = mod
        sys.modules.pop("micro_engram_vllm.model", None)


def serving_config(conf_path=None, model_dir="/nonexistent", **extra):
    additional = {"micro_engram": conf_path} if conf_path else {}
    additional.update(extra)
    return types.SimpleNamespace(
        additional_config=additional, use_v2_model_runner=True,
        model_config=types.SimpleNamespace(architecture="Gemma4ForCausalLM", model=model_dir),
        scheduler_config=types.SimpleNamespace(max_num_batched_tokens=64))


# ---------------------------------------------------------------------------- TP lookup
def _lookup_checks(rank, world):
    from micro_engram.module import MicroEngram
    from micro_engram.rows import row_range
    from micro_engram_vllm.tp import load_rows, tp_lookup

    start, count = row_range(ROWS, rank, world)
    out = {}
    for dtype in (torch.float32, torch.bfloat16):
        full = trained_engram(dtype)
        part = empty_shards(rank, world, dtype)
        part.row_lookup_fn = tp_lookup(summed)
        load_rows(part, full.state_dict(), "test")
        h = torch.randn(24, DIM).to(dtype) * 5
        idx = full.hash_prev(histories(1))
        out[f"masked lookup + all-reduce == full table ({dtype})"] = torch.equal(part.inject(h, idx),
                                                                                full.inject(h, idx))
        out[f"1/TP rows ({dtype})"] = part.row_shards[0].shape[0] == count
    # per-order sizes with 4-grams: each table split on its own
    sizes = {2: 31, 3: 47, 4: 13}
    torch.manual_seed(4)
    full = MicroEngram(model_dim=DIM, table_size=ROWS, engram_dim=EDIM, num_heads=2, vocab_size=VOCAB,
                       gate="scalar_sqrt", orders=(2, 3, 4), table_sizes=sizes)
    with torch.no_grad():
        full.value.weight.normal_(std=0.3)
    part = empty_shards(rank, world, orders=(2, 3, 4), table_sizes=sizes)
    part.row_lookup_fn = tp_lookup(summed)
    load_rows(part, full.state_dict(), "mixed")
    h = torch.randn(24, DIM) * 5
    idx = full.hash_prev(histories(9, width=4))
    out["mixed sizes: exact"] = torch.equal(part.inject(h, idx), full.inject(h, idx))
    out["mixed sizes: split per table"] = ([p.shape[0] for p in part.row_shards] ==
                                           [row_range(n, rank, world)[1] for n in full.table_rows])
    # a state dict arriving in two pieces, and what is refused
    full = trained_engram()
    sd = full.state_dict()
    part = empty_shards(rank, world)
    piece = {k: sd[k] for k in ("tables.0.weight", "tables.1.weight", "key.weight")}
    got = load_rows(part, piece, "piece 1", complete=False)
    got |= load_rows(part, {k: v for k, v in sd.items() if k not in piece}, "piece 2", complete=False)
    out["two pieces"] = (got == {0, 1, 2, 3}
                         and all(torch.equal(p, full.tables[k].weight[start:start + count])
                                 for k, p in enumerate(part.row_shards))
                         and torch.allclose(part.q_scale, torch.full((DIM,), 0.25)))
    for bad, reason in (({k: v for k, v in sd.items() if k != "tables.2.weight"}, "missing tables"),
                        ({**sd, "tables.0.weight": torch.zeros(ROWS + 1, EDIM)}, "is (32, 4)")):
        try:
            load_rows(part, bad, "bad")
            out[f"refuses: {reason}"] = False
        except ValueError as e:
            out[f"refuses: {reason}"] = reason in str(e)
    return out


# ---------------------------------------------------------------------------- the plugin model
def _write(folder, name, obj, rank):
    import torch.distributed as dist

    if rank == 0:
        os.makedirs(folder, exist_ok=True)
        path = os.path.join(folder, name)
        if name.endswith(".json"):
            with open(path, "w") as f:
                json.dump(obj, f)
        else:
            torch.save(obj, path)
    dist.barrier()


def _layer_matches(model, full, ids, h):
    layer = model.model.layers[LAYER]
    layer.micro_engram_ids.copy_(torch.cat([ids, torch.full((64 - ids.shape[0], 3), -1)]).to(torch.int32))
    out, _ = layer(None, h, None)
    return torch.allclose(out, full.inject(torch.tanh(layer.lin(h)), full.hash_prev(ids)), atol=1e-6)


def _model_checks(rank, world, tmp):
    from micro_engram.rows import row_range

    with vllm_faked():
        sys.modules.pop("micro_engram_vllm.model", None)
        from micro_engram_vllm.model import EngramGemma4ForCausalLM

        _, count = row_range(ROWS, rank, world)
        full, ids, h = trained_engram(), histories(2), torch.randn(24, DIM)
        conf = {"layer": LAYER, "table_size": ROWS, "engram_dim": EDIM, "num_heads": 2, "gate": "scalar_sqrt",
                "seed": 0, "orders": [2, 3], "pad_id": 0, "model_dim": DIM, "vocab_size": VOCAB}
        engram_sd = {f"model.layers.{LAYER}.micro_engram.{k}": v for k, v in full.state_dict().items()}
        out = {}

        def base_weights(model):
            return {k: v + 1 for k, v in model.state_dict().items() if ".micro_engram." not in k}

        def check(label, model, loaded, base):
            eng = model.model.layers[LAYER].micro_engram
            out[f"{label}: tables hidden from vLLM's loader, 1/TP of the rows here"] = (
                not any(".tables." in n for n, _ in model.named_parameters())
                and sum(p.numel() for p in eng.row_shards) == 4 * count * EDIM)
            dense = {f"model.layers.{LAYER}.micro_engram.{n}" for n in ("key.weight", "value.weight", "q_scale",
                                                                         "k_scale")}
            out[f"{label}: loaded names reported"] = dense <= loaded and set(base) <= loaded
            out[f"{label}: layer == base + full-table engram"] = _layer_matches(model, full, ids, h)

        # engram weights in their own file (a stale engram inside the checkpoint is ignored)
        files = os.path.join(tmp, "file")
        _write(files, "engram.pt", engram_sd, rank)
        _write(files, "micro_engram_config.json", {**conf, "weights": "engram.pt"}, rank)
        conf_path = os.path.join(files, "micro_engram_config.json")
        model = EngramGemma4ForCausalLM(vllm_config=serving_config(conf_path))
        base = base_weights(model)
        stale = {f"model.layers.{LAYER}.micro_engram.tables.0.weight": torch.zeros(ROWS, EDIM)}
        check("own file", model, model.load_weights(iter([*base.items(), *stale.items()])), base)
        # an assembled checkpoint carrying the engram, loaded in two calls
        assembled = os.path.join(tmp, "assembled")
        _write(assembled, "micro_engram_config.json", conf, rank)
        model = EngramGemma4ForCausalLM(vllm_config=serving_config(model_dir=assembled))
        base = base_weights(model)
        stream = [*base.items(), *engram_sd.items()]
        cut = len(stream) // 2
        loaded = model.load_weights(iter(stream[:cut])) | model.load_weights(iter(stream[cut:]))
        check("in the checkpoint", model, loaded, base)
        # rows in pinned host memory behind (fake) UVA views
        UVA["views"].clear()
        model = EngramGemma4ForCausalLM(vllm_config=serving_config(conf_path, micro_engram_offload=True))
        model.load_weights(iter(base_weights(model).items()))
        eng = model.model.layers[LAYER].micro_engram
        out["offload: host rows, one view per table"] = (
            all(p.device.type == "cpu" for p in eng.row_shards) and len(UVA["views"]) == len(eng.row_shards)
            and all(v.data_ptr() == p.data_ptr() for v, p in zip(eng.row_views, eng.row_shards)))
        out["offload: layer == full-table engram"] = _layer_matches(model, full, ids, h)
        UVA["available"] = False
        try:
            EngramGemma4ForCausalLM(vllm_config=serving_config(conf_path, micro_engram_offload=True))
            out["offload needs UVA"] = False
        except RuntimeError as e:
            out["offload needs UVA"] = "UVA" in str(e)
        finally:
            UVA["available"] = True
        with mock.patch.dict(os.environ, {"MICRO_ENGRAM_OFFLOAD": "1"}):
            m = EngramGemma4ForCausalLM(vllm_config=serving_config(conf_path))
        out["MICRO_ENGRAM_OFFLOAD=1"] = m.model.layers[LAYER].micro_engram.__dict__.get("row_views") is not None
        with mock.patch.dict(os.environ, {"MICRO_ENGRAM_OFF": "1"}):
            m = EngramGemma4ForCausalLM(vllm_config=serving_config(conf_path))
        layer = m.model.layers[LAYER]
        out["MICRO_ENGRAM_OFF=1 bypasses the engram"] = torch.equal(layer(None, h, None)[0],
                                                                    torch.tanh(layer.lin(h)))
        plain = EngramGemma4ForCausalLM(vllm_config=serving_config())
        out["no config: plain Gemma 4"] = plain.micro_engram_ids is None and not plain.micro_engram_slots
    sys.modules.pop("micro_engram_vllm.model", None)
    return out


def _assert_all(results):
    for rank, checks in results.items():
        failed = [name for name, ok in checks.items() if not ok]
        assert not failed, f"rank {rank}: {failed}"


@pytest.mark.parametrize("world", [3, 1])
def test_tp_lookup_and_loading(world):
    _assert_all(run_dist(_lookup_checks, world))


@pytest.mark.parametrize("world", [3, 1])
def test_plugin_model_with_fake_vllm(world, tmp_path):
    _assert_all(run_dist(_model_checks, world, str(tmp_path)))


def test_model_state_attach_fills_history():
    """The model-state wrapper that register() installs fills the history buffer before each step."""
    from micro_engram_vllm.model_state import attach

    class Runner:
        max_num_tokens = 8

        def prepare_inputs(self, batch, req):
            return {"x": 1}

    model = types.SimpleNamespace(micro_engram_ids=torch.full((8, 3), 5, dtype=torch.int32))
    state = attach(Runner(), model)
    batch = types.SimpleNamespace(input_ids=torch.tensor([7, 8, 9, 0], dtype=torch.int32),
                                  positions=torch.tensor([0, 1, 2, 0]), idx_mapping=torch.tensor([0], dtype=torch.int32),
                                  query_start_loc=torch.tensor([0, 3], dtype=torch.int32), num_reqs=1, num_tokens=3,
                                  num_tokens_after_padding=4)
    req = types.SimpleNamespace(all_token_ids=types.SimpleNamespace(gpu=torch.zeros(1, 16, dtype=torch.int32)))
    assert state.prepare_inputs(batch, req) == {"x": 1}
    want = torch.tensor([[7, -1, -1], [8, 7, -1], [9, 8, 7], [-1, -1, -1]], dtype=torch.int32)
    assert torch.equal(model.micro_engram_ids[:4], want) and bool((model.micro_engram_ids[4:] == 5).all())
    assert attach(state, model) is state
    bare = Runner()
    assert attach(bare, types.SimpleNamespace()) is bare
