"""The native engram runtime (engram_runtime/, C++ + sm_100a) against the PyTorch engram:
a tiny Gemma 4 GGUF gets engrams through micro_engram.gguf_export, the runtime reads them
back, and its hash, histories and injection must match MicroEngram. The driver
(engram_logits) runs the four serving modes (whole sequence, ubatches of 7, one token at a
time, two interleaved sequences, history saved / cleared / restored). Variants: the three
gates, bf16 and f32 storage, 4-grams with per-order sizes, token merging; a negative control
(the merge map left out) must fail. Reference counterpart: llama_cpp/test/compare.py."""
import copy
import json
import os
import subprocess

import numpy as np
import pytest
import torch

from micro_engram import engram_runtime as ert
from micro_engram.module import MicroEngram

V, D, N_LAYER, LAYER = 512, 64, 6, 2


@pytest.fixture(scope="module", autouse=True)
def built():
    ert.build()


def _base_gguf(path):
    import gguf

    w = gguf.GGUFWriter(path, arch="gemma4")
    w.add_uint32("gemma4.embedding_length", D)
    w.add_uint32("gemma4.block_count", N_LAYER)
    w.add_token_list([f"t{i}" for i in range(V)])
    w.add_tensor("token_embd.weight", np.random.default_rng(0).standard_normal((V, D)).astype(np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def _engram(gate, orders=(2, 3), sizes=None, canon=None, seed=0):
    torch.manual_seed(seed)
    e = MicroEngram(model_dim=D, table_size=97, engram_dim=8, num_heads=2, vocab_size=V, gate=gate, orders=orders,
                    table_sizes=sizes, canon=canon, seed=LAYER * 10007)
    with torch.no_grad():
        for t in e.tables:
            t.weight.normal_()
        (e.up if gate == "ple" else e.value).weight.normal_(std=0.3)
        if gate == "scalar_sqrt":
            e.q_scale.normal_(std=0.2)
            e.k_scale.normal_(std=0.2)
    return e


def _write(tmp, e, dtype="bf16", name="m", canon_in_file=True):
    folder = os.path.join(tmp, name)
    os.makedirs(folder, exist_ok=True)
    sd = {k: v for k, v in e.state_dict().items() if canon_in_file or k != "canon"}
    torch.save({f"model.layers.{LAYER}.micro_engram.{k}": v for k, v in sd.items()}, os.path.join(folder, "w.pt"))
    conf = {"layer": LAYER, "table_size": e.table_size, "table_sizes": {str(k): v for k, v in e.order_sizes.items()},
            "engram_dim": 8, "num_heads": 2, "orders": list(e.orders), "gate": e.gate, "seed": LAYER * 10007,
            "pad_id": 0, "vocab_size": V, "weights": "w.pt"}
    with open(os.path.join(folder, "micro_engram_config.json"), "w") as f:
        json.dump(conf, f)
    base = os.path.join(tmp, "base.gguf")
    if not os.path.exists(base):
        _base_gguf(base)
    from micro_engram.gguf_export import add_engrams

    out = os.path.join(folder, "model.gguf")
    add_engrams(base, folder, out, dtype=dtype, force=True)
    return out


def _as_stored(e, dtype):
    """The engram with its weights rounded the way the GGUF stores them (the oracle)."""
    q = copy.deepcopy(e).float()
    if dtype != "f32":
        cast = torch.bfloat16 if dtype == "bf16" else torch.float16
        with torch.no_grad():
            for name, p in q.named_parameters():
                if "scale" not in name:
                    p.copy_(p.to(cast).float())
    return q


def _hist(ids, max_order):
    """[n, max_order] rows (t, t-1, ...) of one sequence, -1 before its start."""
    n = len(ids)
    return torch.tensor([[int(ids[t - i]) if t >= i else -1 for i in range(max_order)] for t in range(n)])


def _driver(gguf_path, tokens, hidden, mode, tmp, ubatch=0, gpu=False):
    S, T = tokens.shape
    tp, hp, op = (os.path.join(tmp, n) for n in ("tok.i32", "h.f32", "o.f32"))
    tokens.astype(np.int32).tofile(tp)
    hidden.astype(np.float32).tofile(hp)
    cmd = [ert.DRIVER_PATH, "--gguf", gguf_path, "--n-seq", str(S), "--n-tok", str(T), "--tokens", tp, "--hidden", hp,
           "--mode", mode, "--out", op] + (["--ubatch", str(ubatch)] if ubatch else []) + (["--gpu"] if gpu else [])
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    return np.fromfile(op, dtype=np.float32).reshape(S, T, D)


VARIANTS = [("scalar", (2, 3), None, "bf16"), ("scalar_sqrt", (2, 3), None, "bf16"), ("ple", (2, 3), None, "bf16"),
            ("scalar_sqrt", (2, 3), None, "f32"), ("scalar_sqrt", (2, 3, 4), {2: 97, 3: 131, 4: 29}, "bf16")]


@pytest.mark.parametrize("gate,orders,sizes,dtype", VARIANTS)
def test_runtime_matches_module(tmp_path, gate, orders, sizes, dtype):
    canon = torch.arange(V) & ~1  # merge every even/odd pair
    e = _engram(gate, orders, sizes, canon)
    path = _write(str(tmp_path), e, dtype)
    rt = ert.Runtime(path)
    info = rt.info(0)
    assert rt.n_engrams == 1 and info["layer"] == LAYER and info["n_tables"] == len(e.table_rows)
    assert info["total_rows"] == sum(e.table_rows) and rt.max_order == max(orders) and rt.n_embd == D
    # hash: bit-exact with the module's serving hash (+ each table's offset)
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, V, (40,), generator=g)
    hist = _hist(ids, rt.max_order)
    hist[5, 1:] = -1  # a history cut short (start of a document)
    want = torch.stack(e.hash_prev(hist), 1) + torch.tensor(np.cumsum([0] + e.table_rows[:-1]))
    rows = rt.hash(0, hist[:, 0].numpy(), hist[:, 1:].flip(1).numpy())
    assert np.array_equal(rows, want.numpy())
    # CPU injection == the fp32 module with the stored weights
    oracle = _as_stored(e, dtype)
    h = torch.randn(40, D, generator=g) * 3
    ref = oracle.inject(h, oracle.hash_prev(hist)).detach().numpy()
    got = rt.inject_cpu(0, h.numpy(), rows)
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-4 * np.abs(ref).max())
    os.environ["ME_RT_THREADS"] = "1"  # the positions split over threads above, on one thread here
    try:
        assert np.array_equal(rt.inject_cpu(0, h.numpy(), rows), got)
    finally:
        del os.environ["ME_RT_THREADS"]
    keep = np.ones(40, np.float32)
    keep[3] = 0
    got_k = rt.inject_cpu(0, h.numpy(), rows, keep)
    assert np.array_equal(got_k[3], h[3].numpy()) and np.allclose(got_k[4], got[4])
    # the driver's serving modes == the training forward over whole sequences
    tokens = torch.randint(0, V, (2, 23), generator=g)
    hidden = torch.randn(2, 23, D, generator=g) * 3
    full = np.stack([oracle(hidden[s][None], tokens[s][None])[0].detach().numpy() for s in range(2)])
    tol = dict(rtol=1e-4, atol=1e-4 * np.abs(full).max())
    for mode, ub in (("full", 0), ("full", 7), ("decode", 0), ("two", 0)):
        out = _driver(path, tokens.numpy(), hidden.numpy(), mode, str(tmp_path), ub)
        np.testing.assert_allclose(out, full, **tol, err_msg=f"mode {mode} ubatch {ub}")
    out = _driver(path, tokens.numpy(), hidden.numpy(), "state", str(tmp_path))
    np.testing.assert_allclose(out[0], full[0], **tol, err_msg="mode state")


def test_negative_control_without_merge_map(tmp_path):
    """An engram trained with token merging, exported without its map (identity): the runtime
    must disagree with the oracle, which shows the map is what makes them agree."""
    canon = torch.arange(V) & ~1
    e = _engram("scalar", canon=canon)
    plain = copy.deepcopy(e)
    plain.canon.copy_(torch.arange(V))
    path = _write(str(tmp_path), plain, "f32", name="nomap")
    g = torch.Generator().manual_seed(2)
    tokens = torch.randint(0, V, (1, 30), generator=g)
    hidden = torch.randn(1, 30, D, generator=g) * 3
    want = e(hidden, tokens)[0].detach().numpy()
    out = _driver(path, tokens.numpy(), hidden.numpy(), "full", str(tmp_path))[0]
    assert np.abs(out - want).max() > 1e-2 * np.abs(want).max()


def test_runtime_errors_and_history(tmp_path):
    base = os.path.join(str(tmp_path), "base.gguf")
    _base_gguf(base)
    with pytest.raises(RuntimeError, match="no micro_engram metadata"):
        ert.Runtime(base)
    with pytest.raises(RuntimeError, match="cannot open"):
        ert.Runtime(os.path.join(str(tmp_path), "missing.gguf"))
    e = _engram("scalar")
    path = _write(str(tmp_path), e)
    with pytest.raises(RuntimeError, match="out of range"):
        ert.Runtime(path, n_layer=LAYER)  # the engram's layer is past the model's layers
    h = ert.History()
    for p, t in enumerate([5, 6, 7, 8]):
        h.set(0, p, t)
    assert h.prev([0, 0], [3, 1], 2).tolist() == [[6, 7], [-1, 5]]
    h.copy(0, 3)
    h.remove(0, 2)  # rewind sequence 0 to two tokens
    assert h.prev([0, 3], [3, 3], 2).tolist() == [[6, -1], [6, 7]]  # oldest first; position 2 is gone
    blob = h.save(3)
    h.remove(-1)
    assert h.prev([3], [3], 2).tolist() == [[-1, -1]]
    h.load(9, blob)
    assert h.prev([9], [4], 3).tolist() == [[6, 7, 8]]
    with pytest.raises(RuntimeError, match="history"):
        h.load(1, b"garbage-garbage-garbage")


@pytest.mark.gpu
@pytest.mark.parametrize("gate", ["scalar", "scalar_sqrt", "ple"])
def test_runtime_cuda_matches_cpu(tmp_path, gate):
    e = _engram(gate, orders=(2, 3, 4), sizes={2: 97, 3: 131, 4: 29})
    path = _write(str(tmp_path), e)
    g = torch.Generator().manual_seed(3)
    tokens = torch.randint(0, V, (2, 37), generator=g).numpy()
    hidden = (torch.randn(2, 37, D, generator=g) * 3).numpy()
    for mode in ("full", "decode"):
        cpu = _driver(path, tokens, hidden, mode, str(tmp_path))
        gpu = _driver(path, tokens, hidden, mode, str(tmp_path), gpu=True)
        np.testing.assert_allclose(gpu, cpu, rtol=1e-3, atol=1e-3 * np.abs(cpu).max(), err_msg=mode)
