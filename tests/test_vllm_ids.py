"""Serving-side token histories (micro_engram_vllm.ids): simulated vLLM steps (chunked
prefill, prefix-cache hits, decode, mixed batches, request slots in any row, CUDA-graph
padding) must give every token the same n-gram history, and so the same engram output, as
the training forward over the whole sequence. Reference counterpart: test_vllm_ids.py."""
import random

import pytest
import torch

from micro_engram.module import MicroEngram
from micro_engram_vllm.ids import fill_engram_ids, mask_media

V, D, MAX_REQS, MAX_LEN = 1000, 16, 8, 64
SENTINEL_HIST, SENTINEL_OUT = 999, 777


def _engram(gate="scalar", **kw):
    torch.manual_seed(0)
    eng = MicroEngram(model_dim=D, table_size=257, engram_dim=4, num_heads=2, vocab_size=V, pad_id=0, gate=gate, **kw)
    with torch.no_grad():
        (eng.up if gate == "ple" else eng.value).weight.normal_()
    canon = torch.arange(V)
    canon[11], canon[501] = 10, 500
    eng.canon.copy_(canon)
    return eng


def _step(chunks, hist, slots, width=3, device="cpu", dtype_ids=torch.int32, dtype_pos=torch.int64):
    """chunks: (request, first position, count). The history table holds the real tokens
    before each chunk and garbage from the chunk on, so reading the chunk from history shows."""
    ids, pos, qsl = [], [], [0]
    for r, start, n in chunks:
        ids += hist[r][start:start + n]
        pos += list(range(start, start + n))
        qsl.append(qsl[-1] + n)
    n_tok = len(ids)
    padded = n_tok + 3
    table = torch.full((MAX_REQS, MAX_LEN), SENTINEL_HIST, dtype=torch.int32)
    for r, start, _ in chunks:
        table[slots[r], :start] = torch.tensor(hist[r][:start], dtype=torch.int32)
    out = torch.full((n_tok + 10, width), SENTINEL_OUT, dtype=torch.int32, device=device)
    fill_engram_ids(out, torch.tensor(ids + [5] * 3, dtype=dtype_ids, device=device),
                    torch.tensor(pos + [0] * 3, dtype=dtype_pos, device=device),
                    torch.tensor([slots[r] for r, _, _ in chunks], dtype=torch.int32, device=device),
                    torch.tensor(qsl, dtype=torch.int32, device=device), table.to(device),
                    num_reqs=len(chunks), num_tokens=n_tok, num_tokens_padded=padded)
    return out.cpu(), n_tok, padded


def _expected(chunks, hist, width=3):
    rows = []
    for r, start, n in chunks:
        h = hist[r]
        for p in range(start, start + n):
            rows.append([h[p - i] if p >= i else -1 for i in range(width)])
    return torch.tensor(rows, dtype=torch.int32)


HIST = None


def _hist():
    global HIST
    if HIST is None:
        rnd = random.Random(0)
        HIST = {r: [rnd.randrange(5, V) for _ in range(MAX_LEN)] for r in range(4)}
    return HIST


SLOTS = {0: 5, 1: 2, 2: 7, 3: 0}
CASES = {
    "full prefill": [(0, 0, 20)],
    "chunked prefill, second chunk": [(0, 20, 15)],
    "prefix-cache hit": [(1, 33, 4)],
    "decode": [(0, 40, 1), (1, 37, 1), (2, 2, 1)],
    "decode at positions 0 and 1": [(3, 0, 1), (2, 1, 1)],
    "mixed prefill and decode": [(0, 41, 1), (1, 0, 9), (2, 10, 2), (3, 50, 1)],
}


@pytest.mark.parametrize("packed", [False, True])
def test_hash_prev_matches_training_hash(packed):
    eng = _engram()
    ids = torch.randint(5, V, (1, 30))
    ids[0, 3], ids[0, 9] = 11, 501
    pos = torch.cat([torch.arange(12), torch.arange(13), torch.arange(5)])[None] if packed else None
    ref = eng.hash_ids(ids, pos)
    p = pos[0] if packed else torch.arange(30)
    rows = [[int(ids[0, t - i]) if p[t] >= i else -1 for i in range(3)] for t in range(30)]
    got = eng.hash_prev(torch.tensor(rows))
    assert all(torch.equal(a[0], b) for a, b in zip(ref, got))


@pytest.mark.parametrize("name", list(CASES))
def test_fill_cases(name):
    chunks = CASES[name]
    out, n, padded = _step(chunks, _hist(), SLOTS)
    assert torch.equal(out[:n], _expected(chunks, _hist()))
    assert bool((out[n:padded] == -1).all()) and bool((out[padded:] == SENTINEL_OUT).all())


@pytest.mark.parametrize("gate", MicroEngram.GATES)
def test_served_equals_training(gate):
    eng = _engram(gate)
    seq = torch.tensor(_hist()[0][:30])
    seq[4], seq[17] = 11, 501
    hidden = torch.randn(30, D) * 30
    train = eng(hidden[None], seq[None])[0]
    served = []
    for chunk in [(0, 0, 13), (0, 13, 9)] + [(0, p, 1) for p in range(22, 30)]:
        out, n, _ = _step([chunk], {0: seq.tolist()}, {0: 3})
        _, start, cnt = chunk
        served.append(eng.inject(hidden[start:start + cnt], eng.hash_prev(out[:n])))
    torch.testing.assert_close(torch.cat(served), train, atol=1e-5, rtol=0)


def test_four_grams_mixed_sizes():
    eng = _engram("scalar_sqrt", orders=(2, 3, 4), table_sizes={2: 257, 3: 401, 4: 97})
    seq = torch.tensor(_hist()[1][:30])
    hidden = torch.randn(30, D) * 30
    train = eng(hidden[None], seq[None])[0]
    served = []
    for chunk in [(0, 0, 11), (0, 11, 9)] + [(0, p, 1) for p in range(20, 30)]:
        out, n, _ = _step([chunk], {0: seq.tolist()}, {0: 1}, width=4)
        _, start, cnt = chunk
        served.append(eng.inject(hidden[start:start + cnt], eng.hash_prev(out[:n])))
    torch.testing.assert_close(torch.cat(served), train, atol=1e-5, rtol=0)


def test_media_masking():
    img = 900
    eng = _engram("scalar_sqrt")
    text1, text2 = _hist()[0][:6], _hist()[0][6:14]
    seq = text1 + [img] * 4 + text2
    hidden = torch.randn(len(seq), D) * 30
    out, n, _ = _step([(0, 0, len(seq))], {0: seq}, {0: 3})
    ids, keep = mask_media(out[:n], torch.tensor([img, 901]))
    served = eng.inject(hidden, eng.hash_prev(ids), keep)
    media = slice(len(text1), len(text1) + 4)
    assert torch.equal(served[media], hidden[media]) and not keep[media].any() and keep[:len(text1)].all()
    torch.testing.assert_close(served[:len(text1)], eng(hidden[:len(text1)][None], torch.tensor([text1]))[0],
                               atol=1e-5, rtol=0)
    after = slice(len(text1) + 4, len(seq))  # text right after the image starts a fresh history
    torch.testing.assert_close(served[after], eng(hidden[after][None], torch.tensor([text2]))[0], atol=1e-5, rtol=0)
    plain, plain_keep = mask_media(out[:n], torch.tensor([7777]))
    assert torch.equal(plain, out[:n]) and bool(plain_keep.all())


# ------------------------------------------------------------------ GPU: the sm_100a kernels
@pytest.mark.gpu
@pytest.mark.parametrize("dtypes", [(torch.int32, torch.int64), (torch.int64, torch.int32)])
def test_fill_kernel_matches_cpu(dtypes):
    dev = torch.device("cuda", 0)
    for name, chunks in CASES.items():
        for width in (3, 4):
            cpu, n, padded = _step(chunks, _hist(), SLOTS, width=width, dtype_ids=dtypes[0], dtype_pos=dtypes[1])
            gpu, _, _ = _step(chunks, _hist(), SLOTS, width=width, device=dev, dtype_ids=dtypes[0],
                              dtype_pos=dtypes[1])
            assert torch.equal(cpu, gpu), name


@pytest.mark.gpu
@pytest.mark.parametrize("gate", ["scalar", "scalar_sqrt"])
def test_serve_inject_op_matches_module(gate):
    """The fused serving op (hash -> row-store gather -> projections -> gate) == the module's
    fp32 inject on the same rows, within the bf16 noise floor."""
    from helpers import noise_floor_check
    from micro_engram_vllm.tp import fused_ok, serve_inject

    dev = torch.device("cuda", 0)
    torch.manual_seed(1)
    d = 256
    full = MicroEngram(model_dim=d, table_size=4099, engram_dim=32, num_heads=2, vocab_size=V, gate=gate,
                       orders=(2, 3, 4))
    with torch.no_grad():
        full.value.weight.normal_(std=0.05)
        if gate == "scalar_sqrt":
            full.q_scale.normal_(std=0.1)
            full.k_scale.normal_(std=0.1)
    ref32 = full.to(dev)
    hist = torch.randint(5, V, (300, 4), device=dev, dtype=torch.int32)
    hist[:3, 1:] = -1
    hidden = (torch.randn(300, d, device=dev) * 3).to(torch.bfloat16)
    want = ref32.inject(hidden.float(), ref32.hash_prev(hist))
    bf = MicroEngram(model_dim=d, table_size=4099, engram_dim=32, num_heads=2, vocab_size=V, gate=gate,
                     orders=(2, 3, 4))
    bf.load_state_dict(full.state_dict())
    bf = bf.to(dev).to(torch.bfloat16)
    plain = bf.inject(hidden, bf.hash_prev(hist))  # bf16 torch path (tables still local)
    bf.shard_rows(0, 1, device=dev, dtype=torch.bfloat16, requires_grad=False)
    assert fused_ok(bf, hidden)
    with torch.inference_mode():
        got = serve_inject(bf, hidden, hist)
    bf.row_store.check_status()
    noise_floor_check(got, want, plain, name=f"serve_inject {gate}")
