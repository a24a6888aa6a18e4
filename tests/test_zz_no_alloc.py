"""The allocation-free attention backward, called through its exported C symbol.

`me_attn_bwd_noalloc` serves callers that may not allocate device memory while they run
(graph memory pools, fixed-budget servers, C programs without PyTorch's allocator): its
scratch is a fixed device array inside the library. This test loads the built extension
with ctypes, calls the C entry point twice in a row on fresh inputs (the larger problem first,
so the second, smaller call runs on scratch full of the first call's values), compares
dQ/dK/dV with the PyTorch-facing `attn_bwd` using the same tolerance as the attention test, and
checks that neither call changed the memory PyTorch has allocated or the device's free memory.
It also checks that an oversized problem and a misaligned pointer are refused with a clear
error. This file is collected last on purpose.
"""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    import micro_engram_fork_b200 as me

    lib = ctypes.CDLL(me.native().__file__)
    fn = lib.me_attn_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 7 + [ctypes.c_int] * 5 + [ctypes.c_float] + [ctypes.c_void_p] * 4
    lib.me_noalloc_last_error.restype = ctypes.c_char_p
    return lib, fn


def _call(fn, dout, q, k, v, o, lse, ds, window, scale, dq, dk, dv):
    T, Hq, D = q.shape
    Hk = k.shape[1]
    stream = torch.cuda.current_stream().cuda_stream
    return fn(dout.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(),
              ds.data_ptr(), T, Hq, Hk, D, window or 0, scale, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), stream)


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_no_alloc_attention_backward_matches_attn_bwd():
    from micro_engram_fork_b200.ops.attention import attention_bwd, attention_fwd, doc_starts

    lib, fn = _lib()
    dev = torch.device("cuda", 0)
    # two rounds of the same two problems: the first round also loads each kernel's code on its
    # first launch (lazy module loading can take device memory then); the second round must
    # leave every memory figure exactly as it found it
    for rnd in range(2):
        for call, (D, Hq, Hk, window) in enumerate([(512, 8, 2, None), (256, 4, 2, 100)]):
            torch.manual_seed(10 + call + 2 * rnd)
            lens = [57, 130, 1, 90]
            T = sum(lens)
            pos = torch.cat([torch.arange(n) for n in lens]).to(dev)
            ds = doc_starts(pos).contiguous()
            q = torch.randn(T, Hq, D, device=dev).to(torch.bfloat16)
            k = torch.randn(T, Hk, D, device=dev).to(torch.bfloat16)
            v = torch.randn(T, Hk, D, device=dev).to(torch.bfloat16)
            scale = 1.0 / math.sqrt(D)
            o, lse = attention_fwd(q, k, v, ds, window, scale)
            dout = torch.randn_like(o)
            want = attention_bwd(dout, q, k, v, o, lse, ds, window, scale)
            got = [torch.full_like(q, float("nan")), torch.full_like(k, float("nan")), torch.full_like(v, float("nan"))]
            torch.cuda.synchronize()
            torch_bytes, (free_bytes, _) = torch.cuda.memory_allocated(dev), torch.cuda.mem_get_info(dev)
            rc = _call(fn, dout, q, k, v, o, lse, ds, window, scale, *got)
            assert rc == 0, lib.me_noalloc_last_error().decode()
            torch.cuda.synchronize()
            if rnd == 1:
                assert torch.cuda.memory_allocated(dev) == torch_bytes, "the call allocated through PyTorch"
                assert torch.cuda.mem_get_info(dev)[0] == free_bytes, "the call changed the device's free memory"
            for name, g, w in zip(("dq", "dk", "dv"), got, want):
                err = (g.float() - w.float()).abs().max().item()
                assert err <= 2e-2 * w.float().abs().max().item() + 2e-3, f"round {rnd} call {call} {name}: {err}"


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_no_alloc_rejects_oversized_problem():
    lib, fn = _lib()
    dev = torch.device("cuda", 0)
    T, Hq, Hk, D = 70_000, 32, 4, 64  # Hq*T*4 bytes > the 8 MiB scratch
    tiny = torch.zeros(8, device=dev, dtype=torch.bfloat16)
    lse = torch.zeros(8, device=dev)
    ds = torch.zeros(8, device=dev, dtype=torch.int32)
    stream = torch.cuda.current_stream().cuda_stream
    p = tiny.data_ptr()
    rc = fn(p, p, p, p, p, lse.data_ptr(), ds.data_ptr(), T, Hq, Hk, D, 0, 1.0, p, p, p, stream)
    assert rc == -2
    assert b"exceed" in lib.me_noalloc_last_error()


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_no_alloc_rejects_misaligned_pointers():
    lib, fn = _lib()
    dev = torch.device("cuda", 0)
    T, Hq, Hk, D = 16, 2, 1, 64
    buf = torch.zeros(T * Hq * D + 8, device=dev, dtype=torch.bfloat16)
    lse = torch.zeros(Hq * T, device=dev)
    ds = torch.zeros(T, device=dev, dtype=torch.int32)
    stream = torch.cuda.current_stream().cuda_stream
    p = buf.data_ptr()
    rc = fn(p + 2, p, p, p, p, lse.data_ptr(), ds.data_ptr(), T, Hq, Hk, D, 0, 1.0, p, p, p, stream)  # dout off by 2 B
    assert rc == -1 and b"16-byte" in lib.me_noalloc_last_error()
    rc = fn(p, p, p, p, p, lse.data_ptr() + 2, ds.data_ptr(), T, Hq, Hk, D, 0, 1.0, p, p, p, stream)
    assert rc == -1 and b"4-byte" in lib.me_noalloc_last_error()
