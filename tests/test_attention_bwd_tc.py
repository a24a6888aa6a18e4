"""The tcgen05/TMEM attention backward (dQ, dK, dV kernels) against the fp32 PyTorch oracle,
on packed documents (including one-token documents), sliding windows, causal global rows, GQA
groups of 1, 2 and 8, and lengths that are not multiples of the 128-row tiles."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("D,Hq,Hk,window,lens", [
    (64, 4, 2, 48, [37, 120, 1, 80, 77]),
    (128, 4, 1, None, [300, 5, 211]),
    (256, 4, 2, 100, [37, 120, 1, 80, 77]),
    (256, 8, 1, None, [129, 1, 1, 383]),
    (256, 32, 16, 1024, [1500, 700]),
])
def test_attention_bwd_tc(D, Hq, Hk, window, lens):
    from micro_engram_fork_b200 import native
    from micro_engram_fork_b200.ops.attention import attention_fwd, attention_ref, doc_starts

    torch.manual_seed(0)
    dev = torch.device("cuda", 0)
    T = sum(lens)
    pos = torch.cat([torch.arange(n) for n in lens]).to(dev)
    ds = doc_starts(pos)
    q = torch.randn(T, Hq, D, device=dev).to(torch.bfloat16)
    k = torch.randn(T, Hk, D, device=dev).to(torch.bfloat16)
    v = torch.randn(T, Hk, D, device=dev).to(torch.bfloat16)
    scale = 1.0 / math.sqrt(D)
    o, lse = attention_fwd(q, k, v, ds, window, scale)
    q32, k32, v32 = (t.float().requires_grad_() for t in (q, k, v))
    o32, _ = attention_ref(q32, k32, v32, ds, window, scale)
    do = torch.randn_like(o)
    o32.backward(do.float())
    dq, dk, dv = native().attn_bwd_tc(do, q, k, v, o, lse, ds, int(window or 0), scale)
    torch.cuda.synchronize()
    assert int(native().attn_tc_status(0)[0]) == 0, "a tcgen05 wait timed out"
    mq, mk, mv = native().attn_bwd(do, q, k, v, o, lse, ds, int(window or 0), scale)
    for name, got, old, want in (("dq", dq, mq, q32.grad), ("dk", dk, mk, k32.grad), ("dv", dv, mv, v32.grad)):
        err = (got.float() - want).abs().max().item()
        base = (old.float() - want).abs().max().item()
        assert err <= 2e-2 * want.abs().max().item() + 2e-3, f"{name}: {err} (mma.sync path: {base})"
