"""The head_dim-512 attention backward that writes P / dS tiles to HBM (csrc/attention_tc.cu:
attn_tiles_kernel, attn_bwd_sdp_kernel, attn_bwd_acc_kernel) against the fp32 PyTorch oracle:
packed documents (one-token ones included), sliding windows, GQA groups of 1, 2 and 8, lengths
that are not multiples of the 128-row tiles, and a tile budget small enough to force one GQA
group per pass. head_dim 256 runs through the same kernels as a second check."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("D,Hq,Hk,window,lens,budget", [
    (512, 8, 1, None, [300, 5, 211], 1 << 40),
    (512, 4, 2, 100, [37, 120, 1, 80, 77, 260], 1),
    (512, 16, 2, None, [129, 1, 1, 383, 700], 1 << 40),
    (512, 8, 8, 300, [1000, 77], 1 << 40),
    (256, 4, 2, 100, [37, 120, 1, 80, 77], 1),
    (256, 32, 16, 1024, [1500, 700], 1 << 40),
])
def test_attention_bwd_mat(D, Hq, Hk, window, lens, budget):
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
    native().attn_tc_status(0).zero_()
    dq, dk, dv = native().attn_bwd_mat(do, q, k, v, o, lse, ds, int(window or 0), scale, budget)
    torch.cuda.synchronize()
    assert native().attn_tc_status(0).tolist() == [0, 0], "a wait timed out or a tile index was out of range"
    mq, mk, mv = native().attn_bwd(do, q, k, v, o, lse, ds, int(window or 0), scale)
    for name, got, old, want in (("dq", dq, mq, q32.grad), ("dk", dk, mk, k32.grad), ("dv", dv, mv, v32.grad)):
        err = (got.float() - want).abs().max().item()
        base = (old.float() - want).abs().max().item()
        assert err <= 2e-2 * want.abs().max().item() + 2e-3, f"{name}: {err} (mma.sync path: {base})"
