"""GPU numerics of the sm_100a kernels against plain fp32 PyTorch references.

Rule for bf16 kernels (after the reference's test_kernels_gpu.py:124-127): the kernel's
error against the fp32 reference must be within 1.5x the error of the plain bf16 PyTorch
computation of the same op, plus a small eps. Integer kernels (hash) must match exactly.
"""
import math

import pytest
import torch
import torch.nn.functional as F

from helpers import noise_floor_check

pytestmark = pytest.mark.gpu

cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")


@pytest.fixture(autouse=True)
def _native_loaded():
    if torch.cuda.is_available():
        import micro_engram_fork_b200

        micro_engram_fork_b200.native()  # loud failure when the extension is missing
    yield


def _dev():
    return torch.device("cuda", 0)


# ----------------------------------------------------------------------------- engram
@cuda
def test_hash_exact():
    from micro_engram.module import MicroEngram

    torch.manual_seed(0)
    e = MicroEngram(64, table_size=1000, engram_dim=16, num_heads=3, orders=(2, 3), table_sizes={4: 777},
                    vocab_size=5000, seed=11, canon=torch.arange(5000) // 2 * 2)
    ids = torch.randint(0, 5000, (3, 300))
    pos = torch.cat([torch.arange(100), torch.arange(120), torch.arange(80)]).expand(3, 300).contiguous()
    ref = e.hash_ids(ids, pos)
    got = e.to(_dev()).hash_ids(ids.to(_dev()), pos.to(_dev()))
    for a, b in zip(ref, got):
        assert torch.equal(a, b.cpu())
    prev = torch.randint(-1, 5000, (400, 4))
    e_cpu = MicroEngram(64, table_size=1000, engram_dim=16, num_heads=3, orders=(2, 3), table_sizes={4: 777},
                        vocab_size=5000, seed=11, canon=torch.arange(5000) // 2 * 2)
    for a, b in zip(e_cpu.hash_prev(prev), e.hash_prev(prev.to(_dev()))):
        assert torch.equal(a, b.cpu())


@cuda
@pytest.mark.parametrize("dtype,capacity,hot", [(torch.bfloat16, None, False), (torch.float32, None, False),
                                                (torch.bfloat16, 517, False), (torch.float32, 517, True)])
def test_gather_and_row_grads(dtype, capacity, hot):
    """Row gradients land in the compact accumulator: with a capacity of exactly the lookups
    per table (the trainer's bound), and with every lookup on 7 hot rows so that many warps
    race for the same fresh row (slots lost to the race stay empty holes)."""
    from micro_engram_fork_b200.parallel.row_store import RowStore

    torch.manual_seed(0)
    rows = [1000, 1000, 3001]
    st = RowStore(rows, 64, dtype, 0, 1, _dev(), capacity=capacity)
    full = [torch.randn(r, 64) * 0.02 for r in rows]
    for k in range(3):
        st.shard(k).copy_(full[k].to(dtype))
    idx = torch.stack([torch.randint(0, 7 if hot else r, (517,)) for r in rows]).to(_dev())
    mem = st.gather(idx, torch.bfloat16)
    ref = torch.cat([full[k].to(dtype)[idx[k].cpu()] for k in range(3)], dim=1)
    assert torch.equal(mem.cpu(), ref.to(torch.bfloat16))
    g = torch.randn(517, 3 * 64, device=_dev()).to(torch.bfloat16)
    st.push_grads(g, idx, 0.5)
    torch.cuda.synchronize()
    st.check_status()
    for k in range(3):
        want = torch.zeros(rows[k], 64)
        want.index_add_(0, idx[k].cpu(), g[:, k * 64:(k + 1) * 64].float().cpu() * 0.5)
        r, gr = st.touched(k)
        assert r.numel() == torch.unique(idx[k]).numel()
        torch.testing.assert_close(gr.cpu(), want[r.cpu()], rtol=1e-5, atol=1e-6)
        assert torch.equal(torch.sort(r.cpu()).values, torch.unique(idx[k].cpu()))
        assert int((st.pos[k] > 0).sum()) == r.numel()
    st.zero_grads()
    assert all(int(st.pos[k].abs().sum()) == 0 and float(st.acc[k].abs().sum()) == 0.0 for k in range(3))


def _gate_ref(h, k, v, qs, ks, sqrt_gate, keep=None):
    d = h.shape[-1]
    hn = F.rms_norm(h.float(), (d,), weight=qs)
    kn = F.rms_norm(k.float(), (d,), weight=ks)
    s = (hn * kn).sum(-1, keepdim=True) / d ** 0.5
    if sqrt_gate:
        s = s.sign() * s.abs().clamp_min(1e-6).sqrt()
    a = torch.sigmoid(s)
    out = a * v.float()
    if keep is not None:
        out = out * keep[:, None].float()
    return h + out.to(h.dtype)


@cuda
@pytest.mark.parametrize("sqrt_gate", [False, True])
def test_gate_fwd_bwd(sqrt_gate):
    from micro_engram_fork_b200.ops.engram import gate

    torch.manual_seed(0)
    N, d = 333, 5376
    h = (torch.randn(N, d, device=_dev()) * 3).to(torch.bfloat16).requires_grad_()
    k = torch.randn(N, d, device=_dev()).to(torch.bfloat16).requires_grad_()
    v = (torch.randn(N, d, device=_dev()) * 0.1).to(torch.bfloat16).requires_grad_()
    qd = (torch.randn(d, device=_dev()) * 0.1).requires_grad_() if sqrt_gate else None
    kd = (torch.randn(d, device=_dev()) * 0.1).requires_grad_() if sqrt_gate else None
    keep = torch.rand(N, device=_dev()) > 0.1
    g = torch.randn(N, d, device=_dev()).to(torch.bfloat16)
    out = gate(h, k, v, qd, kd, keep, sqrt_gate, None)
    out.backward(g)
    # fp32 reference on the same bf16 inputs
    h32, k32, v32 = (t.detach().float().requires_grad_() for t in (h, k, v))
    q32 = (1 + qd.detach()).requires_grad_() if sqrt_gate else None
    kk32 = (1 + kd.detach()).requires_grad_() if sqrt_gate else None
    ref = _gate_ref(h32, k32, v32, q32, kk32, sqrt_gate, keep)
    ref.backward(g.float())
    hb, kb, vb = (t.detach().clone().requires_grad_() for t in (h, k, v))
    plain = _gate_ref(hb, kb, vb, (1 + qd.detach()) if sqrt_gate else None, (1 + kd.detach()) if sqrt_gate else None,
                      sqrt_gate, keep)
    plain.backward(g)
    noise_floor_check(out, ref, plain, name="gate out")
    noise_floor_check(h.grad, h32.grad, hb.grad, name="dh")
    noise_floor_check(k.grad, k32.grad, kb.grad, eps=1e-4, name="dk")
    noise_floor_check(v.grad, v32.grad, vb.grad, eps=1e-4, name="dv")
    if sqrt_gate:
        torch.testing.assert_close(qd.grad, q32.grad, rtol=2e-2, atol=2e-3 * q32.grad.abs().max().item())
        torch.testing.assert_close(kd.grad, kk32.grad, rtol=2e-2, atol=2e-3 * kk32.grad.abs().max().item())


@cuda
def test_adam_touched_matches_reference():
    from micro_engram.optim import LazyAdamW
    from micro_engram_fork_b200.ops.engram import adam_touched
    from micro_engram_fork_b200.parallel.row_store import RowStore

    torch.manual_seed(0)
    rows, dim = 2000, 64
    st = RowStore([rows], dim, torch.float32, 0, 1, _dev(), capacity=700)
    w0 = torch.randn(rows, dim) * 0.02
    st.shard(0).copy_(w0)
    idx = torch.randint(0, rows, (1, 700), device=_dev())
    g = torch.randn(700, dim, device=_dev())
    st.push_grads(g, idx, 1.0)
    m = torch.zeros(rows, dim, device=_dev())
    v = torch.zeros(rows, device=_dev())
    adam_touched(st.shard(0), m, v, st.acc[0], st.pos[0], st.list[0], st.count[0], None, 1e-2, 0.9, 0.999, 1e-8,
                 0.0, 1 - 0.9, 1 - 0.999, False, 1, 1, 0)
    # reference: sparse rowwise LazyAdamW on CPU
    p = torch.nn.Parameter(w0.clone())
    u, inv = torch.unique(idx[0].cpu(), return_inverse=True)
    acc = torch.zeros(u.numel(), dim)
    acc.index_add_(0, inv, g.cpu())
    p.sparse_grad = (u, acc)
    opt = LazyAdamW([{"params": [p], "lazy": True, "rowwise": True}], lr=1e-2)
    opt.step()
    torch.testing.assert_close(st.shard(0).cpu(), p.detach(), rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(v.cpu(), opt.state[p]["exp_avg_sq"], rtol=1e-4, atol=1e-9)
    assert float(st.acc[0].abs().sum()) == 0.0 and int(st.pos[0].abs().sum()) == 0


@cuda
@pytest.mark.parametrize("rowwise", [True, False])
def test_adam_touched_host_moments_match_device(rowwise):
    """The touched-row AdamW with its table-sized moments in pinned host memory (read and
    written in place through the device mapping) gives bit-identical weights and moments."""
    from micro_engram_fork_b200.ops.engram import adam_touched
    from micro_engram_fork_b200.parallel.row_store import RowStore

    torch.manual_seed(0)
    rows, dim = 3000, 64
    idx = torch.randint(0, rows, (1, 900), device=_dev())
    g = torch.randn(900, dim, device=_dev()).to(torch.bfloat16)
    w0 = (torch.randn(rows, dim) * 0.02).to(torch.bfloat16)
    m0 = (torch.randn(rows, dim) * 0.01).to(torch.bfloat16)
    v0 = torch.rand(rows) * 1e-4 if rowwise else (torch.rand(rows, dim) * 1e-4).to(torch.bfloat16)
    out = []
    for host in (False, True):
        st = RowStore([rows], dim, torch.bfloat16, 0, 1, _dev(), capacity=900)
        st.shard(0).copy_(w0)
        m, v = m0.clone(), v0.clone()
        m = m.pin_memory() if host else m.to(_dev())
        v = v.to(_dev()) if (rowwise or not host) else v.pin_memory()
        for step in (1, 2):
            st.push_grads(g, idx, 1.0)
            adam_touched(st.shard(0), m, v, st.acc[0], st.pos[0], st.list[0], st.count[0], None, 1e-2, 0.9, 0.999,
                         1e-8, 0.01, 1 - 0.9 ** step, 1 - 0.999 ** step, True, 5, step, 0)
            st.count[0].zero_()
        torch.cuda.synchronize()
        out.append((st.shard(0).cpu().clone(), m.cpu().clone(), v.cpu().clone()))
    for a, b in zip(out[0], out[1]):
        assert torch.equal(a, b)


@cuda
def test_stochastic_rounding_unbiased():
    from micro_engram_fork_b200.ops.engram import adam_dense

    torch.manual_seed(0)
    n = 1 << 20
    # a tiny update on bf16 weights at 1.0: plain rounding would lose it entirely
    p = torch.ones(n, device=_dev(), dtype=torch.bfloat16)
    m = torch.zeros_like(p)
    v = torch.zeros_like(p)
    g = torch.full((n,), 1.0, device=_dev())
    lr = 1e-3  # update -lr, below half a bf16 step at 1.0 (2^-8 = 3.9e-3)
    adam_dense(p, g, m, v, lr, 0.9, 0.999, 1e-8, 0.0, 1 - 0.9, 1 - 0.999, 1.0, True, 7, 1)
    mean = p.float().mean().item()
    assert abs(mean - (1 - lr)) < 2e-4, mean


# ----------------------------------------------------------------------------- norms
@cuda
def test_rmsnorm_and_post_norm_add():
    from micro_engram_fork_b200.ops import norm as N

    torch.manual_seed(0)
    T, d = 257, 5376
    x = (torch.randn(T, d, device=_dev()) * 2).to(torch.bfloat16)
    w = torch.rand(d, device=_dev()) + 0.5
    y, rs = N.rmsnorm(x, w, 1e-6)
    noise_floor_check(y, N.rmsnorm_ref(x.float(), w), N.rmsnorm_ref(x, w), name="rmsnorm")
    dy = torch.randn(T, d, device=_dev()).to(torch.bfloat16)
    x32 = x.float().requires_grad_()
    N.rmsnorm_ref(x32, w).backward(dy.float())
    xb = x.clone().requires_grad_()
    N.rmsnorm_ref(xb, w).backward(dy)
    noise_floor_check(N.rmsnorm_bwd(dy, x, w, rs), x32.grad, xb.grad, name="rmsnorm bwd")
    # post-norm + residual + layer scalar + next pre-norm, forward and backward
    r = (torch.randn(T, d, device=_dev()) * 4).to(torch.bfloat16)
    a = torch.randn(T, d, device=_dev()).to(torch.bfloat16)
    wp, wn = torch.rand(d, device=_dev()) + 0.5, torch.rand(d, device=_dev()) + 0.5
    ls = torch.tensor([0.75], device=_dev())
    xo, h, ra, rx = N.post_norm_add(r, a, wp, ls, wn, 1e-6)
    r32, a32 = r.float().requires_grad_(), a.float().requires_grad_()
    x_ref, h_ref = N.post_norm_add_ref(r32, a32, wp, ls, wn)
    rb, ab = r.clone().requires_grad_(), a.clone().requires_grad_()
    x_pl, h_pl = N.post_norm_add_ref(rb, ab, wp, ls, wn)
    noise_floor_check(xo, x_ref, x_pl, name="post_norm_add x")
    noise_floor_check(h, h_ref, h_pl, name="post_norm_add h")
    gx = torch.randn(T, d, device=_dev()).to(torch.bfloat16)
    gh = torch.randn(T, d, device=_dev()).to(torch.bfloat16)
    (x_ref * gx.float() + h_ref * gh.float()).sum().backward()
    (x_pl * gx + h_pl * gh).float().sum().backward()
    dr, da = N.post_norm_add_bwd(gx, gh, a, xo, wp, ls, wn, ra, rx)
    noise_floor_check(dr, r32.grad, rb.grad, rel=2.0, name="d residual")
    noise_floor_check(da, a32.grad, ab.grad, rel=2.0, name="d branch")


@cuda
@pytest.mark.parametrize("D,kv_shared", [(64, False), (256, False), (512, True), (128, True)])
def test_qkv_norm_rope(D, kv_shared):
    from micro_engram_fork_b200.models.gemma import GemmaConfig
    from micro_engram_fork_b200.ops import norm as N

    torch.manual_seed(0)
    T, Hq, Hk = 131, 4, 2
    cfg = GemmaConfig(num_hidden_layers=2, layer_types=["sliding_attention", "full_attention"])
    inv = cfg.inv_freq("full_attention" if kv_shared else "sliding_attention", D).to(_dev())
    width = (Hq + (1 if kv_shared else 2) * Hk) * D
    qkv = torch.randn(T, width, device=_dev()).to(torch.bfloat16)
    qw, kw = torch.rand(D, device=_dev()) + 0.5, torch.rand(D, device=_dev()) + 0.5
    pos = torch.cat([torch.arange(70), torch.arange(61)]).to(_dev())
    q, k, v, rs = N.qkv_norm_rope(qkv, qw, kw, inv, pos, Hq, Hk, D, kv_shared)

    def ref(x, dtype):
        x = x.to(dtype)
        qq = x[:, :Hq * D].view(T, Hq, D)
        kk = x[:, Hq * D:(Hq + Hk) * D].view(T, Hk, D)
        vv = kk if kv_shared else x[:, (Hq + Hk) * D:].view(T, Hk, D)
        cos, sin = N.rope_cos_sin(pos, inv, dtype)
        qo = N.rope_ref(N.rmsnorm_ref(qq, qw), cos[:, None], sin[:, None])
        ko = N.rope_ref(N.rmsnorm_ref(kk, kw), cos[:, None], sin[:, None])
        vo = N.rmsnorm_ref(vv, None)
        return qo, ko, vo

    x32 = qkv.float().requires_grad_()
    xb = qkv.clone().requires_grad_()
    r32, rb = ref(x32, torch.float32), ref(xb, torch.bfloat16)
    for name, a, b, c in zip("qkv", (q, k, v), r32, rb):
        noise_floor_check(a, b, c, rel=2.0, name=f"{name} fwd")
    gs = [torch.randn_like(t) for t in (q, k, v)]
    sum((a.float() * g.float()).sum() for a, g in zip(r32, gs)).backward()
    sum((a * g).float().sum() for a, g in zip(rb, gs)).backward()
    d = N.qkv_norm_rope_bwd(gs[0], gs[1], gs[2], qkv, qw, kw, inv, pos, rs, Hq, Hk, D, kv_shared)
    noise_floor_check(d, x32.grad, xb.grad, rel=2.0, name="qkv bwd")


@cuda
def test_geglu():
    from micro_engram_fork_b200.ops import norm as N

    torch.manual_seed(0)
    gu = (torch.randn(77, 2 * 1024, device=_dev()) * 2).to(torch.bfloat16)
    m = N.geglu(gu)
    g32 = gu.float().requires_grad_()
    gb = gu.clone().requires_grad_()
    r32, rb = N.geglu_ref(g32), N.geglu_ref(gb)
    noise_floor_check(m, r32, rb, name="geglu")
    dm = torch.randn_like(m)
    r32.backward(dm.float())
    rb.backward(dm)
    noise_floor_check(N.geglu_bwd(dm, gu), g32.grad, gb.grad, rel=2.0, name="geglu bwd")


# ----------------------------------------------------------------------------- loss
@cuda
@pytest.mark.parametrize("softcap,V", [(None, 5000), (30.0, 5000), (30.0, 4999)])
def test_fused_ce(softcap, V, dist_env):
    """The tcgen05 head GEMM with the softcapped-LSE epilogue, the in-place gradient and the
    fp32-output dH GEMM against the full-logit loss in fp64 (V = 4999: the padded shard)."""
    import torch.distributed as dist

    from micro_engram.train.head import VocabShard, reference_loss_sum

    dist.init_process_group("gloo", rank=0, world_size=1)
    torch.manual_seed(0)
    d, N = 256, 700
    W = (torch.randn(V, d) * 0.05).to(torch.bfloat16)
    shard = VocabShard(W, 0, 1, embed_scale=d ** 0.5, softcap=softcap, chunk_tokens=256, device=_dev())
    h = torch.randn(N, d, device=_dev()).to(torch.bfloat16).requires_grad_()
    labels = torch.randint(0, V, (N,), device=_dev())
    labels[::7] = -100
    total, count = shard.loss_sum(h, labels)
    (total * 0.37).backward()  # the gradient is formed in the forward and scaled in the backward
    with torch.no_grad():
        again, _ = shard.loss_sum(h, labels)
    assert torch.equal(again, total.detach())
    h32 = h.detach().float().requires_grad_()
    ref = reference_loss_sum(h32, labels, W.float().to(_dev()), softcap)
    (ref * 0.37).backward()
    ref64 = reference_loss_sum(h.detach().double(), labels, W.double().to(_dev()), softcap)
    assert abs(total.item() - ref64.item()) <= 2e-3 * abs(ref64.item()) + 1e-2
    assert abs(total.item() - ref.item()) <= 2e-3 * abs(ref.item()) + 1e-2
    assert int(count) == int((labels != -100).sum())
    err = (h.grad.float() - h32.grad).abs().max().item()
    assert err <= 3e-2 * h32.grad.abs().max().item() + 1e-4, err
    emb = shard.embed(labels.clamp_min(0))
    want = (W.to(_dev())[labels.clamp_min(0)] * torch.tensor(d ** 0.5, dtype=torch.bfloat16)).to(torch.bfloat16)
    assert torch.equal(emb, want)


# ----------------------------------------------------------------------------- attention
@cuda
@pytest.mark.parametrize("D,Hq,Hk,window", [(64, 4, 2, 48), (128, 4, 1, None), (256, 4, 2, 100), (512, 8, 2, None)])
def test_attention(D, Hq, Hk, window):
    from micro_engram_fork_b200.ops.attention import attention_bwd, attention_fwd, attention_ref, doc_starts

    torch.manual_seed(0)
    lens = [37, 120, 1, 80, 77]
    T = sum(lens)
    pos = torch.cat([torch.arange(n) for n in lens]).to(_dev())
    ds = doc_starts(pos)
    q = torch.randn(T, Hq, D, device=_dev()).to(torch.bfloat16)
    k = torch.randn(T, Hk, D, device=_dev()).to(torch.bfloat16)
    v = torch.randn(T, Hk, D, device=_dev()).to(torch.bfloat16)
    scale = 1.0 / math.sqrt(D)
    o, lse = attention_fwd(q, k, v, ds, window, scale)
    q32, k32, v32 = (t.float().requires_grad_() for t in (q, k, v))
    o32, lse32 = attention_ref(q32, k32, v32, ds, window, scale)
    qb, kb, vb = (t.clone().requires_grad_() for t in (q, k, v))
    ob, _ = attention_ref(qb, kb, vb, ds, window, scale)
    noise_floor_check(o, o32, ob.to(torch.bfloat16), rel=2.0, eps=2e-3, name="attn out")
    torch.testing.assert_close(lse, lse32.detach(), rtol=1e-3, atol=1e-3)
    do = torch.randn_like(o)
    o32.backward(do.float())
    dq, dk, dv = attention_bwd(do, q, k, v, o, lse, ds, window, scale)
    for name, got, want in (("dq", dq, q32.grad), ("dk", dk, k32.grad), ("dv", dv, v32.grad)):
        err = (got.float() - want).abs().max().item()
        assert err <= 2e-2 * want.abs().max().item() + 2e-3, f"{name}: {err}"


# ----------------------------------------------------------------------------- decoder layer
@cuda
@pytest.mark.parametrize("checkpoint", [False, "full", "selective", "none"])
def test_decoder_native_vs_torch(checkpoint):
    from micro_engram_fork_b200.models import gemma as G
    from micro_engram_fork_b200.ops.attention import doc_starts

    torch.manual_seed(0)
    cfg = G.tiny_config(hidden_size=512, intermediate_size=1024)
    model = G.GemmaForCausalLM(cfg).to(_dev())
    G.init_random_(model, seed=3)
    G.cast_projections_(model, torch.bfloat16)
    text = model.model
    if checkpoint:
        text.gradient_checkpointing_enable(policy=checkpoint)
    T = 300
    pos = torch.cat([torch.arange(100), torch.arange(200)]).to(_dev())
    x = (torch.randn(T, cfg.hidden_size, device=_dev())).to(torch.bfloat16).requires_grad_()
    y = text(x, pos)
    g = torch.randn_like(y)
    y.backward(g)
    import os

    def torch_path(model_dtype):
        m = G.GemmaForCausalLM(cfg).to(_dev())
        m.load_state_dict(model.state_dict())
        G.cast_projections_(m, model_dtype)
        xr = x.detach().to(model_dtype).clone().requires_grad_()
        os.environ["MICRO_ENGRAM_REFERENCE_OPS"] = "1"
        try:
            yr = m.model(xr, pos)
            yr.backward(g.to(model_dtype))
        finally:
            os.environ.pop("MICRO_ENGRAM_REFERENCE_OPS")
        return yr, xr.grad

    y32, gx32 = torch_path(torch.float32)   # fp32 oracle on the same (bf16-valued) weights
    yb, gxb = torch_path(torch.bfloat16)    # plain PyTorch in bf16: the noise floor

    def rel(a, b):
        return float((a.float() - b.float()).norm() / b.float().norm())

    assert rel(y, y32) <= 1.5 * rel(yb, y32) + 2e-3, (rel(y, y32), rel(yb, y32))
    assert rel(x.grad, gx32) <= 1.5 * rel(gxb, gx32) + 2e-3, (rel(x.grad, gx32), rel(gxb, gx32))


# ----------------------------------------------------------------------------- tcgen05 attention forward
@cuda
@pytest.mark.parametrize("D,Hq,Hk,window,lens", [
    (64, 4, 2, 48, [37, 120, 1, 80, 77]),
    (128, 4, 1, None, [300, 2, 211]),
    (256, 4, 2, 100, [37, 260, 1, 80, 140]),
    (512, 8, 2, None, [700, 33, 290]),
])
def test_attention_fwd_tcgen05(D, Hq, Hk, window, lens):
    import micro_engram_fork_b200 as me
    from micro_engram_fork_b200.ops.attention import attention_ref, doc_starts

    torch.manual_seed(0)
    T = sum(lens)
    pos = torch.cat([torch.arange(n) for n in lens]).to(_dev())
    ds = doc_starts(pos)
    q = torch.randn(T, Hq, D, device=_dev()).to(torch.bfloat16)
    k = torch.randn(T, Hk, D, device=_dev()).to(torch.bfloat16)
    v = torch.randn(T, Hk, D, device=_dev()).to(torch.bfloat16)
    scale = 1.0 / math.sqrt(D)
    o, lse = me.native().attn_fwd_tc(q, k, v, ds, window or 0, scale)
    torch.cuda.synchronize()
    assert int(me.native().attn_tc_status(0)[0]) == 0, "tcgen05 attention reported a timeout"
    o32, lse32 = attention_ref(q.float(), k.float(), v.float(), ds, window, scale)
    ob, _ = attention_ref(q, k, v, ds, window, scale)
    noise_floor_check(o, o32, ob.to(torch.bfloat16), rel=2.0, eps=2e-3, name="attn tc out")
    torch.testing.assert_close(lse, lse32, rtol=1e-3, atol=1e-3)


@cuda
@pytest.mark.parametrize("D,Hq,Hk,window", [(128, 4, 2, None), (256, 4, 2, 300), (512, 4, 1, None)])
def test_attention_fwd_tcgen05_rescale(D, Hq, Hk, window):
    """Logits with a large spread (scale 1, keys growing along the sequence): the running max
    climbs block after block, so the lazy O rescale and the two softmax warps' max exchange run
    on most blocks."""
    import micro_engram_fork_b200 as me
    from micro_engram_fork_b200.ops.attention import attention_ref, doc_starts

    torch.manual_seed(1)
    lens = [600, 3, 420]
    T = sum(lens)
    pos = torch.cat([torch.arange(n) for n in lens]).to(_dev())
    ds = doc_starts(pos)
    q = (torch.randn(T, Hq, D, device=_dev()) * 0.5 + 0.3).to(torch.bfloat16)
    ramp = torch.linspace(0.0, 1.0, T, device=_dev())[:, None, None]
    k = (torch.randn(T, Hk, D, device=_dev()) * 0.5 + ramp).to(torch.bfloat16)
    v = torch.randn(T, Hk, D, device=_dev()).to(torch.bfloat16)
    o, lse = me.native().attn_fwd_tc(q, k, v, ds, window or 0, 1.0)
    torch.cuda.synchronize()
    assert int(me.native().attn_tc_status(0)[0]) == 0, "tcgen05 attention reported a timeout"
    o32, lse32 = attention_ref(q.float(), k.float(), v.float(), ds, window, 1.0)
    ob, _ = attention_ref(q, k, v, ds, window, 1.0)
    noise_floor_check(o, o32, ob.to(torch.bfloat16), rel=2.0, eps=2e-3, name="attn tc out (rescale)")
    torch.testing.assert_close(lse, lse32, rtol=1e-3, atol=1e-2)


@cuda
@pytest.mark.parametrize("dtype,rowwise", [(torch.float32, True), (torch.bfloat16, True), (torch.bfloat16, False)])
def test_adam_rows_batched_matches_per_table(dtype, rowwise):
    """The batched touched-row AdamW (all tables of a store in one launch, 8 lanes per row) against
    the per-table kernel, without stochastic rounding: same updates up to the order of the
    row-mean reduction; accumulators, pos entries cleared in both."""
    from micro_engram_fork_b200 import native
    from micro_engram_fork_b200.ops.engram import adam_touched
    from micro_engram_fork_b200.parallel.row_store import RowStore

    torch.manual_seed(3)
    rows, dim, n = [1500, 2600, 999], 64, 800
    idx = torch.stack([torch.randint(0, r, (n,)) for r in rows]).to(_dev())
    g = torch.randn(n, len(rows) * dim, device=_dev()).to(dtype)
    results = []
    for batched in (False, True):
        st = RowStore(rows, dim, dtype, 0, 1, _dev(), capacity=n)
        gen = torch.Generator().manual_seed(1)
        for k in range(len(rows)):
            st.shard(k).copy_(torch.randn(rows[k], dim, generator=gen) * 0.02)
        ms = [torch.zeros(r, dim, device=_dev(), dtype=dtype) for r in rows]
        vs = [torch.zeros(r, device=_dev()) if rowwise else torch.zeros(r, dim, device=_dev(), dtype=dtype)
              for r in rows]
        for step in (1, 2):
            st.push_grads(g, idx, 1.0)
            bc1, bc2 = 1 - 0.9 ** step, 1 - 0.999 ** step
            if batched:
                native().engram_adam_rows([st.shard(k) for k in range(3)], ms, vs, st.acc, st.pos, st.list, st.count,
                                          [0, 1, 2], [bc1] * 3, [bc2] * 3, [step] * 3, None, 1e-2, 0.9, 0.999, 1e-8,
                                          0.01, False, 5)
            else:
                for k in range(3):
                    adam_touched(st.shard(k), ms[k], vs[k], st.acc[k], st.pos[k], st.list[k], st.count[k], None, 1e-2,
                                 0.9, 0.999, 1e-8, 0.01, bc1, bc2, False, 5, step, k)
            for c in st.count:
                c.zero_()
        torch.cuda.synchronize()
        results.append(([st.shard(k).float().cpu() for k in range(3)], [m.float().cpu() for m in ms],
                        [v.float().cpu() for v in vs]))
        assert all(float(a.abs().sum()) == 0.0 for a in st.acc) and all(int(p.abs().sum()) == 0 for p in st.pos)
    tol = 1e-6 if dtype == torch.float32 else 1e-2
    for a_list, b_list in zip(results[0], results[1]):
        for a, b in zip(a_list, b_list):
            torch.testing.assert_close(b, a, rtol=tol, atol=tol * float(a.abs().max()) + 1e-12)
