"""GPU numerics of the persistent tcgen05 GEMM (csrc/gemm.cu) and its fused epilogues against
plain fp32 PyTorch: within 1.5x the bf16 noise floor (the error of the same product computed
by PyTorch in bf16), plus a small eps. Shapes cover tails in M, N and K, both B layouts, and
the decoder's projections at a reduced token count."""
import pytest
import torch

from helpers import noise_floor_check

pytestmark = pytest.mark.gpu

cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")


def _dev():
    return torch.device("cuda", 0)


def _status_ok():
    import micro_engram_fork_b200 as me

    torch.cuda.synchronize()
    st = me.native().gemm_status(0)
    code = int(st[0])
    st.zero_()
    return code == 0


SHAPES = [(128, 256, 64), (300, 520, 200), (1024, 1536, 4096), (257, 384, 1536), (40, 8, 24),
          (2048, 5376, 8192), (1024, 16384, 5376)]


@cuda
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_kmajor(M, N, K):
    from micro_engram_fork_b200.ops.linear import linear

    torch.manual_seed(0)
    A = torch.randn(M, K, device=_dev()).to(torch.bfloat16)
    W = (torch.randn(N, K, device=_dev()) / K ** 0.5).to(torch.bfloat16)
    C = linear(A, W)
    assert _status_ok(), "tcgen05 GEMM reported a timeout"
    noise_floor_check(C, A.float() @ W.float().t(), A @ W.t(), rel=1.5, eps=1e-2, name=f"gemm {M}x{N}x{K}")


@cuda
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_nmajor(M, N, K):
    """out[M, N] = A[M, K] . W[K, N] (the dX product of a frozen projection)."""
    from micro_engram_fork_b200.ops.linear import linear_t

    torch.manual_seed(1)
    A = torch.randn(M, K, device=_dev()).to(torch.bfloat16)
    W = (torch.randn(K, N, device=_dev()) / K ** 0.5).to(torch.bfloat16)
    C = linear_t(A, W)
    assert _status_ok(), "tcgen05 GEMM reported a timeout"
    noise_floor_check(C, A.float() @ W.float(), A @ W, rel=1.5, eps=1e-2, name=f"gemm_t {M}x{N}x{K}")


@cuda
def test_gemm_out_strided():
    """Writing into a column slice of a wider buffer (row stride > N)."""
    import micro_engram_fork_b200 as me

    torch.manual_seed(2)
    A = torch.randn(300, 512, device=_dev()).to(torch.bfloat16)
    W = (torch.randn(264, 512, device=_dev()) / 23).to(torch.bfloat16)
    buf = torch.full((300, 1024), 7.0, device=_dev(), dtype=torch.bfloat16)
    me.native().gemm(A, W, True, buf[:, 256:520])
    assert _status_ok()
    noise_floor_check(buf[:, 256:520], A.float() @ W.float().t(), A @ W.t(), rel=1.5, eps=1e-2, name="strided")
    assert bool((buf[:, :256] == 7).all()) and bool((buf[:, 520:] == 7).all()), "wrote outside the output slice"


@cuda
@pytest.mark.parametrize("M,F,K", [(300, 264, 200), (1024, 1536, 512), (520, 21504 // 8, 5376 // 4)])
def test_gemm_geglu(M, F, K):
    from micro_engram_fork_b200.ops.linear import geglu_linear
    from micro_engram_fork_b200.ops.norm import geglu_ref

    torch.manual_seed(3)
    h = torch.randn(M, K, device=_dev()).to(torch.bfloat16)
    W = (torch.randn(2 * F, K, device=_dev()) / K ** 0.5).to(torch.bfloat16)
    m, gu = geglu_linear(h, W, save_gu=True)
    assert _status_ok()
    gu32 = h.float() @ W.float().t()
    noise_floor_check(gu, gu32, h @ W.t(), rel=1.5, eps=1e-2, name="gemm_geglu gu")
    noise_floor_check(m, geglu_ref(gu32), geglu_ref(h @ W.t()), rel=1.5, eps=1e-2, name="gemm_geglu m")
    m2, none = geglu_linear(h, W, save_gu=False)
    assert none is None and torch.equal(m, m2)


@cuda
@pytest.mark.parametrize("M,F,K", [(300, 264, 200), (1024, 1536, 512), (520, 21504 // 8, 5376 // 4)])
def test_gemm_dgeglu(M, F, K):
    from micro_engram_fork_b200.ops.linear import dgeglu_linear
    from micro_engram_fork_b200.ops.norm import geglu_bwd_ref

    torch.manual_seed(4)
    g = torch.randn(M, K, device=_dev()).to(torch.bfloat16)
    Wd = (torch.randn(K, F, device=_dev()) / K ** 0.5).to(torch.bfloat16)
    gu = torch.randn(M, 2 * F, device=_dev()).to(torch.bfloat16)
    d = dgeglu_linear(g, Wd, gu)
    assert _status_ok()
    ref = geglu_bwd_ref(g.float() @ Wd.float(), gu.float())
    plain = geglu_bwd_ref(g @ Wd, gu)
    noise_floor_check(d, ref, plain, rel=1.5, eps=1e-2, name="gemm_dgeglu")


@cuda
@pytest.mark.parametrize("T,N,K", [(700, 264, 200), (8192, 5376, 1536), (300, 10752, 1536)])
def test_projection_grads(T, N, K):
    """The trained projection's dX and dW (= dY^T . X on the M-major-A GEMM, fp32 accumulation)
    against fp32 autograd."""
    from micro_engram_fork_b200.ops.linear import projection

    torch.manual_seed(5)
    x = torch.randn(T, K, device=_dev()).to(torch.bfloat16).requires_grad_()
    W = (torch.randn(N, K, device=_dev()) / K ** 0.5).to(torch.bfloat16).requires_grad_()
    g = torch.randn(T, N, device=_dev()).to(torch.bfloat16)
    y = projection(x, W)
    y.backward(g)
    assert _status_ok()
    x32, W32 = x.detach().float().requires_grad_(), W.detach().float().requires_grad_()
    (x32 @ W32.t()).backward(g.float())
    xb, Wb = x.detach().clone().requires_grad_(), W.detach().clone().requires_grad_()
    (xb @ Wb.t()).backward(g)
    noise_floor_check(y, x32 @ W32.t(), xb @ Wb.t(), rel=1.5, eps=1e-2, name="proj y")
    noise_floor_check(x.grad, x32.grad, xb.grad, rel=1.5, eps=1e-2, name="proj dx")
    noise_floor_check(W.grad, W32.grad, Wb.grad, rel=1.5, eps=1e-2, name="proj dW")


@cuda
@pytest.mark.parametrize("kmajor", [True, False])
def test_gemm_bitwise_repeatable(kmajor):
    """Shapes whose last partial wave is split along K (a 5376-wide output over 8192 rows):
    two runs give identical bits (the split partials are summed in a fixed order)."""
    import micro_engram_fork_b200 as me

    torch.manual_seed(6)
    A = torch.randn(8192, 2048, device=_dev()).to(torch.bfloat16)
    W = (torch.randn(5376, 2048, device=_dev()) if kmajor else torch.randn(2048, 5376, device=_dev())) / 45
    W = W.to(torch.bfloat16)
    first = me.native().gemm(A, W, kmajor, None)
    second = me.native().gemm(A, W, kmajor, None)
    assert _status_ok()
    assert torch.equal(first, second)
    ref32 = A.float() @ (W.float().t() if kmajor else W.float())
    noise_floor_check(first, ref32, A @ (W.t() if kmajor else W), rel=1.5, eps=1e-2, name="tail split")
