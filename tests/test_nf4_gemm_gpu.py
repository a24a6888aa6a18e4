"""The tcgen05 GEMM with its B operand dequantised from NF4 inside the kernel (gemm_nf4,
gemm_geglu_nf4, gemm_dgeglu_nf4) against the two-step path: nf4_dequant into a bf16 weight,
then the bf16 GEMM. Both feed the tensor cores the same bf16 values in the same order, so the
outputs must be bitwise equal. The two-step path itself is checked against fp32 PyTorch in
test_gemm_gpu.py and test_nf4 tests; here the dequantised weight is also compared with the CPU
NF4 codec. Shapes cover partial tiles in M and N, K tails (N-major), and both layouts."""
import pytest
import torch

pytestmark = pytest.mark.gpu

cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")


def _dev():
    return torch.device("cuda", 0)


def _nf4(rows, cols, seed):
    from micro_engram_fork_b200 import native
    from micro_engram_fork_b200.models.nf4 import dequant_ref

    g = torch.Generator(device=_dev()).manual_seed(seed)
    w = (torch.randn(rows, cols, device=_dev(), generator=g) * 0.05).to(torch.bfloat16)
    codes, absmax = native().nf4_quantize(w)[:2]
    wq = torch.empty_like(w)
    native().nf4_dequant(codes, absmax, wq)
    assert torch.equal(wq.cpu(), dequant_ref(codes.cpu(), absmax.cpu(), (rows, cols)))
    return codes, absmax, wq


def _status_ok():
    from micro_engram_fork_b200 import native

    return int(native().gemm_status(0)[0]) == 0


@cuda
@pytest.mark.parametrize("M,N,K", [(300, 520, 256), (1024, 1536, 4096), (40, 64, 128), (2048, 5376, 1024)])
def test_nf4_forward_matches_two_step(M, N, K):
    from micro_engram_fork_b200 import native

    C = native()
    codes, absmax, wq = _nf4(N, K, M + N)
    A = torch.randn(M, K, device=_dev()).to(torch.bfloat16)
    got = C.gemm_nf4(A, codes, absmax, N, K, True, None)
    want = C.gemm(A, wq, True, None)
    torch.cuda.synchronize()
    assert _status_ok()
    assert torch.equal(got, want), (got.float() - want.float()).abs().max().item()


@cuda
@pytest.mark.parametrize("M,N,K", [(300, 576, 200), (1024, 1536, 4096), (520, 2688, 1344)])
def test_nf4_input_grad_matches_two_step(M, N, K):
    """dX = g . W with W [K, N] stored NF4 along its rows (the N-major B operand)."""
    from micro_engram_fork_b200 import native

    C = native()
    codes, absmax, wq = _nf4(K, N, M + 7)
    g = torch.randn(M, K, device=_dev()).to(torch.bfloat16)
    got = C.gemm_nf4(g, codes, absmax, K, N, False, None)
    want = C.gemm(g, wq, False, None)
    torch.cuda.synchronize()
    assert _status_ok()
    assert torch.equal(got, want), (got.float() - want.float()).abs().max().item()


@cuda
@pytest.mark.parametrize("M,F,K", [(300, 264, 256), (1024, 1536, 512)])
def test_nf4_geglu_matches_two_step(M, F, K):
    from micro_engram_fork_b200 import native

    C = native()
    codes, absmax, wq = _nf4(2 * F, K, F)
    h = torch.randn(M, K, device=_dev()).to(torch.bfloat16)
    m, gu = C.gemm_geglu_nf4(h, codes, absmax, 2 * F, K, True)
    m2, gu2 = C.gemm_geglu(h, wq, True)
    torch.cuda.synchronize()
    assert _status_ok()
    assert torch.equal(m, m2) and torch.equal(gu, gu2)


@cuda
@pytest.mark.parametrize("M,F,K", [(300, 320, 200), (520, 2688, 1344)])
def test_nf4_dgeglu_matches_two_step(M, F, K):
    from micro_engram_fork_b200 import native

    C = native()
    codes, absmax, wq = _nf4(K, F, K + 1)
    dy = torch.randn(M, K, device=_dev()).to(torch.bfloat16)
    gu = torch.randn(M, 2 * F, device=_dev()).to(torch.bfloat16)
    got = C.gemm_dgeglu_nf4(dy, codes, absmax, K, F, gu)
    want = C.gemm_dgeglu(dy, wq, gu)
    torch.cuda.synchronize()
    assert _status_ok()
    assert torch.equal(got, want), (got.float() - want.float()).abs().max().item()
