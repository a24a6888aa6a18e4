"""NF4 frozen base (load_in_4bit): the codec against its definition, the CUDA kernels against
the PyTorch reference codec, and a quantized model against the same model holding the
dequantized weights in bf16 (identical math, so identical outputs)."""
import copy

import pytest
import torch

from micro_engram_fork_b200.models import gemma as G
from micro_engram_fork_b200.models import nf4


def test_codec_reference():
    torch.manual_seed(0)
    w = torch.randn(8, 128) * torch.linspace(0.1, 3, 8)[:, None]
    codes, absmax = nf4.quantize_ref(w)
    assert codes.dtype == torch.uint8 and codes.numel() == w.numel() // 2 and absmax.numel() == w.numel() // 64
    back = nf4.dequant_ref(codes, absmax, w.shape, torch.float32)
    # every weight lands on its nearest level: error at most half the widest level gap x absmax
    gap = (nf4.NF4_LEVELS[1:] - nf4.NF4_LEVELS[:-1]).max().item() / 2
    err = (back - w).abs().reshape(-1, 64) / absmax[:, None]
    assert err.max().item() <= gap + 1e-6
    # the block maximum and exact zeros survive exactly
    w2 = w.clone()
    w2[0, :64] = 0
    c2, a2 = nf4.quantize_ref(w2)
    b2 = nf4.dequant_ref(c2, a2, w2.shape, torch.float32)
    assert torch.equal(b2[0, :64], torch.zeros(64))
    i = w[1, :64].abs().argmax()
    assert torch.allclose(back[1, i], w[1, i])


def _tiny(seed=0):
    cfg = G.tiny_config()
    torch.manual_seed(seed)
    m = G.GemmaForCausalLM(cfg)
    G.init_random_(m, seed=seed)
    return m.eval()


def _dequantized_copy(m):
    """The same model with every projection replaced by its NF4 round trip, in plain bf16 buffers."""
    ref = copy.deepcopy(m)
    for layer in G.text_of(ref).layers:
        for name, w in zip(nf4.NF4Weights.NAMES, nf4._weights(layer)):
            c, a = nf4.quantize_ref(w)
            w.data.copy_(nf4.dequant_ref(c, a, w.shape, w.dtype))
    return ref


def test_quantized_model_equals_dequantized_weights_cpu():
    m = _tiny()
    ref = _dequantized_copy(m)
    stored, freed = nf4.quantize_model_nf4(m)
    assert 0 < stored < freed
    ids = torch.randint(0, G.tiny_config().vocab_size, (1, 40))
    with torch.no_grad():
        torch.testing.assert_close(m(ids), ref(ids), rtol=0, atol=0)


@pytest.mark.gpu
def test_nf4_kernels_match_reference():
    torch.manual_seed(1)
    w = (torch.randn(384, 512) * 0.05).to(torch.bfloat16).cuda()
    codes, absmax = nf4.quantize(w)
    rc, ra = nf4.quantize_ref(w.cpu())
    assert torch.equal(codes.cpu(), rc) and torch.equal(absmax.cpu(), ra)
    out = torch.empty_like(w)
    nf4.dequant_into(codes, absmax, out)
    assert torch.equal(out.cpu(), nf4.dequant_ref(rc, ra, w.shape))


@pytest.mark.gpu
@pytest.mark.parametrize("checkpoint", [False, "full", "selective"])
def test_quantized_model_equals_dequantized_weights_gpu(checkpoint):
    """Forward and backward of the native layers: each layer re-expands its own weights."""
    m = _tiny(2)
    G.cast_projections_(m, torch.bfloat16)
    m = m.cuda()
    ref = _dequantized_copy(m)
    nf4.quantize_model_nf4(m)
    ids = torch.randint(0, G.tiny_config().vocab_size, (1, 200), device="cuda")
    with torch.no_grad():
        torch.testing.assert_close(m(ids), ref(ids), rtol=0, atol=0)
    grads = []
    x0 = torch.randn(200, G.tiny_config().hidden_size, device="cuda", dtype=torch.bfloat16)
    for model in (m, ref):
        text = G.text_of(model)
        emb = x0.clone().requires_grad_(True)
        pos = torch.arange(200, device="cuda")
        from micro_engram_fork_b200.ops.attention import doc_starts

        ds = doc_starts(pos)
        x = emb
        for layer in text.layers:
            layer.gradient_checkpointing = checkpoint
            x = layer(x, pos, ds)
        x.float().pow(2).sum().backward()
        grads.append(emb.grad)
    torch.testing.assert_close(grads[0], grads[1], rtol=0, atol=0)
