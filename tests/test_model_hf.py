"""Our Gemma-4-style decoder == HF transformers' Gemma4ForCausalLM (the oracle), on CPU fp32:
weights saved by HF load through our safetensors loader; logits match for one document and
for packed documents (HF isolates them via position_ids on the eager path with a mask)."""
import tempfile

import pytest
import torch

from micro_engram_fork_b200.models import gemma as G


def _hf_model(kv_eq):
    from transformers import Gemma4ForCausalLM
    from transformers.models.gemma4.configuration_gemma4 import Gemma4TextConfig

    cfg = Gemma4TextConfig(vocab_size=512, hidden_size=128, intermediate_size=256, num_hidden_layers=3,
                           num_attention_heads=4, num_key_value_heads=2, head_dim=32, global_head_dim=64,
                           num_global_key_value_heads=1, attention_k_eq_v=kv_eq, hidden_size_per_layer_input=0,
                           layer_types=["sliding_attention", "sliding_attention", "full_attention"], sliding_window=8,
                           final_logit_softcapping=30.0, attn_implementation="eager")
    torch.manual_seed(0)
    m = Gemma4ForCausalLM(cfg).float().eval()
    with torch.no_grad():  # non-trivial norm weights and layer scalars
        for n, p in m.named_parameters():
            if "norm" in n:
                p.uniform_(0.5, 1.5)
        for layer in m.model.layers:
            layer.layer_scalar.fill_(0.9)
    return m


@pytest.mark.parametrize("kv_eq", [False, True])
def test_decoder_matches_hf(kv_eq):
    hf = _hf_model(kv_eq)
    d = tempfile.mkdtemp()
    hf.save_pretrained(d)
    ours = G.GemmaForCausalLM(G.GemmaConfig.from_pretrained(d))
    missing = G.load_hf_weights(ours, d)
    assert not missing, missing
    ours.eval()
    torch.manual_seed(1)
    ids = torch.randint(0, 512, (1, 40))
    with torch.no_grad():
        want = hf(input_ids=ids).logits[0].float()
        got = ours(ids)
    torch.testing.assert_close(got, want, rtol=1e-4, atol=1e-4)


def test_packed_documents_are_isolated():
    hf = _hf_model(True)
    d = tempfile.mkdtemp()
    hf.save_pretrained(d)
    ours = G.GemmaForCausalLM(G.GemmaConfig.from_pretrained(d))
    G.load_hf_weights(ours, d)
    torch.manual_seed(2)
    a, b = torch.randint(0, 512, (1, 17)), torch.randint(0, 512, (1, 23))
    packed = torch.cat([a, b], dim=1)
    pos = torch.cat([torch.arange(17), torch.arange(23)])
    with torch.no_grad():
        got = ours(packed, pos)
        ref_a = hf(input_ids=a).logits[0].float()
        ref_b = hf(input_ids=b).logits[0].float()
    torch.testing.assert_close(got[:17], ref_a, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(got[17:], ref_b, rtol=1e-4, atol=1e-4)


def test_fused_views_and_state_dict_names():
    cfg = G.tiny_config()
    m = G.GemmaForCausalLM(cfg)
    G.init_random_(m, 0)
    layer = m.model.layers[0]
    assert layer.self_attn.q_proj.weight.data_ptr() == layer.qkv_weight.data_ptr()
    keys = set(m.state_dict())
    assert "model.layers.0.self_attn.q_proj.weight" in keys and "model.layers.3.self_attn.v_proj.weight" not in keys
    assert "model.layers.0.mlp.gate_proj.weight" in keys and not any("qkv_weight" in k for k in keys)
    G.cast_projections_(m, torch.bfloat16)
    assert layer.self_attn.q_proj.weight.dtype == torch.bfloat16 and layer.input_layernorm.weight.dtype == torch.float32
    assert layer.self_attn.k_proj.weight.data_ptr() == layer.qkv_weight.data_ptr() + \
        layer.n_q * layer.head_dim * cfg.hidden_size * 2
