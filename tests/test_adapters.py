"""The module adapter (reference ``profiling/decode_stage2_ablation.py:78-143``) on
a small random-init ``transformers`` Qwen3 model: structure on CPU, numerics on
the GPU against the oracle."""
import copy

import numpy as np
import pytest
import torch

from oracle import quant_oracle as O
from tests.conftest import assert_matches_oracle, load_kl

kl = load_kl()
transformers = pytest.importorskip("transformers")


def tiny_qwen(layers=2, seed=0):
    cfg = transformers.Qwen3Config(vocab_size=1024, hidden_size=256, intermediate_size=512,
                                   num_hidden_layers=layers, num_attention_heads=4, num_key_value_heads=2,
                                   head_dim=64, tie_word_embeddings=False, max_position_embeddings=256)
    torch.manual_seed(seed)
    model = transformers.Qwen3ForCausalLM(cfg).eval()
    with torch.no_grad():
        for p in model.parameters():
            if p.ndim == 2:
                p.normal_(0.0, 0.02)
    return model


def test_install_structure_on_cpu():
    model = tiny_qwen()
    info = kl.install_quantized_projections(model, layers=[1], lm_head="w8_row")
    assert info["linear_modules"] == 8 and info["layers"] == {1: "w8_row"} and info["lm_head"] == "w8_row"
    attn0, attn1 = model.model.layers[0].self_attn, model.model.layers[1].self_attn
    assert isinstance(attn0.q_proj, torch.nn.Linear)                      # layer 0 untouched
    assert isinstance(attn1.q_proj, kl.adapters.QKVSlice) and attn1.q_proj.out_features == 256
    assert attn1.k_proj.out_features == 128 and attn1.v_proj.out_features == 128
    gp = model.model.layers[1].mlp.gate_proj                              # dense gate/up released
    assert isinstance(gp, kl.adapters.RowSlice) and isinstance(gp.weight, kl.QuantWeight)
    assert isinstance(model.lm_head, kl.QuantLinear)
    assert info["packed_bytes"] < info["dense_bytes_released"]
    # the reference's call-order rule: k before q is an error (no kernel is reached)
    with pytest.raises(RuntimeError, match="call order"):
        attn1.k_proj(torch.zeros(1, 256, dtype=torch.bfloat16))


def test_install_rejects_bad_arguments():
    with pytest.raises(ValueError):
        kl.install_quantized_projections(tiny_qwen(), layers=[2])
    with pytest.raises(ValueError):
        kl.install_quantized_projections(tiny_qwen(), fmt="int3")


def test_fallback_policy_installs_nothing():
    model = tiny_qwen()
    P = kl.kernel_policy
    policy = P.select_qwen_policy(P.DeviceCapabilities("t", 10, 0, 148, 32, 1 << 30), P.qwen_signature(model),
                                  {"model_signature": {"layers": 28, "hidden_size": 1024, "attention_heads": 16,
                                                       "kv_heads": 8, "head_dim": 128}, "architectures": {}})
    assert policy.profile == "fallback"
    assert kl.install_quantized_projections(model, policy)["linear_modules"] == 0


def _deq_w8(w):
    d, s = O.quantize_int8_rowwise(w.detach().float().cpu().numpy())
    return O.dequantize_int8_rowwise(d, s)


@pytest.mark.gpu
@pytest.mark.parametrize("tokens", [1, 5, 300])
def test_fused_modules_match_oracle(tokens):
    model = tiny_qwen().cuda().to(torch.bfloat16)
    layer = model.model.layers[0]
    a, m = layer.self_attn, layer.mlp
    w_qkv = torch.cat([a.q_proj.weight, a.k_proj.weight, a.v_proj.weight]).detach().float()
    w_gu = torch.cat([m.gate_proj.weight, m.up_proj.weight]).detach().float()
    w_down = m.down_proj.weight.detach().float()
    kl.install_quantized_projections(model, layers=[0])
    x = (torch.randn(1, tokens, 256, generator=torch.Generator().manual_seed(tokens))).bfloat16()
    xf = x.float().numpy().reshape(tokens, 256)
    # Q, K, V from one fused launch, served in the module call order
    with torch.no_grad():
        q, k, v = a.q_proj(x.cuda()), a.k_proj(x.cuda()), a.v_proj(x.cuda())
    ref = O.linear_f32(xf, _deq_w8(w_qkv))
    assert_matches_oracle(q.reshape(tokens, -1), ref[:, :256], what="q")
    assert_matches_oracle(k.reshape(tokens, -1), ref[:, 256:384], what="k")
    assert_matches_oracle(v.reshape(tokens, -1), ref[:, 384:], what="v")
    # MLP: fused gate_up + SwiGLU, then down
    with torch.no_grad():
        y = m(x.cuda())
    h = O.bf16_round(O.swiglu(O.bf16_round(O.linear_f32(xf, _deq_w8(w_gu)))))
    assert_matches_oracle(y.reshape(tokens, -1), O.linear_f32(h, _deq_w8(w_down)), what="mlp")


@pytest.mark.gpu
def test_full_forward_tracks_dequantised_dense_model():
    dense = tiny_qwen(layers=2, seed=3).cuda().to(torch.bfloat16)
    quant = copy.deepcopy(dense)
    kl.install_quantized_projections(quant, lm_head="w8_row")
    # the dense twin carries the same dequantised weights (rounded to bf16)
    with torch.no_grad():
        for layer in dense.model.layers:
            for mod in (layer.self_attn.q_proj, layer.self_attn.k_proj, layer.self_attn.v_proj,
                        layer.self_attn.o_proj, layer.mlp.gate_proj, layer.mlp.up_proj, layer.mlp.down_proj):
                mod.weight.copy_(torch.from_numpy(_deq_w8(mod.weight)).to(mod.weight))
        dense.lm_head.weight.copy_(torch.from_numpy(_deq_w8(dense.lm_head.weight)).to(dense.lm_head.weight))
    ids = torch.randint(0, 1024, (2, 24), generator=torch.Generator().manual_seed(5)).cuda()
    with torch.no_grad():
        a = dense(input_ids=ids).logits.float()
        b = quant(input_ids=ids).logits.float()
    cos = torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0).item()
    assert cos > 0.999, cos
    agree = (a.argmax(-1) == b.argmax(-1)).float().mean().item()
    assert agree >= 0.9, agree
    # a decode step (one new token per sequence) through the same modules
    with torch.no_grad():
        step = quant(input_ids=ids[:, :1]).logits
    assert step.shape == (2, 1, 1024) and torch.isfinite(step).all()
