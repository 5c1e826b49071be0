"""The quantized projections as a drop-in for the serving executor's call
pattern (``serving/qwen_executor.py:90-108,155-240``, restated in
``tests/executor_pattern.py``) and its CUDA-graph buckets
(``serving/graph_buckets.py:13-41``), on a small random-init Qwen3.

CPU: the executor's fused weights build from the installed modules without
copying the packed matrices, and an executor built before the install is
switched over.  GPU: batched decode steps at M in {1, 2, 4, 8, 16} through the
fused F.linear sites track the same steps with the dequantised dense weights,
and every batch bucket captured in a CUDA graph replays bit-identically."""
import copy

import pytest
import torch

from oracle import quant_oracle as O
from tests.conftest import load_kl
from tests.executor_pattern import DecodeStepPattern, GraphBuckets, fused_projection_weights

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


def tiny_policy(model):
    """A dispatch row for the tiny model: every layer int8 with fused QKV and
    gate_up in the executor, quantized lm_head (keys of kernel_policy.py)."""
    P = kl.kernel_policy
    layers = list(range(len(model.model.layers)))
    sig = P.qwen_signature(model)
    profiles = {"model_signature": {"layers": sig.layers, "hidden_size": sig.hidden_size,
                                    "attention_heads": sig.attention_heads, "kv_heads": sig.kv_heads,
                                    "head_dim": sig.head_dim},
                "architectures": {"sm100": {"name": "tiny", "quality_gate_passed": True, "block_size": 16,
                                            "attention_tile": 128, "direct_attention_layers": [],
                                            "fused_gather": False, "native_gqa": False,
                                            "fused_qkv_layers": layers, "fused_mlp_layers": layers,
                                            "w8a16_layers": layers, "quantized_lm_head": "w8_row",
                                            "reason": "test row"}}}
    return P.select_qwen_policy(P.DeviceCapabilities("t", 10, 0, 148, 32, 1 << 30), sig, profiles)


class _Executor:
    """The attributes ``install_quantized_executor`` uses, as the reference's
    QwenPagedExecutor has them (``qwen_executor.py:44-108``)."""

    def __init__(self, model, policy):
        self.model = model
        self.fused_qkv_layers = frozenset(policy.fused_qkv_layers)
        self.fused_mlp_layers = frozenset(policy.fused_mlp_layers)
        self._projection_weights = None
        if self.fused_qkv_layers or self.fused_mlp_layers:
            self.enable_fused_projections(qkv=self.fused_qkv_layers, mlp=self.fused_mlp_layers)

    def enable_fused_projections(self, *, qkv=True, mlp=True):
        self._projection_weights = fused_projection_weights(self.model)
        return self


def test_fused_weights_are_packed_views_on_cpu():
    model = tiny_qwen()
    policy = tiny_policy(model)
    kl.install_quantized_projections(model, policy)
    ex = _Executor(model, policy)
    for li, (wqkv, wgu) in enumerate(ex._projection_weights):
        layer = model.model.layers[li]
        assert isinstance(wqkv, kl.QuantWeight) and tuple(wqkv.shape) == (512, 256)
        assert isinstance(wgu, kl.QuantWeight) and tuple(wgu.shape) == (1024, 256)
        # the cat of adjacent row views is the installed fused matrix itself (no copy)
        assert wqkv.packed.data.data_ptr() == layer.self_attn.kl_qkv.weight_q.data.data_ptr()
        assert wgu.packed.data.data_ptr() == layer.mlp.kl_gate_up.weight_q.data.data_ptr()
    # a dense operation on a quantized weight fails loudly instead of computing something else
    with pytest.raises(TypeError):
        model.model.layers[0].self_attn.o_proj.weight.float()


def test_executor_built_before_install_is_switched_over():
    model = tiny_qwen()
    policy = tiny_policy(model)
    ex = _Executor(model, policy)
    assert not isinstance(ex._projection_weights[0][0], kl.QuantWeight)     # dense bf16 copies
    info = kl.install_quantized_executor(ex, policy)
    assert info["executor_fused_weights"].startswith("rebuilt")
    assert all(isinstance(w, kl.QuantWeight) for pair in ex._projection_weights for w in pair)


def _dequantised_twin(dense):
    """The model with every projection replaced by its dequantised int8 weight (bf16)."""
    twin = copy.deepcopy(dense)
    with torch.no_grad():
        for layer in twin.model.layers:
            for mod in (layer.self_attn.q_proj, layer.self_attn.k_proj, layer.self_attn.v_proj,
                        layer.self_attn.o_proj, layer.mlp.gate_proj, layer.mlp.up_proj, layer.mlp.down_proj):
                q, s = O.quantize_int8_rowwise(mod.weight.detach().float().cpu().numpy())
                mod.weight.copy_(torch.from_numpy(O.dequantize_int8_rowwise(q, s)).to(mod.weight))
        w = twin.lm_head.weight
        q, s = O.quantize_int8_rowwise(w.detach().float().cpu().numpy())
        w.copy_(torch.from_numpy(O.dequantize_int8_rowwise(q, s)).to(w))
    return twin


@pytest.mark.gpu
def test_batched_decode_steps_and_graph_buckets():
    dense = tiny_qwen(seed=7).cuda().to(torch.bfloat16)
    twin = _dequantised_twin(dense)
    quant = copy.deepcopy(dense)
    policy = tiny_policy(quant)
    kl.install_quantized_projections(quant, policy)
    buckets = GraphBuckets()
    gen = torch.Generator().manual_seed(3)
    steps = 6
    decided = 0
    for batch in (1, 2, 4, 8, 16):
        ex_q = DecodeStepPattern(quant, batch, max_len=32)
        ex_d = DecodeStepPattern(twin, batch, max_len=32)
        assert isinstance(ex_q.projection_weights[0][0], kl.QuantWeight)
        tokens = torch.randint(0, 1024, (steps, batch), generator=gen).cuda()
        for t in range(steps):
            pos = torch.full((batch,), t, dtype=torch.long, device="cuda")
            a = ex_q.forward(tokens[t], pos)
            b = ex_d.forward(tokens[t], pos)
            cos = torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0).item()
            assert cos > 0.999, (batch, t, cos)
            # argmax agreement wherever the dense step's decision is clear: its
            # top-1 / top-2 margin exceeds twice the largest logit difference
            err = (a - b).abs().max()
            top2 = b.topk(2, dim=-1).values
            clear = (top2[:, 0] - top2[:, 1]) > 2 * err
            assert torch.equal(a.argmax(-1)[clear], b.argmax(-1)[clear]), (batch, t)
            decided += int(clear.sum())
        # the same decode step captured for this batch bucket replays bit-identically
        tok = tokens[-1].clone()
        pos = torch.full((batch,), steps, dtype=torch.long, device="cuda")
        keys0, values0 = ex_q.keys.clone(), ex_q.values.clone()
        eager = ex_q.forward(tok, pos).clone()
        ex_q.keys.copy_(keys0)
        ex_q.values.copy_(values0)
        buckets.capture(batch, ex_q.forward, tok.clone(), pos.clone())
        ex_q.keys.copy_(keys0)
        ex_q.values.copy_(values0)
        out = buckets.replay(batch, tok, pos)
        torch.cuda.synchronize()
        torch.testing.assert_close(out, eager, rtol=0, atol=0)
    assert decided >= 0.5 * steps * 31, decided      # most rows carry a clear decision
    assert kl._native.device_status(0) == 0


@pytest.mark.gpu
def test_hf_decode_step_graph_with_adapters():
    """A whole greedy decode step of the transformers model with the quantized
    modules installed, captured once and replayed (the fixed-address pattern of
    learning/12_decode_runtime/decode_runtime.py:119-175): replay equals eager."""
    model = tiny_qwen(seed=11).cuda().to(torch.bfloat16)
    kl.install_quantized_projections(model, lm_head="w8_row")
    ids = torch.randint(0, 1024, (1, 1), generator=torch.Generator().manual_seed(1)).cuda()

    @torch.inference_mode()
    def step(tok):
        logits = model(input_ids=tok, use_cache=False).logits
        return logits[:, -1].argmax(-1, keepdim=True), logits[:, -1].float()

    eager_tok, eager_logits = step(ids)
    torch.cuda.synchronize()
    static = ids.clone()
    step(static)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out_tok, out_logits = step(static)
    static.copy_(ids)
    g.replay()
    torch.cuda.synchronize()
    torch.testing.assert_close(out_logits, eager_logits, rtol=0, atol=0)
    assert torch.equal(out_tok, eager_tok)
    # the graph's token feeds the next replay, as the decode loop does
    static.copy_(out_tok)
    g.replay()
    torch.cuda.synchronize()
    nxt_tok, nxt_logits = step(eager_tok)
    torch.testing.assert_close(out_logits, nxt_logits, rtol=0, atol=0)
