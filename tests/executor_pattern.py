"""Test helper: the projection call pattern of the reference's serving executor
and its CUDA-graph bucket registry, restated for a contiguous (unpaged) KV
cache so that the quantized drop-in can be exercised where the reference
package is not installed.

* ``fused_projection_weights`` follows ``serving/qwen_executor.py:90-108``
  (``torch.cat`` of ``q/k/v_proj.weight`` and ``gate/up_proj.weight``,
  ``.contiguous()``);
* ``DecodeStepPattern.forward`` follows ``_forward_batch`` (``:155-240``): the
  fused QKV site ``F.linear(normalized, W_qkv).split(...)`` (``:171-174``), q/k
  norms and RoPE, attention over the cache, ``o_proj`` (``:227``), the fused MLP
  site ``F.linear(normalized, W_gate_up).chunk(2)`` then ``down_proj(act(gate) *
  up)`` (``:230-234``), and ``lm_head`` (``:237``);
* ``GraphBuckets`` follows ``serving/graph_buckets.py:13-41`` (warm-up call,
  capture with static inputs, replay copying the inputs in).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def _rotate_half(x):
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def fused_projection_weights(model):
    packed = []
    with torch.no_grad():
        for layer in model.model.layers:
            a, m = layer.self_attn, layer.mlp
            packed.append((torch.cat((a.q_proj.weight, a.k_proj.weight, a.v_proj.weight), dim=0).contiguous(),
                           torch.cat((m.gate_proj.weight, m.up_proj.weight), dim=0).contiguous()))
    return tuple(packed)


class DecodeStepPattern:
    """One decode token per sequence, K/V in a contiguous static cache."""

    def __init__(self, model, batch, max_len, fused_qkv=True, fused_mlp=True):
        self.model = model
        cfg = model.config
        dev = next(p for p in model.parameters()).device
        dt = model.model.embed_tokens.weight.dtype
        nl = len(model.model.layers)
        self.keys = torch.zeros(nl, batch, cfg.num_key_value_heads, max_len, cfg.head_dim, device=dev, dtype=dt)
        self.values = torch.zeros_like(self.keys)
        self.fused_qkv, self.fused_mlp = fused_qkv, fused_mlp
        self.projection_weights = fused_projection_weights(model) if (fused_qkv or fused_mlp) else None

    @torch.inference_mode()
    def forward(self, tokens, positions):
        model, cfg = self.model, self.model.config
        batch = tokens.shape[0]
        hidden = model.model.embed_tokens(tokens[:, None])
        cos, sin = model.model.rotary_emb(hidden, positions[:, None])
        cos, sin = cos[:, None], sin[:, None]
        max_len = self.keys.shape[3]
        steps = torch.arange(max_len, device=tokens.device)
        mask = torch.zeros(batch, 1, 1, max_len, device=tokens.device, dtype=hidden.dtype)
        mask.masked_fill_(steps[None, None, None, :] > positions[:, None, None, None], torch.finfo(hidden.dtype).min)
        rows = torch.arange(batch, device=tokens.device)
        for li, layer in enumerate(model.model.layers):
            residual = hidden
            normalized = layer.input_layernorm(hidden)
            att = layer.self_attn
            q_size, k_size = cfg.num_attention_heads * cfg.head_dim, cfg.num_key_value_heads * cfg.head_dim
            if self.fused_qkv:
                q_raw, k_raw, v_raw = F.linear(normalized, self.projection_weights[li][0]).split(
                    (q_size, k_size, k_size), dim=-1)
            else:
                q_raw, k_raw, v_raw = att.q_proj(normalized), att.k_proj(normalized), att.v_proj(normalized)
            q = att.q_norm(q_raw.view(batch, 1, cfg.num_attention_heads, cfg.head_dim)).transpose(1, 2)
            k = att.k_norm(k_raw.view(batch, 1, cfg.num_key_value_heads, cfg.head_dim)).transpose(1, 2)
            v = v_raw.view(batch, 1, cfg.num_key_value_heads, cfg.head_dim).transpose(1, 2)
            q = q * cos + _rotate_half(q) * sin
            k = k * cos + _rotate_half(k) * sin
            self.keys[li, rows, :, positions] = k[:, :, 0]
            self.values[li, rows, :, positions] = v[:, :, 0]
            out = F.scaled_dot_product_attention(q, self.keys[li], self.values[li], attn_mask=mask,
                                                 scale=cfg.head_dim ** -0.5, enable_gqa=True)
            hidden = residual + att.o_proj(out.transpose(1, 2).reshape(batch, 1, -1))
            residual = hidden
            normalized = layer.post_attention_layernorm(hidden)
            if self.fused_mlp:
                gate, up = F.linear(normalized, self.projection_weights[li][1]).chunk(2, dim=-1)
                mlp_out = layer.mlp.down_proj(layer.mlp.act_fn(gate) * up)
            else:
                mlp_out = layer.mlp(normalized)
            hidden = residual + mlp_out
        hidden = model.model.norm(hidden)
        return model.lm_head(hidden)[:, 0].float()


class GraphBuckets:
    """Shape-keyed CUDA graphs: warm-up call, capture on static inputs, replay."""

    def __init__(self):
        self.graphs = {}

    @torch.inference_mode()
    def capture(self, key, fn, *static_inputs):
        fn(*static_inputs)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            out = fn(*static_inputs)
        self.graphs[key] = (g, static_inputs, out)

    @torch.inference_mode()
    def replay(self, key, *inputs):
        g, static, out = self.graphs[key]
        for dst, src in zip(static, inputs):
            dst.copy_(src)
        g.replay()
        return out
