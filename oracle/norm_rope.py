"""CPU restatement of the per-layer q/k RMSNorm + rotary embedding of the
Qwen3 attention block and the following slot write -- test infrastructure
only (see oracle/__init__.py).

Reference: q_norm / k_norm (nanokvllm/models/qwen3.py:109-111 with
RMSNorm, nanokvllm/layers/layernorm.py:16-25), rotary_emb (qwen3.py:113 with
RotaryEmbedding, nanokvllm/layers/rotary_embedding.py:7-45), then
store_kvcache (nanokvllm/layers/attention.py:72-73).
"""

from __future__ import annotations

import torch


def rope_cache(max_positions: int, base: float, head_dim: int = 128) -> torch.Tensor:
    """[max_positions, head_dim] fp32: cos(t * f_i) for the first half, sin for
    the second, f_i = base^(-2i / head_dim) (rotary_embedding.py:28-35)."""
    inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float) / head_dim))
    t = torch.arange(max_positions, dtype=torch.float)
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1)


def rms_norm_ref(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """bf16(bf16(x * rsqrt(mean(x^2) + eps)) * weight), fp32 inside
    (layernorm.py:16-25)."""
    xf = x.float()
    var = xf.pow(2).mean(dim=-1, keepdim=True)
    return (xf * torch.rsqrt(var + eps)).to(x.dtype) * weight


def rope_ref(x: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor) -> torch.Tensor:
    """Rotate-half rotary embedding in fp32, result rounded to x's dtype
    (rotary_embedding.py:7-15, 37-45). x [T, H, D], cos_sin [max_pos, D]."""
    cs = cos_sin[positions.long()].unsqueeze(1)
    cos, sin = cs.chunk(2, dim=-1)
    x1, x2 = torch.chunk(x.float(), 2, dim=-1)
    return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1).to(x.dtype)


def qk_norm_rope_store_ref(qkv: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor,
                           q_weight: torch.Tensor, k_weight: torch.Tensor, eps: float,
                           num_q_heads: int, num_kv_heads: int, k_cache=None, v_cache=None,
                           slot_mapping=None):
    """Returns (q, k, v) as the attention layer receives them, and writes k / v
    into the cache slots like store_kvcache (slot -1 skipped)."""
    D = 128
    T = qkv.shape[0]
    q, k, v = qkv.split([num_q_heads * D, num_kv_heads * D, num_kv_heads * D], dim=-1)
    q = rms_norm_ref(q.reshape(T, num_q_heads, D), q_weight, eps)
    k = rms_norm_ref(k.reshape(T, num_kv_heads, D), k_weight, eps)
    q = rope_ref(q, positions, cos_sin)
    k = rope_ref(k, positions, cos_sin)
    v = v.reshape(T, num_kv_heads, D)
    if k_cache is not None:
        from oracle.attention import store_kvcache_ref
        store_kvcache_ref(k, v, k_cache, v_cache, slot_mapping)
    return q, k, v
