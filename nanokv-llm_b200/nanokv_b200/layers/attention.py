"""Drop-in Attention module for nano-kvllm's decode path on B200.

Same class name, constructor and forward(q, k, v, Layer) as the reference's
nanokvllm/layers/attention.py:42-108, same order of work per layer:

  1. store_kvcache of the step's K/V rows      -> nkv_store_kvcache
  2. periodic window compression when the Context asks for it
                                               -> nkv_window_compress (MyCompressCompact)
  3. decode attention over the paged cache     -> nkv_paged_decode
     (flash_attn_with_kvcache in the reference), or, on prefill / mixed
     steps (use_decode_kernel False), variable-length causal attention
                                               -> nkv_paged_prefill
     (flash_attn_varlen_func in the reference, :96-102)

On a decode step that does not compress, 1 and 3 run as one launch
(nkv_decode_step), which writes each kv head's new row right before reading
that tile.
"""

from __future__ import annotations

import torch
from torch import nn

from .. import ops
from ..ops import store_kvcache  # noqa: F401  (same public name as the reference module)
from ..utils.context import get_context
from .compress_utils import MyCompressCompact


class Attention(nn.Module):

    def __init__(self, num_heads, head_dim, scale, num_kv_heads, vllm_config, num_layers):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.scale = scale
        self.num_kv_heads = num_kv_heads
        self.k_cache = self.v_cache = torch.tensor([])
        self.kv_compress_enabled = vllm_config.kv_compress_enabled
        if self.kv_compress_enabled:
            self.num_layers = num_layers
            self.kv_compress_window_blocks = vllm_config.kv_compress_window_blocks
            self.kv_compress_keep_blocks = vllm_config.kv_compress_keep_blocks
            self.kv_compress_keep_extra_tokens = vllm_config.kv_compress_keep_extra_tokens

    def forward_qkv(self, qkv: torch.Tensor, positions: torch.Tensor,
                    q_norm_weight: torch.Tensor, k_norm_weight: torch.Tensor,
                    cos_sin_cache: torch.Tensor, eps: float, Layer):
        """The block of nanokvllm/models/qwen3.py:109-114 from the qkv
        projection output: q/k RMSNorm + RoPE + the slot write in one launch
        (nkv_qk_norm_rope_store), then this layer's attention (compression,
        decode or prefill) on the stored cache. Same result as
        q_norm / k_norm / rotary_emb followed by forward(q, k, v, Layer)."""
        context = get_context()
        k_cache, v_cache = self.k_cache, self.v_cache
        has_cache = bool(k_cache.numel() and v_cache.numel())
        q, v, k = ops.qk_norm_rope_store(
            qkv, positions, cos_sin_cache, q_norm_weight, k_norm_weight, eps, self.num_heads,
            self.num_kv_heads, k_cache=k_cache if has_cache else None,
            v_cache=v_cache if has_cache else None,
            slot_mapping=context.slot_mapping if has_cache else None,
            k_out=None if (has_cache and context.use_decode_kernel) else torch.empty(
                qkv.size(0), self.num_kv_heads, self.head_dim, dtype=qkv.dtype,
                device=qkv.device))
        return self._attend(q, k, v, Layer, stored=has_cache)

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, Layer):
        return self._attend(q, k, v, Layer, stored=False)

    def _attend(self, q, k, v, Layer, stored: bool):
        context = get_context()
        k_cache, v_cache = self.k_cache, self.v_cache
        compressing = (context.use_decode_kernel and self.kv_compress_enabled
                       and context.is_compress_step
                       and (context.compress_device_select
                            or bool(context.compress_selected_batch_indices)))
        if (not stored and context.use_decode_kernel and not compressing and k_cache.numel()
                and q.size(0) == context.block_tables.size(0)):
            # decode step without compression: slot write + decode in one launch;
            # the step's metadata comes from host copies, so no kernel right
            # before this one writes it
            o = ops.decode_step(q, k, v, k_cache, v_cache, context.slot_mapping,
                                context.block_tables, context.context_lens, self.scale,
                                metadata_ready=True)
            return o.unsqueeze(1)
        if not stored and k_cache.numel() and v_cache.numel():
            ops.store_kvcache(k, v, k_cache, v_cache, context.slot_mapping)

        if compressing:
            MyCompressCompact(q_current=q, k_cache=k_cache, v_cache=v_cache, layer_id=Layer,
                              block_size=k_cache.size(1),
                              window_blocks=self.kv_compress_window_blocks,
                              keep_blocks=self.kv_compress_keep_blocks,
                              keep_extra_tokens=self.kv_compress_keep_extra_tokens,
                              num_layers=self.num_layers, context=context)

        if not context.use_decode_kernel:
            if context.block_tables is not None:  # keys come from the paged cache
                k, v = k_cache, v_cache
            return ops.flash_attn_varlen_func(q, k, v, max_seqlen_q=context.max_seqlen_q,
                                              cu_seqlens_q=context.cu_seqlens_q,
                                              max_seqlen_k=context.max_seqlen_k,
                                              cu_seqlens_k=context.cu_seqlens_k,
                                              softmax_scale=self.scale, causal=True,
                                              block_table=context.block_tables)
        return ops.flash_decode_with_kvcache(q.unsqueeze(1), k_cache, v_cache,
                                             cache_seqlens=context.context_lens,
                                             block_table=context.block_tables,
                                             softmax_scale=self.scale, causal=True)
