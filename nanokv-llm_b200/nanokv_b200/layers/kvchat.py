"""Drop-in KvChat attention (threshold S -> R compression with a query window).

Attention and MyCompressCompact keep the signatures of
KvChat/layers/attention.py:122-197 and KvChat/layers/compress_utils.py:10-171.
Per layer: store (nkv_store_kvcache), append the active sequences' queries to
the device query ring (nkv_query_window_append), compress the sequences whose
length reached S (nkv_threshold_compress: gather, SnapKV over the W-query
window, top-k and in-place compaction to positions [0, R) in one launch), then
decode (nkv_paged_decode). Prefill steps run nkv_paged_prefill where the
reference calls flash_attn_varlen_func (KvChat/layers/attention.py:105-111).
"""

from __future__ import annotations

import torch
from torch import nn

from .. import ops
from ..utils.context import get_context


def MyCompressCompact(query_window_manager, k_cache: torch.Tensor, v_cache: torch.Tensor,
                      layer_id: int, block_size: int, S: int, R: int, query_window_size: int,
                      num_layers: int, context=None) -> bool:
    """Threshold compression of one layer for every sequence whose
    compress_need_mask entry is True; returns False where the reference does."""
    if context is None:
        context = get_context()
    need_mask = context.compress_need_mask
    if not need_mask or not any(need_mask):
        return False
    W = query_window_size
    num_keep = R - W - 1
    if S - W <= 0 or S <= num_keep + W:  # SnapKV skip rule, L = S
        return False
    seq_idxs = [i for i, n in enumerate(need_mask) if n]
    seq_ids = context.seq_ids
    assert seq_ids is not None, "context.seq_ids is None"
    compress_seq_ids = [seq_ids[i] for i in seq_idxs]
    dev = k_cache.device
    sel = context.compress_selected_t
    slots = context.compress_ring_slots_t
    if sel is None or slots is None:
        t = torch.tensor([seq_idxs, [query_window_manager.slot_of(s) for s in compress_seq_ids]],
                         dtype=torch.int32).to(dev, non_blocking=True)
        sel, slots = t[0], t[1]
        context.compress_selected_t, context.compress_ring_slots_t = sel, slots
    ops.threshold_compress(query_window_manager.ring, slots, layer_id, k_cache, v_cache,
                           context.block_tables, context.context_lens, sel, S, R)
    if layer_id + 1 >= num_layers:
        keep_blocks = (R + block_size - 1) // block_size
        tables = context.block_tables_host
        if tables is None:
            tables = context.block_tables.tolist()
        if context.compression_events is None:
            context.compression_events = []
        for b in seq_idxs:
            context.compression_events.append({
                "batch_index": int(b),
                "layer": int(layer_id),
                "R": int(R),
                "keep_blocks": int(keep_blocks),
                "freed_block_ids": [int(x) for x in tables[b][keep_blocks:] if int(x) >= 0],
            })
        for sid in compress_seq_ids:
            query_window_manager.free(sid)
    return True


class Attention(nn.Module):
    """KvChat/layers/attention.py:122-197 on libnkv."""

    def __init__(self, num_heads, head_dim, scale, num_kv_heads, vllm_config, num_layers):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.scale = scale
        self.num_kv_heads = num_kv_heads
        self.k_cache = self.v_cache = torch.tensor([])
        self.kv_compress_enabled = vllm_config.kv_compress_enabled
        self.kv_compress_N = vllm_config.kv_compress_N
        self.kv_compress_S = vllm_config.kv_compress_S
        self.kv_compress_R = vllm_config.kv_compress_R
        if self.kv_compress_enabled:
            self.query_window_manager = None
            self.query_window_size = vllm_config.query_window_size
            self.num_layers = num_layers

    def forward_qkv(self, qkv: torch.Tensor, positions: torch.Tensor,
                    q_norm_weight: torch.Tensor, k_norm_weight: torch.Tensor,
                    cos_sin_cache: torch.Tensor, eps: float, Layer):
        """KvChat/models/qwen3.py's q/k norm + RoPE + this layer's attention,
        from the qkv projection output: norm, RoPE and the slot write in one
        launch (nkv_qk_norm_rope_store), then the query window, compression
        and decode / prefill on the stored cache."""
        context = get_context()
        k_cache, v_cache = self.k_cache, self.v_cache
        has_cache = bool(k_cache.numel() and v_cache.numel())
        q, v, k = ops.qk_norm_rope_store(
            qkv, positions, cos_sin_cache, q_norm_weight, k_norm_weight, eps, self.num_heads,
            self.num_kv_heads, k_cache=k_cache if has_cache else None,
            v_cache=v_cache if has_cache else None,
            slot_mapping=context.slot_mapping if has_cache else None,
            k_out=None if (has_cache and not context.is_prefill) else torch.empty(
                qkv.size(0), self.num_kv_heads, self.head_dim, dtype=qkv.dtype,
                device=qkv.device))
        return self._attend(q, k, v, Layer, stored=has_cache)

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, Layer):
        return self._attend(q, k, v, Layer, stored=False)

    def _attend(self, q, k, v, Layer, stored: bool):
        context = get_context()
        k_cache, v_cache = self.k_cache, self.v_cache
        qwm = getattr(self, "query_window_manager", None)
        if (not stored and not context.is_prefill and not context.compress_any and k_cache.numel()
                and q.size(0) == context.block_tables.size(0)):
            # decode step without compression: slot write, query-window append
            # and decode in one launch
            ring_args = {}
            if self.kv_compress_enabled and qwm is not None and context.q_window_active_indices:
                if context.q_window_row_slot_t is None:
                    context.q_window_row_slot_t, context.q_window_row_pos_t = qwm.row_indices(
                        context.q_window_active_seq_ids, context.q_window_active_indices,
                        q.size(0))
                ring_args = dict(ring=qwm.ring, layer_id=Layer,
                                 ring_slot_of_row=context.q_window_row_slot_t,
                                 ring_pos_of_row=context.q_window_row_pos_t)
            # the step's metadata and ring indices come from host copies
            o = ops.decode_step(q, k, v, k_cache, v_cache, context.slot_mapping,
                                context.block_tables, context.context_lens, self.scale,
                                metadata_ready=True, **ring_args)
            if ring_args:
                qwm.advance(context.q_window_active_seq_ids, Layer)
            return o.unsqueeze(1)
        if not stored and k_cache.numel() and v_cache.numel():
            ops.store_kvcache(k, v, k_cache, v_cache, context.slot_mapping)
        if not context.is_prefill and self.kv_compress_enabled:
            qwm = self.query_window_manager
            if qwm is not None and context.q_window_active_indices:
                idx = None
                if context.q_window_batch_t is not None:
                    idx = (context.q_window_batch_t, context.q_window_slot_t, context.q_window_pos_t)
                else:
                    idx = qwm.step_indices(context.q_window_active_seq_ids,
                                           context.q_window_active_indices)
                    context.q_window_batch_t, context.q_window_slot_t, context.q_window_pos_t = idx
                qwm.append(context.q_window_active_seq_ids, Layer, q, indices=idx)
            if context.compress_any:
                S = context.runtime_compress_S if context.runtime_compress_S > 0 else self.kv_compress_S
                R = context.runtime_compress_R if context.runtime_compress_R > 0 else self.kv_compress_R
                MyCompressCompact(query_window_manager=qwm, k_cache=k_cache, v_cache=v_cache,
                                  layer_id=Layer, block_size=k_cache.size(1), S=S, R=R,
                                  query_window_size=self.query_window_size, context=context,
                                  num_layers=self.num_layers)
        if context.is_prefill:
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
