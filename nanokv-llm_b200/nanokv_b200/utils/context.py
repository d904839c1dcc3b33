"""The per-step metadata contract of the attention path.

Field names, defaults and the set_context / get_context / reset_context
functions follow the reference's Context (nanokvllm/utils/context.py:3-40)
so that ModelRunner code written against it runs unchanged. The KvChat
variant's fields (KvChat/utils/context.py:3-21: is_prefill, seq_ids,
q_window_active_*, runtime_compress_S/R) are carried by the same class.

Additions, all optional and defaulting to "not provided":
  compress_selected_t        int32 device tensor of compress_selected_batch_indices
                             (built once per step instead of once per layer)
  compress_base_context_lens_host / block_tables_host
                             host copies the scheduler already has, so the
                             last layer builds compression events without a
                             device->host sync
  compress_ring_slots_t / q_window_*_t
                             device index tensors of the KvChat query window
                             (per active row, and per batch row for the fused
                             decode step)
  compress_device_select, compress_topk, compress_tail_uncompressed_t,
  compress_selected_host     selection of a periodic compression step on the
                             device, so the step can be replayed from a CUDA
                             graph (see compress_utils.MyCompressCompact)
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class Context:
    use_decode_kernel: bool = False
    cu_seqlens_q: torch.Tensor | None = None
    cu_seqlens_k: torch.Tensor | None = None
    max_seqlen_q: int = 0
    max_seqlen_k: int = 0
    slot_mapping: torch.Tensor | None = None
    context_lens: torch.Tensor | None = None
    block_tables: torch.Tensor | None = None

    compression_events: list | None = None
    compress_need_mask: list | None = None
    compress_any: bool = False

    is_compress_step: bool = False
    compress_selected_batch_indices: list | None = None
    compress_selected_seq_ids: list[int] | None = None
    compress_base_context_lens: torch.Tensor | None = None

    # KvChat threshold path (KvChat/utils/context.py)
    is_prefill: bool = False
    seq_ids: list[int] | None = None
    q_window_active_indices: list | None = None
    q_window_active_seq_ids: list[int] | None = None
    runtime_compress_S: int = 0
    runtime_compress_R: int = 0

    # device/host companions (see module docstring)
    compress_selected_t: torch.Tensor | None = None
    compress_base_context_lens_host: list[int] | None = None
    block_tables_host: list[list[int]] | None = None
    compress_ring_slots_t: torch.Tensor | None = None
    q_window_batch_t: torch.Tensor | None = None
    q_window_slot_t: torch.Tensor | None = None
    q_window_pos_t: torch.Tensor | None = None
    q_window_row_slot_t: torch.Tensor | None = None
    q_window_row_pos_t: torch.Tensor | None = None

    # device-side selection of a periodic compression step (graph-capturable):
    # the layers select at layer 0 into compress_selected_t ([topk], -1
    # padded) from context_lens and compress_tail_uncompressed_t, compress
    # with that fixed-size list, and copy it to compress_selected_host (pinned)
    # at the last layer; the host builds the events after the step.
    compress_device_select: bool = False
    compress_topk: int = 0
    compress_tail_uncompressed_t: torch.Tensor | None = None
    compress_selected_host: torch.Tensor | None = None


_CONTEXT = Context()


def get_context() -> Context:
    return _CONTEXT


def set_context(use_decode_kernel, cu_seqlens_q=None, cu_seqlens_k=None, max_seqlen_q=0,
                max_seqlen_k=0, slot_mapping=None, context_lens=None, block_tables=None) -> None:
    """Same positional contract as the reference's set_context
    (nanokvllm/utils/context.py:27-36): the compression fields start empty."""
    global _CONTEXT
    _CONTEXT = Context(use_decode_kernel, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                       slot_mapping, context_lens, block_tables, compression_events=[],
                       compress_need_mask=None, compress_any=False, is_compress_step=False,
                       compress_selected_batch_indices=None, compress_selected_seq_ids=None,
                       compress_base_context_lens=None, is_prefill=not use_decode_kernel)


def set_kvchat_context(is_prefill, cu_seqlens_q=None, cu_seqlens_k=None, max_seqlen_q=0,
                       max_seqlen_k=0, slot_mapping=None, context_lens=None,
                       block_tables=None) -> None:
    """KvChat's set_context (KvChat/utils/context.py:27-36), whose first
    argument is is_prefill rather than use_decode_kernel."""
    set_context(not is_prefill, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                slot_mapping, context_lens, block_tables)
    _CONTEXT.is_prefill = bool(is_prefill)
    _CONTEXT.runtime_compress_S = 0
    _CONTEXT.runtime_compress_R = 0


def reset_context() -> None:
    global _CONTEXT
    _CONTEXT = Context()
