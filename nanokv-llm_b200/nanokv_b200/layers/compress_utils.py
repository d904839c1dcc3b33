"""Host side of the periodic window compression, same entry point as the
reference's MyCompressCompact (nanokvllm/layers/compress_utils.py:100-290).

Everything the reference does with torch ops and host syncs -- window slot
construction, the K/V gather, SnapKV, the in-place compaction and the
context_lens update -- is one kernel launch here (nkv_window_compress). The
compression events of the last layer are built from host-side copies of the
base lengths and block tables when the scheduler provides them, so a compress
step needs no device->host synchronisation; otherwise they are read back once,
as the reference does.
"""

from __future__ import annotations

import torch

from .. import ops
from ..utils.context import get_context


def _selected_tensor(context, device) -> torch.Tensor:
    t = context.compress_selected_t
    if t is None or t.device != device:
        t = torch.tensor(context.compress_selected_batch_indices, dtype=torch.int32, device=device)
        context.compress_selected_t = t
    return t


def MyCompressCompact(q_current: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                      layer_id: int, block_size: int, window_blocks: int, keep_blocks: int,
                      keep_extra_tokens: int, num_layers: int, context=None) -> bool:
    """Periodic compression of one layer: score the last `window_blocks` full
    blocks with the current query (SnapKV, window=1), keep bos + the top
    keep_tokens-2 + the window's last token, compact them into the window's
    first keep_tokens slots, move the partial tail block after them and set
    context_lens[b] = old - window_tokens + keep_tokens. Returns False exactly
    where the reference does."""
    if context is None:
        context = get_context()
    if (not context.use_decode_kernel) or context.context_lens is None or context.block_tables is None:
        return False
    if context.compress_device_select:
        return _compress_device_selected(q_current, k_cache, v_cache, layer_id, block_size,
                                         window_blocks, keep_blocks, keep_extra_tokens,
                                         num_layers, context)
    selected = context.compress_selected_batch_indices
    if not selected:
        return False
    B = block_size
    window_tokens = window_blocks * B
    keep_tokens = keep_blocks * B + keep_extra_tokens
    num_keep = keep_tokens - 2
    # SnapKV's skip rule (CompressMethod.py:17-18) with L = window_tokens, window = 1
    if window_tokens - 1 <= 0 or window_tokens <= num_keep + 1:
        return False
    base = context.compress_base_context_lens
    assert base is not None, "compress_base_context_lens is None during compress step"
    base_h = context.compress_base_context_lens_host
    if base_h is not None:
        full = [base_h[b] // B for b in selected]
        assert all(f >= window_blocks for f in full), f"some full_blocks < window_blocks: {full}"
    sel = _selected_tensor(context, k_cache.device)
    ops.window_compress(q_current, k_cache, v_cache, context.block_tables, base,
                        context.context_lens, sel, window_blocks, keep_tokens, obs_window=1)

    if layer_id + 1 >= num_layers:
        if context.compression_events is None:
            context.compression_events = []
        if base_h is None:
            base_h = base.tolist()
        tables = context.block_tables_host
        if tables is None:
            tables = context.block_tables.tolist()
        for b in selected:
            new_len = int(base_h[b]) - window_tokens + keep_tokens
            keep_blocks_after = (new_len + B - 1) // B
            freed = [int(x) for x in tables[b][keep_blocks_after:] if int(x) >= 0]
            context.compression_events.append({
                "batch_index": int(b),
                "layer": int(layer_id),
                "new_context_len": int(new_len),
                "keep_blocks": int(keep_blocks_after),
                "freed_block_ids": freed,
                "tail_uncompressed_len_after": 0,
            })
    return True


def _compress_device_selected(q_current, k_cache, v_cache, layer_id, block_size, window_blocks,
                              keep_blocks, keep_extra_tokens, num_layers, context) -> bool:
    """A compression step whose rows are chosen on the device, so that the
    same kernel sequence serves every compression step of a batch size and
    can be captured in a CUDA graph: layer 0 runs nkv_window_select (the
    reference's selection rule) into the fixed-size compress_selected_t and
    snapshots the base lengths; every layer compresses with the -1-padded
    list; the last layer copies the list to pinned host memory, from which
    the host builds the events once the step has finished
    (PeriodicCompressScheduler.events_from_device). Nothing here depends on
    this step's host-side values."""
    B = block_size
    window_tokens = window_blocks * B
    keep_tokens = keep_blocks * B + keep_extra_tokens
    num_keep = keep_tokens - 2
    if window_tokens - 1 <= 0 or window_tokens <= num_keep + 1:
        return False
    sel = context.compress_selected_t
    base = context.compress_base_context_lens
    assert sel is not None and base is not None and context.compress_tail_uncompressed_t is not None
    if layer_id == 0:
        ops.window_select(context.context_lens, context.compress_tail_uncompressed_t, B,
                          window_blocks, context.compress_topk, out_selected=sel,
                          out_base_lens=base)
    ops.window_compress(q_current, k_cache, v_cache, context.block_tables, base,
                        context.context_lens, sel, window_blocks, keep_tokens, obs_window=1)
    if layer_id + 1 >= num_layers and context.compress_selected_host is not None:
        context.compress_selected_host.copy_(sel, non_blocking=True)
    return True
