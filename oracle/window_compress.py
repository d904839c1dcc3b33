"""CPU restatement of the periodic window compression MyCompressCompact
(nanokvllm/layers/compress_utils.py:9-290). Test infrastructure only.
"""

from __future__ import annotations

import torch

from .snapkv import snapkv_keep


def tail_window(block_tables: torch.Tensor, base_lens: torch.Tensor, seq_idxs: list[int],
                block_size: int, window_blocks: int):
    """get_tail_window_and_tail_slots (compress_utils.py:9-72): window slots
    [m, window_blocks*block_size], old lens, tail lens, tail block ids (-1
    when there is no partial tail block)."""
    B = block_size
    old = base_lens[seq_idxs].long()
    bt = block_tables[seq_idxs].long()
    full = old // B
    tail = old % B
    assert torch.all(full >= window_blocks), f"some full_blocks < window_blocks: {full}"
    wb = (full - window_blocks).unsqueeze(1) + torch.arange(window_blocks).view(1, -1)
    ids = torch.gather(bt, 1, wb)
    assert torch.all(ids >= 0), "window_block_ids contains invalid block id"
    slots = (ids.unsqueeze(-1) * B + torch.arange(B).view(1, 1, B)).reshape(len(seq_idxs), -1)
    tail_idx = torch.clamp(full, max=bt.size(1) - 1)
    tail_ids = torch.gather(bt, 1, tail_idx.unsqueeze(1)).squeeze(1)
    tail_ids = torch.where(tail > 0, tail_ids, torch.full_like(tail_ids, -1))
    return slots, old, tail, tail_ids


def window_compress_ref(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                        block_tables: torch.Tensor, base_lens: torch.Tensor,
                        context_lens: torch.Tensor, seq_idxs: list[int], block_size: int,
                        window_blocks: int, keep_blocks: int, keep_extra_tokens: int,
                        keep_idx_override: torch.Tensor | None = None,
                        exact_scores: bool = False):
    """One layer of MyCompressCompact on CPU tensors, in place.

    Returns (keep_idx [m, keep_tokens] window-relative, new_lens [m]) or
    False where the reference returns False. `keep_idx_override` replaces the
    SnapKV selection (to check the compaction alone on a given kept set);
    `exact_scores` as in oracle.snapkv.snapkv_importance.
    """
    if not seq_idxs:
        return False
    B = block_size
    window_tokens = window_blocks * B
    keep_tokens = keep_blocks * B + keep_extra_tokens
    q_sub = q[seq_idxs].unsqueeze(2)
    slots, old, tail, tail_ids = tail_window(block_tables, base_lens, seq_idxs, B, window_blocks)
    num_blocks, _, Hk, D = k_cache.shape
    kf = k_cache.view(-1, Hk, D)
    k_sub = kf[slots].permute(0, 2, 1, 3).contiguous()
    if keep_idx_override is None:
        keep_idx, _ = snapkv_keep(q_sub, k_sub, num_keep=keep_tokens - 2, window=1,
                                  exact_scores=exact_scores)
        if keep_idx is False:
            return False
    else:
        keep_idx = keep_idx_override.long()
    m = len(seq_idxs)
    src_keep = torch.gather(slots, 1, keep_idx)
    new_lens = old - window_tokens + keep_tokens
    dst_keep = slots[:, :keep_tokens]
    src = [src_keep.reshape(-1)]
    dst = [dst_keep.reshape(-1)]
    for i in range(m):
        t = int(tail[i])
        if t > 0:
            off = torch.arange(t)
            src.append(tail_ids[i] * B + off)
            dst.append(dst_keep[i, -1] + 1 + off)
    src = torch.cat(src)
    dst = torch.cat(dst)
    kflat = k_cache.view(-1, Hk * D)
    vflat = v_cache.view(-1, Hk * D)
    vals_k = kflat.index_select(0, src).clone()
    vals_v = vflat.index_select(0, src).clone()
    kflat.index_copy_(0, dst, vals_k)
    vflat.index_copy_(0, dst, vals_v)
    context_lens[seq_idxs] = new_lens.to(context_lens.dtype)
    return keep_idx, new_lens


def compression_events(block_tables: torch.Tensor, seq_idxs: list[int], new_lens: torch.Tensor,
                       block_size: int, layer_id: int) -> list[dict]:
    """Event records built on the last layer (compress_utils.py:266-288)."""
    events = []
    for i, b in enumerate(seq_idxs):
        keep_blocks_after = (int(new_lens[i]) + block_size - 1) // block_size
        freed = [int(x) for x in block_tables[b, keep_blocks_after:].tolist() if int(x) >= 0]
        events.append({
            "batch_index": int(b),
            "layer": int(layer_id),
            "new_context_len": int(new_lens[i]),
            "keep_blocks": int(keep_blocks_after),
            "freed_block_ids": freed,
            "tail_uncompressed_len_after": 0,
        })
    return events


def window_importance(q: torch.Tensor, k_cache: torch.Tensor, block_tables: torch.Tensor,
                      base_lens: torch.Tensor, seq_idxs: list[int], block_size: int,
                      window_blocks: int, exact_scores: bool = False) -> torch.Tensor:
    """The bf16 SnapKV importance [m, window_tokens - 1] that MyCompressCompact
    ranks for each selected sequence."""
    from .snapkv import snapkv_importance
    slots, _, _, _ = tail_window(block_tables, base_lens, seq_idxs, block_size, window_blocks)
    _, _, Hk, D = k_cache.shape
    k_sub = k_cache.view(-1, Hk, D)[slots].permute(0, 2, 1, 3).contiguous()
    return snapkv_importance(q[seq_idxs].unsqueeze(2), k_sub, 1, exact_scores)


def window_score_rounding_keys(q: torch.Tensor, k_cache: torch.Tensor, block_tables: torch.Tensor,
                               base_lens: torch.Tensor, seq_idxs: list[int], block_size: int,
                               window_blocks: int) -> torch.Tensor:
    """[m, window_tokens - 1] bool: keys where, for some q head, the CPU bf16
    matmul's score differs from the exactly rounded score -- the only keys
    at which the reference's importance on this CPU and the exact-score
    importance may differ."""
    slots, _, _, _ = tail_window(block_tables, base_lens, seq_idxs, block_size, window_blocks)
    _, _, Hk, D = k_cache.shape
    K = k_cache.view(-1, Hk, D)[slots].permute(0, 2, 1, 3)[:, :, :-1]   # [m, Hk, n, D]
    Q = q[seq_idxs]                                                     # [m, Hq, D]
    g = Q.size(1) // Hk
    Qg = Q.view(len(seq_idxs), Hk, g, 1, D)
    Kt = K.transpose(-1, -2).unsqueeze(2)
    cpu = torch.matmul(Qg, Kt)
    exact = torch.matmul(Qg.double(), Kt.double()).float().to(torch.bfloat16)
    return (cpu.view(torch.int16) != exact.view(torch.int16)).flatten(1, 3).any(1)
