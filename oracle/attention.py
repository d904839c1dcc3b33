"""CPU restatement of the store and paged-decode halves of Attention.forward.

Test infrastructure only (see oracle/__init__.py).
"""

from __future__ import annotations

import torch


def store_kvcache_ref(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor,
                      v_cache: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    """In-place slot write, nanokvllm/layers/attention.py:10-30:
    k_cache.view(-1, Hk*D)[slot] = key[i] for every i with slot != -1."""
    N, Hk, D = key.shape
    kf = k_cache.view(-1, Hk * D)
    vf = v_cache.view(-1, Hk * D)
    slots = slot_mapping.to(torch.long)
    live = slots != -1
    idx = torch.nonzero(live).flatten()
    if idx.numel():
        kf[slots[idx]] = key[idx].reshape(-1, Hk * D)
        vf[slots[idx]] = value[idx].reshape(-1, Hk * D)


def paged_decode_ref(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     block_tables: torch.Tensor, context_lens: torch.Tensor,
                     scale: float) -> torch.Tensor:
    """fp32 restatement of flash_attn_with_kvcache(q.unsqueeze(1), k_cache,
    v_cache, cache_seqlens, block_table, softmax_scale, causal=True) for one
    query token (nanokvllm/layers/attention.py:104-107).

    q [B, Hq, D] -> out [B, Hq, D] fp32. Keys t < context_lens[b] are found at
    block_tables[b, t // block_size]; query head h reads kv head h // g
    (GQA). With seqlen_q == 1, `causal` admits every key. A zero context
    length yields zeros.
    """
    B, Hq, D = q.shape
    _, bs, Hk, _ = k_cache.shape
    g = Hq // Hk
    out = torch.zeros(B, Hq, D, dtype=torch.float32)
    for b in range(B):
        L = int(context_lens[b])
        if L <= 0:
            continue
        nb = (L + bs - 1) // bs
        ids = block_tables[b, :nb].long()
        K = k_cache[ids].reshape(-1, Hk, D)[:L].float()
        V = v_cache[ids].reshape(-1, Hk, D)[:L].float()
        qq = q[b].float().view(Hk, g, D)
        s = torch.einsum("hgd,lhd->hgl", qq, K) * scale
        p = torch.softmax(s, dim=-1)
        out[b] = torch.einsum("hgl,lhd->hgd", p, V).reshape(Hq, D)
    return out
