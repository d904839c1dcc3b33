"""CPU restatement of Attention.forward: slot write, paged decode and the
prefill / mixed-batch variable-length attention.

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


def varlen_attention_ref(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                         cu_seqlens_q, cu_seqlens_k, scale: float, causal: bool = True,
                         block_table: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 restatement of flash_attn_varlen_func(q, k, v, cu_seqlens_q,
    cu_seqlens_k, max_seqlen_q, max_seqlen_k, softmax_scale, causal,
    block_table) as called for prefill / mixed batches at
    nanokvllm/layers/attention.py:96-102 (metadata built at
    nanokvllm/engine/model_runner.py:160-220).

    q [T, Hq, D] -> out [T, Hq, D] fp32. Sequence b owns query rows
    cu_seqlens_q[b] .. cu_seqlens_q[b+1] and Lk = cu_seqlens_k[b+1] -
    cu_seqlens_k[b] keys: with block_table, key j is row j % block_size of
    block block_table[b, j // block_size] of the paged cache k [num_blocks,
    block_size, Hk, D]; without, it is row cu_seqlens_k[b] + j of k [Tk, Hk, D].
    causal admits keys j <= Lk - Lq + i for query i (flash-attn >= 2.1's
    bottom-right alignment). Rows that admit no key are zeros.
    """
    T, Hq, D = q.shape
    Hk = k.shape[-2]
    g = Hq // Hk
    cq = [int(x) for x in cu_seqlens_q]
    ck = [int(x) for x in cu_seqlens_k]
    out = torch.zeros(T, Hq, D, dtype=torch.float32)
    for b in range(len(cq) - 1):
        Lq, Lk = cq[b + 1] - cq[b], ck[b + 1] - ck[b]
        if Lq <= 0 or Lk <= 0:
            continue
        if block_table is not None:
            bs = k.shape[1]
            nb = (Lk + bs - 1) // bs
            ids = block_table[b, :nb].long()
            K = k[ids].reshape(-1, Hk, D)[:Lk].float()
            V = v[ids].reshape(-1, Hk, D)[:Lk].float()
        else:
            K = k[ck[b]:ck[b] + Lk].float()
            V = v[ck[b]:ck[b] + Lk].float()
        qq = q[cq[b]:cq[b] + Lq].float().view(Lq, Hk, g, D)
        s = torch.einsum("ihgd,jhd->hgij", qq, K) * scale
        if causal:
            i = torch.arange(Lq).view(Lq, 1)
            j = torch.arange(Lk).view(1, Lk)
            s = s.masked_fill(j > (Lk - Lq) + i, float("-inf"))
        p = torch.softmax(s, dim=-1)
        p = torch.nan_to_num(p, nan=0.0)  # rows without an admissible key
        o = torch.einsum("hgij,jhd->ihgd", p, V)
        out[cq[b]:cq[b] + Lq] = o.reshape(Lq, Hq, D)
    return out
