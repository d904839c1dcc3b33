"""Seeded synthetic inputs for the parity tests and golden vectors.

Test infrastructure only. Values come from numpy's PCG64 generator (its
normal and integer streams are platform-independent), converted to bf16 with
round-to-nearest-even, so the same seed gives the same bytes on every host.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass

import numpy as np
import torch


def bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16)


def digest(t: torch.Tensor) -> str:
    """sha256 of a tensor's raw bytes (bf16 viewed as int16)."""
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.contiguous().cpu().numpy().tobytes()).hexdigest()


@dataclass
class PagedBatch:
    q: torch.Tensor            # [B, Hq, D] bf16
    k_new: torch.Tensor        # [B, Hk, D] bf16 (the current token's K)
    v_new: torch.Tensor        # [B, Hk, D]
    k_cache: torch.Tensor      # [num_blocks, block_size, Hk, D] bf16
    v_cache: torch.Tensor
    block_tables: torch.Tensor  # [B, max_blocks] int32, -1 padded
    context_lens: torch.Tensor  # [B] int32 (includes the current token)
    slot_mapping: torch.Tensor  # [B] int32: slot of the current token
    block_size: int


def make_paged_batch(seed: int, lens: list[int], Hq: int, Hk: int, D: int = 128,
                     block_size: int = 256, num_blocks: int | None = None,
                     outlier_sigma: float = 0.0, outlier_frac: float = 0.0) -> PagedBatch:
    """Random paged KV state: N(0,1) q/k/v and cache, a random permutation
    of the block pool handed out sequence by sequence (non-contiguous tables).
    Optional per-head outlier channels: a fixed `outlier_frac` of each kv
    head's dims scaled by `outlier_sigma`."""
    rng = np.random.default_rng(seed)
    need = sum((L + block_size - 1) // block_size for L in lens)
    if num_blocks is None:
        num_blocks = need
    assert num_blocks >= need
    kc = rng.standard_normal((num_blocks, block_size, Hk, D), dtype=np.float32)
    vc = rng.standard_normal((num_blocks, block_size, Hk, D), dtype=np.float32)
    if outlier_sigma > 0 and outlier_frac > 0:
        nd = max(1, int(round(outlier_frac * D)))
        for h in range(Hk):
            dims = rng.choice(D, size=nd, replace=False)
            kc[:, :, h, dims] *= outlier_sigma
            vc[:, :, h, dims] *= outlier_sigma
    perm = rng.permutation(num_blocks)
    tables, o = [], 0
    for L in lens:
        n = (L + block_size - 1) // block_size
        tables.append([int(x) for x in perm[o:o + n]])
        o += n
    mx = max(1, max(len(t) for t in tables))
    bt = torch.tensor([t + [-1] * (mx - len(t)) for t in tables], dtype=torch.int32)
    q = rng.standard_normal((len(lens), Hq, D), dtype=np.float32)
    kn = rng.standard_normal((len(lens), Hk, D), dtype=np.float32)
    vn = rng.standard_normal((len(lens), Hk, D), dtype=np.float32)
    slots = []
    for L, t in zip(lens, tables):
        if L <= 0:
            slots.append(-1)
        else:
            pos = L - 1
            slots.append(t[pos // block_size] * block_size + pos % block_size)
    return PagedBatch(
        q=bf16(q), k_new=bf16(kn), v_new=bf16(vn), k_cache=bf16(kc), v_cache=bf16(vc),
        block_tables=bt, context_lens=torch.tensor(lens, dtype=torch.int32),
        slot_mapping=torch.tensor(slots, dtype=torch.int32), block_size=block_size)


# Qwen3-0.6B-shaped single layer, B=4, 64-block pool,
# lens {300, 700, 1024, 1500} (including the current token), compression on seq 3.
CONFIG1 = dict(seed=0, lens=[300, 700, 1024, 1500], Hq=16, Hk=8, D=128, block_size=256,
               num_blocks=64)
CONFIG1_COMPRESS = dict(selected=[3], window_blocks=4, keep_blocks=2, keep_extra_tokens=1)


def make_config1() -> PagedBatch:
    return make_paged_batch(**CONFIG1)


@dataclass
class VarlenBatch:
    q: torch.Tensor             # [T, Hq, D] bf16: the step's query rows
    k_new: torch.Tensor         # [T, Hk, D] bf16: the step's key rows
    v_new: torch.Tensor
    k_cache: torch.Tensor | None  # [num_blocks, block_size, Hk, D] (paged) or None
    v_cache: torch.Tensor | None
    block_tables: torch.Tensor | None  # [B, max_blocks] int32, -1 padded
    slot_mapping: torch.Tensor  # [T] int32: cache slot of each step row (paged)
    cu_seqlens_q: torch.Tensor  # [B + 1] int32
    cu_seqlens_k: torch.Tensor  # [B + 1] int32
    max_seqlen_q: int
    max_seqlen_k: int


def make_varlen_batch(seed: int, q_lens: list[int], k_lens: list[int], Hq: int, Hk: int,
                      D: int = 128, block_size: int = 256, paged: bool = True) -> VarlenBatch:
    """A prefill / mixed batch as the reference's prepare_step builds it
    (nanokvllm/engine/model_runner.py:160-220): sequence b advances q_lens[b]
    tokens and then holds k_lens[b] >= q_lens[b] tokens, so its step rows are
    positions k_lens[b] - q_lens[b] .. k_lens[b] - 1. Paged: the cache holds
    every sequence's k_lens[b] tokens in randomly permuted blocks, the step's
    rows included (as after store_kvcache). Unpaged (no cached prefix,
    k_lens == q_lens): keys are the step's rows themselves."""
    rng = np.random.default_rng(seed)
    assert len(q_lens) == len(k_lens)
    T = sum(q_lens)
    cu_q = np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32)
    cu_k = np.concatenate([[0], np.cumsum(k_lens)]).astype(np.int32)
    q = bf16(rng.standard_normal((T, Hq, D), dtype=np.float32))
    if not paged:
        assert list(q_lens) == list(k_lens)
        kn = bf16(rng.standard_normal((T, Hk, D), dtype=np.float32))
        vn = bf16(rng.standard_normal((T, Hk, D), dtype=np.float32))
        return VarlenBatch(q=q, k_new=kn, v_new=vn, k_cache=None, v_cache=None,
                           block_tables=None, slot_mapping=torch.full((T,), -1, dtype=torch.int32),
                           cu_seqlens_q=torch.from_numpy(cu_q), cu_seqlens_k=torch.from_numpy(cu_k),
                           max_seqlen_q=max(q_lens, default=0), max_seqlen_k=max(k_lens, default=0))
    pb = make_paged_batch(seed + 1000, list(k_lens), Hq, Hk, D, block_size)
    slots = []
    for b, (lq, lk) in enumerate(zip(q_lens, k_lens)):
        assert lk >= lq
        t = pb.block_tables[b].tolist()
        for pos in range(lk - lq, lk):
            slots.append(t[pos // block_size] * block_size + pos % block_size)
    sm = torch.tensor(slots, dtype=torch.int32)
    flat_k = pb.k_cache.view(-1, Hk, D)
    flat_v = pb.v_cache.view(-1, Hk, D)
    kn = flat_k[sm.long()].clone() if T else torch.zeros(0, Hk, D, dtype=torch.bfloat16)
    vn = flat_v[sm.long()].clone() if T else torch.zeros(0, Hk, D, dtype=torch.bfloat16)
    return VarlenBatch(q=q, k_new=kn, v_new=vn, k_cache=pb.k_cache, v_cache=pb.v_cache,
                       block_tables=pb.block_tables, slot_mapping=sm,
                       cu_seqlens_q=torch.from_numpy(cu_q), cu_seqlens_k=torch.from_numpy(cu_k),
                       max_seqlen_q=max(q_lens, default=0), max_seqlen_k=max(k_lens, default=0))
