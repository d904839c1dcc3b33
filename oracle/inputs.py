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
