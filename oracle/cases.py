"""Parameter tables of the golden cases, shared by tests/golden/make_golden.py
(which runs the reference on them) and the parity tests. Test infrastructure only.
"""

from __future__ import annotations

import numpy as np
import torch

from .inputs import CONFIG1, CONFIG1_COMPRESS, bf16, make_paged_batch

SNAPKV_CASES = [
    # name, seed, m, Hq, Hk, L, window, num_keep, outlier
    ("cfg1_g2", 101, 2, 16, 8, 1024, 1, 511, 0.0),
    ("qwen8b_g4", 102, 2, 32, 8, 1024, 1, 511, 0.0),
    ("qwen8b_g4_outlier", 103, 2, 32, 8, 1024, 1, 511, 4.0),
    ("qwen32b_g8", 104, 1, 64, 8, 1024, 1, 511, 0.0),
    ("mha", 105, 1, 8, 8, 1024, 1, 511, 0.0),
    ("tp8_g4", 106, 3, 4, 1, 1024, 1, 511, 0.0),
    ("kvchat_w50", 107, 1, 16, 8, 767, 50, 462, 0.0),
]


def snapkv_inputs(seed, m, Hq, Hk, L, window, outlier):
    rng = np.random.default_rng(seed)
    Q = rng.standard_normal((m, Hq, window, 128), dtype=np.float32)
    K = rng.standard_normal((m, Hk, L, 128), dtype=np.float32)
    if outlier:
        for h in range(Hk):
            dims = rng.choice(128, size=6, replace=False)
            K[:, h, :, dims] *= outlier
    return bf16(Q), bf16(K)


WINDOW_CASES = [
    # name, paged batch kwargs, selected, window_blocks, keep_blocks, keep_extra
    ("config1", CONFIG1, CONFIG1_COMPRESS["selected"], 4, 2, 1),
    ("gqa4_multi", dict(seed=7, lens=[1300, 2100, 1050, 1800, 999, 1024], Hq=32, Hk=8, D=128,
                        block_size=256, num_blocks=48), [0, 1, 3, 5], 4, 2, 1),
    ("outlier_g4", dict(seed=8, lens=[2304, 1500], Hq=32, Hk=8, D=128, block_size=256,
                        num_blocks=20, outlier_sigma=4.0, outlier_frac=0.05), [0, 1], 4, 2, 1),
]


THRESHOLD_CASES = [
    # name, seed, prompt, Hq, Hk, W, S_cfg, R_cfg, num_layers, compress layer
    ("cfg5_p256", 21, 256, 16, 8, 50, 511, 257, 1, 0),
    ("cfg5_p100_rotated", 22, 100, 16, 8, 50, 511, 257, 2, 0),
]


def threshold_inputs(seed: int, P: int, Hq: int, Hk: int, W: int, S_cfg: int, L: int):
    """Paged batch of one sequence at length S = P + S_cfg plus W steps of
    per-layer queries [W, L, 1, Hq, 128]."""
    S = P + S_cfg
    pb = make_paged_batch(seed=seed, lens=[S], Hq=Hq, Hk=Hk, D=128, block_size=256)
    rng = np.random.default_rng(seed + 1000)
    qsteps = bf16(rng.standard_normal((W, L, 1, Hq, 128), dtype=np.float32))
    return pb, qsteps


# Prefill / mixed-batch attention (flash_attn_varlen_func at
# nanokvllm/layers/attention.py:96-102): (name, make_varlen_batch kwargs).
# Covers prefill without a cached prefix (contiguous K/V), prefix-cached
# prefill, chunked-prefill mixed batches with decode rows (Lq = 1), GQA
# widths 1/2/3/4/8, empty sequences and queries longer than their keys.
VARLEN_CASES = [
    ("prefill_nocache_g2", dict(seed=41, q_lens=[1, 77, 300, 1024], k_lens=[1, 77, 300, 1024],
                                Hq=16, Hk=8, paged=False)),
    ("prefix_paged_g4", dict(seed=42, q_lens=[200, 64, 513], k_lens=[456, 1000, 769],
                             Hq=32, Hk=8)),
    ("mixed_chunked_g4", dict(seed=43, q_lens=[1, 1, 300, 1, 130], k_lens=[700, 1, 2300, 4097, 130],
                              Hq=32, Hk=8)),
    ("g8_paged", dict(seed=44, q_lens=[129, 3], k_lens=[129, 2000], Hq=64, Hk=8)),
    ("mha_empty_rows", dict(seed=45, q_lens=[0, 5, 17, 0], k_lens=[0, 5, 17, 40], Hq=8, Hk=8)),
    ("g3_nocache", dict(seed=46, q_lens=[50, 400], k_lens=[50, 400], Hq=24, Hk=8, paged=False)),
]


# q/k RMSNorm + RoPE + slot write (qwen3.py:109-113): (name, seed, tokens,
# Hq, Hk, max_positions, rope base, eps). Qwen3-8B / 32B / 0.6B head shapes.
NORM_ROPE_CASES = [
    ("decode_8b", 61, 64, 32, 8, 16384, 1000000.0, 1e-6),
    ("prefill_32b", 62, 48, 64, 8, 40960, 1000000.0, 1e-6),
    ("small_06b", 63, 7, 16, 8, 2048, 10000.0, 1e-5),
]


def norm_rope_inputs(seed: int, T: int, Hq: int, Hk: int, max_pos: int):
    """Seeded qkv rows ([T, (Hq + 2 Hk) * 128] bf16, N(0, 2^2) with a few
    large channels as real activations have), positions in [0, max_pos),
    norm weights N(1, 0.3^2) in bf16, and slots (every 5th token -1)."""
    rng = np.random.default_rng(seed)
    D = 128
    x = rng.standard_normal((T, (Hq + 2 * Hk) * D), dtype=np.float32) * 2.0
    x[:, rng.choice(x.shape[1], size=x.shape[1] // 64, replace=False)] *= 8.0
    pos = rng.integers(0, max_pos, size=T).astype(np.int64)
    pos[: min(T, 3)] = [0, 1, max_pos - 1][: min(T, 3)]
    qw = rng.normal(1.0, 0.3, size=D).astype(np.float32)
    kw = rng.normal(1.0, 0.3, size=D).astype(np.float32)
    slots = rng.permutation(T * 4)[:T].astype(np.int32)
    slots[::5] = -1
    return (bf16(x), torch.from_numpy(pos), bf16(qw), bf16(kw), torch.from_numpy(slots))
