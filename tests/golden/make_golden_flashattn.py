"""Records the reference's decode kernel -- flash_attn_with_kvcache, called
exactly as nanokvllm/layers/attention.py:104-107 calls it -- on seeded inputs,
so the CPU decode oracle (oracle/attention.py) can be pinned against it.
Needs a CUDA GPU on which flash-attn runs (recorded on a B200 with
flash-attn 2.8.3). Usage:

    python tests/golden/make_golden_flashattn.py OUT.npz

Inputs are regenerated from seeds by oracle.inputs.make_paged_batch; the
file stores their digests and the bf16 outputs (as int16 bits).
"""

import sys
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))

from oracle.inputs import CONFIG1, digest, make_paged_batch  # noqa: E402

DECODE_CASES = [
    ("config1", CONFIG1),
    ("gqa4_ragged", dict(seed=31, lens=[1, 129, 700, 2500, 4096], Hq=32, Hk=8, D=128, block_size=256)),
    ("g8_long", dict(seed=32, lens=[9000], Hq=64, Hk=8, D=128, block_size=256)),
    ("mha_zero_len", dict(seed=33, lens=[0, 300, 1000], Hq=8, Hk=8, D=128, block_size=256)),
]


def main():
    from flash_attn import flash_attn_with_kvcache

    out_path = Path(sys.argv[1])
    res = {}
    for name, kw in DECODE_CASES:
        pb = make_paged_batch(**kw)
        dev = "cuda"
        o = flash_attn_with_kvcache(pb.q.to(dev).unsqueeze(1), pb.k_cache.to(dev), pb.v_cache.to(dev),
                                    cache_seqlens=pb.context_lens.to(dev),
                                    block_table=pb.block_tables.to(dev),
                                    softmax_scale=kw["D"] ** -0.5, causal=True)
        torch.cuda.synchronize()
        res[f"{name}/out_bits"] = o[:, 0].cpu().view(torch.int16).numpy()
        res[f"{name}/q_digest"] = np.array(digest(pb.q))
        res[f"{name}/k_digest"] = np.array(digest(pb.k_cache))
    res["flash_attn_version"] = np.array(__import__("flash_attn").__version__)
    res["device"] = np.array(torch.cuda.get_device_name(0))
    np.savez_compressed(out_path, **res)
    print("wrote", out_path, list(res))


if __name__ == "__main__":
    main()
