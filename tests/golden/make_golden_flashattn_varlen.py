"""Records the reference's prefill / mixed-batch kernel -- flash_attn_varlen_func,
called exactly as nanokvllm/layers/attention.py:96-102 calls it (causal,
block_table = the paged cache's tables when keys are cached, None otherwise)
-- on the seeded cases of oracle.cases.VARLEN_CASES, so the CPU oracle
(oracle/attention.py: varlen_attention_ref) can be pinned against it.
Needs a CUDA GPU on which flash-attn runs (recorded on a B200 with
flash-attn 2.8.3). Usage:

    python tests/golden/make_golden_flashattn_varlen.py OUT.npz

The file stores the inputs' digests and the bf16 outputs (as int16 bits) of
the rows golden_rows() picks.
"""

import sys
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))

from oracle.cases import VARLEN_CASES  # noqa: E402
from oracle.inputs import digest, make_varlen_batch  # noqa: E402


def golden_rows(cu_q: list[int]) -> np.ndarray:
    """The query rows kept in the file (to keep it small): every 8th row plus
    the first and last row of every sequence."""
    rows = set(range(0, cu_q[-1], 8))
    for a, b in zip(cu_q[:-1], cu_q[1:]):
        if b > a:
            rows.update((a, b - 1))
    return np.array(sorted(rows), dtype=np.int64)


def main():
    from flash_attn import flash_attn_varlen_func

    out_path = Path(sys.argv[1])
    res = {}
    dev = "cuda"
    for name, kw in VARLEN_CASES:
        vb = make_varlen_batch(**kw)
        paged = vb.block_tables is not None
        k = vb.k_cache if paged else vb.k_new
        v = vb.v_cache if paged else vb.v_new
        o = flash_attn_varlen_func(vb.q.to(dev), k.to(dev), v.to(dev),
                                   max_seqlen_q=vb.max_seqlen_q,
                                   cu_seqlens_q=vb.cu_seqlens_q.to(dev),
                                   max_seqlen_k=vb.max_seqlen_k,
                                   cu_seqlens_k=vb.cu_seqlens_k.to(dev),
                                   softmax_scale=kw.get("D", 128) ** -0.5, causal=True,
                                   block_table=vb.block_tables.to(dev) if paged else None)
        torch.cuda.synchronize()
        rows = golden_rows(vb.cu_seqlens_q.tolist())
        res[f"{name}/rows"] = rows
        res[f"{name}/out_bits"] = o.cpu().view(torch.int16).numpy()[rows]
        res[f"{name}/q_digest"] = np.array(digest(vb.q))
        res[f"{name}/k_digest"] = np.array(digest(k))
    res["flash_attn_version"] = np.array(__import__("flash_attn").__version__)
    res["device"] = np.array(torch.cuda.get_device_name(0))
    np.savez_compressed(out_path, **res)
    print("wrote", out_path, list(res))


if __name__ == "__main__":
    main()
