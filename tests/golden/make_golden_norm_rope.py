"""Records the reference's own q/k RMSNorm and rotary-embedding modules
(nanokvllm/layers/layernorm.py RMSNorm, nanokvllm/layers/rotary_embedding.py
RotaryEmbedding, as nanokvllm/models/qwen3.py:109-113 applies them) on the
seeded cases of oracle.cases.NORM_ROPE_CASES, run eagerly on the CPU (the
modules' torch.compile is disabled through TORCHDYNAMO_DISABLE), so the
oracle (oracle/norm_rope.py) is pinned to them. Usage:

    python tests/golden/make_golden_norm_rope.py [REFERENCE_ROOT]

Writes tests/golden/norm_rope.npz: input digests, the module's cos/sin
cache digest and the bf16 outputs (as int16 bits).
"""

import os
import sys
from pathlib import Path

os.environ["TORCHDYNAMO_DISABLE"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))

from oracle.cases import NORM_ROPE_CASES, norm_rope_inputs  # noqa: E402
from oracle.inputs import digest  # noqa: E402


def main():
    arg = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("NANOKV_REFERENCE")
    if not arg:
        raise SystemExit(f"usage: python {Path(__file__).name} /path/to/nanokv-llm checkout "
                         "(or set NANOKV_REFERENCE)")
    ref = Path(arg).resolve()
    sys.path.insert(0, str(ref))
    from nanokvllm.layers.layernorm import RMSNorm
    from nanokvllm.layers.rotary_embedding import RotaryEmbedding

    out = {}
    for name, seed, T, Hq, Hk, max_pos, base, eps in NORM_ROPE_CASES:
        qkv, pos, qw, kw, _ = norm_rope_inputs(seed, T, Hq, Hk, max_pos)
        q, k, _ = qkv.split([Hq * 128, Hk * 128, Hk * 128], dim=-1)
        qn, kn = RMSNorm(128, eps=eps), RMSNorm(128, eps=eps)
        with torch.no_grad():
            qn.weight = torch.nn.Parameter(qw.clone())
            kn.weight = torch.nn.Parameter(kw.clone())
            rope = RotaryEmbedding(128, 128, max_pos, base)
            qo = qn(q.reshape(T, Hq, 128).contiguous())
            ko = kn(k.reshape(T, Hk, 128).contiguous())
            qo, ko = rope(pos, qo, ko)
        out[f"{name}/q_bits"] = qo.view(torch.int16).numpy()
        out[f"{name}/k_bits"] = ko.view(torch.int16).numpy()
        out[f"{name}/qkv_digest"] = np.array(digest(qkv))
        out[f"{name}/cos_sin_digest"] = np.array(
            digest(rope.cos_sin_cache.reshape(max_pos, 128).contiguous().view(torch.int32)))
    np.savez_compressed(REPO / "tests" / "golden" / "norm_rope.npz", **out)
    print("norm_rope.npz:", len(NORM_ROPE_CASES), "cases")


if __name__ == "__main__":
    main()
