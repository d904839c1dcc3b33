"""CPU restatement of SnapKV (nanokvllm/layers/CompressMethod.py:4-58; the
KvChat copy at KvChat/layers/CompressMethod.py:4-58 is identical).

Test infrastructure only (see oracle/__init__.py).

The importance is computed with the same torch operations, dtypes and
rounding points as the reference (bf16 matmul, bf16 scale multiply, sink
mask, bf16 softmax, bf16 sum over the window, bf16 sum over the heads), so on
the CPU it is bit-identical to the reference's. The reference then calls
torch.topk(sorted=False), whose order among exactly tied values is
unspecified; `topk_low_index` is the deterministic refinement libnkv
implements: the k largest values, ties at the cut broken towards the lower
index.
"""

from __future__ import annotations

import torch


def snapkv_importance(Q: torch.Tensor, K: torch.Tensor, window: int,
                      exact_scores: bool = False) -> torch.Tensor:
    """key_importance [B, L - window] (bf16) exactly as CompressMethod.py:19-42.

    Q: [B, Hq, window, D]; K: [B, Hk, L, D] (bf16).

    exact_scores: the bf16 q.k products are rounded once from their exact
    value (an fp64 product rounded to fp32, then to bf16) instead of from
    torch's CPU bf16 matmul, whose fp32 accumulation order is the CPU
    library's and can land on the other side of a bf16 rounding boundary
    (38 of the 654,720 scores of a 20-sequence Qwen3-8B event, changing one
    importance value by one bf16 ulp). Every later step is the
    reference's. This is the platform-independent definition libnkv's
    window kernel implements; with exact_scores=False the function is the
    reference's own computation on this CPU.
    """
    B, Hk, L, D = K.shape
    Hq = Q.size(1)
    K_cut = K[:, :, :-window, :]
    scale = 1.0 / (D ** 0.5)

    def mm(a, b):
        if exact_scores:
            return torch.matmul(a.double(), b.double()).float().to(torch.bfloat16)
        return torch.matmul(a, b)

    if Hq == Hk:
        scores = mm(Q, K_cut.transpose(-1, -2)) * scale
    else:
        g = Hq // Hk
        Qg = Q.view(B, Hk, g, window, D)
        Kt = K_cut.transpose(-1, -2).unsqueeze(2)
        scores = (mm(Qg, Kt) * scale).view(B, Hq, window, L - window)
    scores[:, :, :, 0] = -float("inf")
    probs = torch.softmax(scores, dim=-1)
    imp = probs.sum(dim=2)
    if imp.size(1) > 1:
        imp = imp.sum(dim=1, keepdim=True)
    return imp.view(B, L - window)


def topk_low_index(values: torch.Tensor, k: int) -> torch.Tensor:
    """Indices of the k largest entries of each row of `values` [B, n],
    ascending; among equal values the lower index wins."""
    B, n = values.shape
    v = values.float()
    # a stable sort of -value keeps equal values in index order
    order = torch.sort(-v, dim=-1, stable=True).indices
    kept = order[:, :k]
    return torch.sort(kept, dim=-1).values


def snapkv_keep(Q: torch.Tensor, K: torch.Tensor, num_keep: int, window: int,
                exact_scores: bool = False):
    """final_idx [B, 1 + num_keep + window] = cat(0, kept ascending, last
    `window` positions), or False when the reference skips
    (CompressMethod.py:17-18). Also returns the importance."""
    B, Hk, L, D = K.shape
    if L - window <= 0 or L <= num_keep + window:
        return False, None
    imp = snapkv_importance(Q, K, window, exact_scores)
    kept = topk_low_index(imp, num_keep)
    tail = torch.arange(L - window, L).unsqueeze(0).expand(B, -1)
    bos = torch.zeros((B, 1), dtype=torch.long)
    return torch.cat([bos, kept, tail], dim=-1), imp


def tie_band_ok(imp: torch.Tensor, kept_a: torch.Tensor, kept_b: torch.Tensor, k: int,
                band: float = 0.0) -> tuple[bool, str]:
    """True if two kept sets of size k (indices into imp) can both be a valid
    top-k of `imp` up to `band`: every index only one of them keeps must lie
    within `band` of the k-th largest value. band=0 allows swaps inside the
    exact-tie group at the cut only."""
    a, b = set(kept_a.tolist()), set(kept_b.tolist())
    if len(a) != k or len(b) != k:
        return False, f"sizes {len(a)} {len(b)} != {k}"
    v = imp.float()
    cut = torch.sort(v, descending=True).values[k - 1].item()
    for t in a ^ b:
        if abs(v[t].item() - cut) > band:
            return False, f"index {t} value {v[t].item()} vs cut {cut} band {band}"
    return True, ""
