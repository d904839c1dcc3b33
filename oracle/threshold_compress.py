"""CPU restatement of KvChat's threshold compression and query window.
Test infrastructure only (see oracle/__init__.py).

  * QueryWindowRef mirrors QueryWindowManager (KvChat/engine/query_window_manager.py:20-81).
  * threshold_compress_ref mirrors MyCompressCompact
    (KvChat/layers/compress_utils.py:10-171) with TritonGetKVForComp
    (:218-252) restated as a torch gather of positions [0, S).
"""

from __future__ import annotations

import torch

from .snapkv import snapkv_keep


class QueryWindowRef:
    """Per-sequence ring [num_layers, W, Hq, D]; append writes at write_pos for
    every layer and advances write_pos after the last layer; gather returns
    the window starting at write_pos (query_window_manager.py:46-77)."""

    def __init__(self, num_layers: int, window: int, num_heads: int, head_dim: int,
                 dtype=torch.bfloat16):
        self.num_layers, self.window = num_layers, window
        self.num_heads, self.head_dim, self.dtype = num_heads, head_dim, dtype
        self.buffers: dict[int, dict] = {}

    def has(self, seq_id: int) -> bool:
        return seq_id in self.buffers

    def activate(self, seq_id: int) -> None:
        if seq_id not in self.buffers:
            self.buffers[seq_id] = {
                "data": torch.zeros(self.num_layers, self.window, self.num_heads, self.head_dim,
                                    dtype=self.dtype),
                "write_pos": 0, "valid_len": 0,
            }
        else:
            self.buffers[seq_id].update(write_pos=0, valid_len=0)

    def append(self, seq_ids: list[int], layer_id: int, q: torch.Tensor) -> None:
        for i, sid in enumerate(seq_ids):
            buf = self.buffers[sid]
            buf["data"][layer_id, buf["write_pos"]].copy_(q[i])
        if layer_id == self.num_layers - 1:
            for sid in seq_ids:
                buf = self.buffers[sid]
                buf["write_pos"] = (buf["write_pos"] + 1) % self.window
                buf["valid_len"] = min(buf["valid_len"] + 1, self.window)

    def gather(self, seq_ids: list[int], layer_id: int) -> torch.Tensor:
        out = []
        for sid in seq_ids:
            buf = self.buffers[sid]
            pos = buf["write_pos"]
            lb = buf["data"][layer_id]
            out.append(lb if pos == 0 else torch.cat([lb[pos:], lb[:pos]], dim=0))
        return torch.stack(out, 0).permute(0, 2, 1, 3).contiguous()

    def free(self, seq_id: int) -> None:
        self.buffers.pop(seq_id, None)


def gather_first_positions(k_cache: torch.Tensor, v_cache: torch.Tensor, block_tables: torch.Tensor,
                           seq_idxs: list[int], S: int):
    """TritonGetKVForComp (compress_utils.py:174-252): K/V of positions
    [0, S) of each selected sequence, [m, Hk, S, D]; unmapped positions read 0."""
    _, bs, Hk, D = k_cache.shape
    kf = k_cache.view(-1, Hk, D)
    vf = v_cache.view(-1, Hk, D)
    pos = torch.arange(S)
    ks, vs = [], []
    for b in seq_idxs:
        bi = pos // bs
        ids = torch.where(bi < block_tables.size(1), block_tables[b].long()[bi.clamp(max=block_tables.size(1) - 1)],
                          torch.full_like(bi, -1))
        slot = ids * bs + pos % bs
        valid = ids >= 0
        kk = torch.zeros(S, Hk, D, dtype=k_cache.dtype)
        vv = torch.zeros(S, Hk, D, dtype=v_cache.dtype)
        kk[valid] = kf[slot[valid]]
        vv[valid] = vf[slot[valid]]
        ks.append(kk)
        vs.append(vv)
    return (torch.stack(ks).permute(0, 2, 1, 3).contiguous(),
            torch.stack(vs).permute(0, 2, 1, 3).contiguous())


def threshold_compress_ref(q_sub: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                           block_tables: torch.Tensor, context_lens: torch.Tensor,
                           seq_idxs: list[int], S: int, R: int, window: int,
                           keep_idx_override: torch.Tensor | None = None):
    """One layer of KvChat MyCompressCompact, in place on CPU tensors.

    q_sub: [m, Hq, W, D] gathered window queries. Returns keep_idx [m, R]
    (relative to the source window) or False.
    """
    if not seq_idxs:
        return False
    num_blocks, bs, Hk, D = k_cache.shape
    k_sub, _ = gather_first_positions(k_cache, v_cache, block_tables, seq_idxs, S)
    if keep_idx_override is None:
        keep_idx, _ = snapkv_keep(q_sub, k_sub, num_keep=R - window - 1, window=window)
        if keep_idx is False:
            return False
    else:
        keep_idx = keep_idx_override.long()
    max_blocks = block_tables.size(1)
    slots_flat = (block_tables.long().unsqueeze(-1) * bs + torch.arange(bs)).reshape(
        block_tables.size(0), max_blocks * bs)
    start = (context_lens.long() - S).clamp(min=0)
    idx = start.unsqueeze(1) + torch.arange(S)
    src_sub = torch.gather(slots_flat, 1, idx)[seq_idxs]
    src = torch.gather(src_sub, 1, keep_idx).reshape(-1)
    keep_blocks = (R + bs - 1) // bs
    dest_blocks = block_tables[seq_idxs, :keep_blocks].long()
    dst = (dest_blocks.unsqueeze(-1) * bs + torch.arange(bs).view(1, 1, -1)).reshape(
        len(seq_idxs), keep_blocks * bs)[:, :R].reshape(-1)
    kflat = k_cache.view(-1, Hk * D)
    vflat = v_cache.view(-1, Hk * D)
    vals_k = kflat.index_select(0, src).clone()
    vals_v = vflat.index_select(0, src).clone()
    kflat.index_copy_(0, dst, vals_k)
    vflat.index_copy_(0, dst, vals_v)
    context_lens[seq_idxs] = R
    return keep_idx
