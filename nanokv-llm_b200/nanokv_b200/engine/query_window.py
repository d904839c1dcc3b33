"""KvChat's query window on the device.

Same methods and semantics as the reference's QueryWindowManager
(KvChat/engine/query_window_manager.py:20-81) -- has / activate / append /
gather / free, write_pos advancing after the last layer's append -- but the
windows of all sequences live in ONE preallocated device ring
[max_slots, num_layers, W, Hq, D] and appends are a single kernel launch per
layer (nkv_query_window_append) with device index tensors. Nothing is
allocated after construction, so the appends can be captured in the decode
CUDA graph (in the reference they run as Python in forward and are skipped by
graph replays).
"""

from __future__ import annotations

import torch

from .. import ops


class QueryWindowManager:
    def __init__(self, num_layers, window_size, num_heads, head_dim, device="cuda",
                 dtype=torch.bfloat16, max_slots: int = 64):
        self.num_layers = num_layers
        self.window_size = window_size
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.device = torch.device(device)
        self.dtype = dtype
        self.ring = torch.zeros(max_slots, num_layers, window_size, num_heads, head_dim,
                                dtype=dtype, device=self.device)
        self.free_slots = list(range(max_slots - 1, -1, -1))
        # seq_id -> [slot, write_pos, valid_len]
        self.buffers: dict[int, list[int]] = {}

    def has(self, seq_id: int) -> bool:
        return seq_id in self.buffers

    def activate(self, seq_id: int) -> None:
        if seq_id not in self.buffers:
            if not self.free_slots:
                raise RuntimeError("query window ring is full; raise max_slots")
            self.buffers[seq_id] = [self.free_slots.pop(), 0, 0]
        else:
            self.buffers[seq_id][1] = 0
            self.buffers[seq_id][2] = 0

    def slot_of(self, seq_id: int) -> int:
        return self.buffers[seq_id][0]

    def step_indices(self, seq_ids: list[int], batch_index: list[int] | None = None):
        """Device tensors (batch rows, ring slots, write positions) for this
        step's appends; build once per step and reuse for every layer."""
        if batch_index is None:
            batch_index = list(range(len(seq_ids)))
        slots = [self.buffers[s][0] for s in seq_ids]
        pos = [self.buffers[s][1] for s in seq_ids]
        t = torch.tensor([batch_index, slots, pos], dtype=torch.int32).to(self.device, non_blocking=True)
        return t[0], t[1], t[2]

    def row_indices(self, seq_ids: list[int], batch_index: list[int], batch: int):
        """Per batch row (ring slot or -1, write position) as device tensors,
        for the fused decode step that appends inside the decode launch."""
        slot = [-1] * batch
        pos = [0] * batch
        for sid, b in zip(seq_ids, batch_index):
            slot[b], pos[b] = self.buffers[sid][0], self.buffers[sid][1]
        t = torch.tensor([slot, pos], dtype=torch.int32).to(self.device, non_blocking=True)
        return t[0], t[1]

    def advance(self, seq_ids: list[int], layer_id: int) -> None:
        """Bookkeeping of an append done elsewhere (the fused decode step):
        write positions move on after the last layer, as in append()."""
        if layer_id == self.num_layers - 1:
            for s in seq_ids:
                buf = self.buffers[s]
                buf[1] = (buf[1] + 1) % self.window_size
                if buf[2] < self.window_size:
                    buf[2] += 1

    def append(self, seq_ids: list[int], layer_id: int, q: torch.Tensor,
               indices=None) -> None:
        """ring[slot(seq), layer_id, write_pos(seq)] = q[row]. `q` holds one
        row per entry of seq_ids (as in the reference) unless `indices`
        (from step_indices) maps seq_ids to rows of a full batch q."""
        if not seq_ids:
            return
        if indices is None:
            indices = self.step_indices(seq_ids)
        bidx, slots, pos = indices
        ops.query_window_append(q, self.ring, layer_id, bidx, slots, pos)
        self.advance(seq_ids, layer_id)

    def gather(self, seq_ids: list[int], layer_id: int) -> torch.Tensor:
        """[m, Hq, W, D] in the reference's order (window starting at write_pos)."""
        out = []
        for s in seq_ids:
            slot, pos, _ = self.buffers[s]
            lb = self.ring[slot, layer_id]
            out.append(lb if pos == 0 else torch.cat([lb[pos:], lb[:pos]], dim=0))
        return torch.stack(out, 0).permute(0, 2, 1, 3).contiguous()

    def free(self, seq_id: int) -> None:
        buf = self.buffers.pop(seq_id, None)
        if buf is not None:
            self.free_slots.append(buf[0])
