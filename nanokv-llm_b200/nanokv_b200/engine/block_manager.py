"""Paged-block bookkeeping with compression truncation.

Behaviourally identical to the reference's BlockManager
(nanokvllm/engine/block_manager.py:7-138): blocks are handed out from the
front of a FIFO free list and returned to its back, full blocks are hashed
(xxh64 over the 8-byte little-endian prefix hash and the int64 token ids) for
prefix sharing, and truncate_blocks releases everything past keep_blocks --
the host half of a compression event. Free-list order is part of the
contract: it decides which physical blocks later sequences get, so block
tables stay bit-exact with the reference's.
"""

from __future__ import annotations

from collections import deque

import numpy as np
import xxhash


class Block:
    __slots__ = ("block_id", "ref_count", "hash", "token_ids")

    def __init__(self, block_id: int):
        self.block_id = block_id
        self.ref_count = 0
        self.hash = -1
        self.token_ids: list[int] = []

    def update(self, h: int, token_ids: list[int]) -> None:
        self.hash = h
        self.token_ids = token_ids

    def reset(self) -> None:
        self.ref_count = 1
        self.hash = -1
        self.token_ids = []


class BlockManager:
    def __init__(self, num_blocks: int, block_size: int):
        self.block_size = block_size
        self.blocks = [Block(i) for i in range(num_blocks)]
        self.hash_to_block_id: dict[int, int] = {}
        self.free_block_ids: deque[int] = deque(range(num_blocks))
        self.used_block_ids: set[int] = set()

    @classmethod
    def compute_hash(cls, token_ids: list[int], prefix: int = -1) -> int:
        h = xxhash.xxh64()
        if prefix != -1:
            h.update(prefix.to_bytes(8, "little"))
        h.update(np.asarray(token_ids, dtype=np.int64).tobytes())
        return h.intdigest()

    # -- low level
    def _take(self, block_id: int) -> Block:
        blk = self.blocks[block_id]
        assert blk.ref_count == 0
        blk.reset()
        self.free_block_ids.remove(block_id)
        self.used_block_ids.add(block_id)
        return blk

    def _release(self, block_id: int) -> None:
        assert self.blocks[block_id].ref_count == 0
        self.used_block_ids.remove(block_id)
        self.free_block_ids.append(block_id)

    def _unref(self, block_id: int) -> None:
        blk = self.blocks[block_id]
        blk.ref_count -= 1
        if blk.ref_count == 0:
            self._release(block_id)

    # -- sequences
    def can_allocate(self, seq) -> bool:
        return len(self.free_block_ids) >= seq.num_blocks

    def allocate(self, seq) -> None:
        assert not seq.block_table
        h = -1
        miss = False
        for i in range(seq.num_blocks):
            ids = seq.block(i)
            h = self.compute_hash(ids, h) if len(ids) == self.block_size else -1
            bid = self.hash_to_block_id.get(h, -1)
            if bid == -1 or self.blocks[bid].token_ids != ids:
                miss = True
            if miss:
                blk = self._take(self.free_block_ids[0])
            else:
                seq.num_cached_tokens += self.block_size
                if bid in self.used_block_ids:
                    blk = self.blocks[bid]
                    blk.ref_count += 1
                else:
                    blk = self._take(bid)
            if h != -1:
                blk.update(h, ids)
                self.hash_to_block_id[h] = blk.block_id
            seq.block_table.append(blk.block_id)

    def deallocate(self, seq) -> None:
        for bid in reversed(seq.block_table):
            self._unref(bid)
        seq.num_cached_tokens = 0
        seq.block_table.clear()

    def can_append(self, seq) -> bool:
        return len(self.free_block_ids) >= (len(seq) % self.block_size == 1)

    def may_append(self, seq) -> None:
        table = seq.block_table
        last = self.blocks[table[-1]]
        r = len(seq) % self.block_size
        if r == 1:
            assert last.hash != -1
            blk = self._take(self.free_block_ids[0])
            table.append(blk.block_id)
        elif r == 0:
            assert last.hash == -1
            ids = seq.block(seq.num_blocks - 1)
            prefix = self.blocks[table[-2]].hash if len(table) > 1 else -1
            h = self.compute_hash(ids, prefix)
            last.update(h, ids)
            self.hash_to_block_id[h] = last.block_id
        else:
            assert last.hash == -1

    def truncate_blocks(self, seq, keep_blocks: int) -> None:
        """Releases seq.block_table[keep_blocks:] (last first) after a
        compression; the new last block loses its hash (its content changed)."""
        if keep_blocks >= len(seq.block_table):
            return
        for bid in reversed(seq.block_table[keep_blocks:]):
            self._unref(bid)
        seq.block_table = seq.block_table[:keep_blocks]
        seq.num_cached_tokens = min(seq.num_cached_tokens, keep_blocks * self.block_size)
        if seq.block_table:
            self.blocks[seq.block_table[-1]].hash = -1
