"""Host-side request state and KV block bookkeeping -- TEST INFRASTRUCTURE
ONLY (see the package header).

The product's host code (nanokv_b200.engine) never owns sequences or blocks:
it reads and updates the caller's objects -- in deployment the reference's
own Sequence (nanokvllm/engine/sequence.py:16-139) and BlockManager
(nanokvllm/engine/block_manager.py:27-138) -- through the attributes and the
one method it needs (num_tokens, block_table, tail_uncompressed_len,
rope_pos, ...; BlockManager.truncate_blocks). The tests need stand-ins for
both that behave exactly like the reference's, so that traces recorded from
the reference (tests/golden/host_metadata.json, step_metadata.json, made by
tests/golden/make_golden.py) can be replayed through the product's event
appliers and metadata builders on a machine without the reference checkout.

SeqState models a request: physical length num_tokens (shrinks when a
compression event is applied), the logical position rope_pos that only
grows, and the count of generated tokens since the last compression.

BlockPool models the block allocator as a small state machine over three
per-block arrays (reference count, chained content hash, content) and a FIFO
free list. The behaviour the traces pin:
  * allocation always takes the head of the free list; a released block goes
    to its tail; a block's reference count starts at 1 when taken;
  * a full block carries xxh64(8-byte little-endian previous hash, if any,
    then the block's token ids as int64); allocate() reuses a block whose
    hash and content match, until the first miss, after which every block is
    fresh;
  * appending token 1 of a block takes a new block; completing a block
    hashes it;
  * releases (deallocate, truncate_blocks) walk the released blocks from the
    last to the first; truncate_blocks clears the hash of the new last block
    (compaction rewrote its content).
"""

from __future__ import annotations

from collections import deque
from dataclasses import dataclass
from itertools import count

import numpy as np


class SeqState:
    """A request's state as the compression path sees it."""

    block_size = 256
    counter = count()

    def __init__(self, token_ids, max_tokens: int = 64, ignore_eos: bool = False):
        self.seq_id = next(SeqState.counter)
        self.token_ids = list(token_ids)
        self.num_prompt_tokens = len(self.token_ids)
        self.num_tokens = self.num_prompt_tokens
        self.num_cached_tokens = 0
        self.num_computed_tokens = 0
        self.block_table: list[int] = []
        self.max_tokens = max_tokens
        self.ignore_eos = ignore_eos
        self.rope_pos = self.num_tokens - 1
        self.tail_uncompressed_len = 0

    def __len__(self) -> int:
        return self.num_tokens

    @property
    def last_token(self) -> int:
        return self.token_ids[-1]

    @property
    def num_blocks(self) -> int:
        return -(-self.num_tokens // self.block_size)

    def block(self, i: int) -> list[int]:
        """Ids i*block_size .. of the token list. The list only grows (ids are
        never dropped by a compression event, only num_tokens shrinks), so
        after an event these are the ids at those list positions, as the
        reference hashes them."""
        assert 0 <= i < self.num_blocks
        return self.token_ids[i * self.block_size:(i + 1) * self.block_size]

    def append_token(self, token_id: int) -> None:
        self.token_ids.append(token_id)
        self.num_tokens += 1
        self.rope_pos += 1
        self.tail_uncompressed_len += 1


@dataclass
class Scheduled:
    """One row of a unified-scheduler step: a request and how many of its
    tokens this step computes."""
    seq: SeqState
    num_new_tokens: int


def chained_hash(token_ids, prev: int) -> int:
    import xxhash
    h = xxhash.xxh64()
    if prev != -1:
        h.update(int(prev).to_bytes(8, "little"))
    h.update(np.asarray(token_ids, dtype=np.int64).tobytes())
    return h.intdigest()


class BlockPool:
    """The block allocator's state machine (see the module header)."""

    def __init__(self, num_blocks: int, block_size: int):
        self.block_size = block_size
        self.ref = [0] * num_blocks
        self.hash = [-1] * num_blocks
        self.content: list[list[int] | None] = [None] * num_blocks
        self.free = deque(range(num_blocks))
        self.used: set[int] = set()
        self.index: dict[int, int] = {}  # hash -> block id

    # -- primitive transitions
    def _take(self, b: int) -> int:
        assert self.ref[b] == 0, f"block {b} is in use"
        self.free.remove(b)
        self.used.add(b)
        self.ref[b], self.hash[b], self.content[b] = 1, -1, None
        return b

    def _release(self, blocks) -> None:
        for b in reversed(list(blocks)):
            self.ref[b] -= 1
            if self.ref[b] == 0:
                self.used.discard(b)
                self.free.append(b)

    def _seal(self, b: int, h: int, tokens: list[int]) -> None:
        self.hash[b], self.content[b] = h, tokens
        self.index[h] = b

    # -- the operations the scheduler performs
    def can_allocate(self, seq) -> bool:
        return len(self.free) >= seq.num_blocks

    def allocate(self, seq) -> None:
        assert not seq.block_table
        prev, missed = -1, False
        for i in range(seq.num_blocks):
            tokens = seq.block(i)
            full = len(tokens) == self.block_size
            h = chained_hash(tokens, prev) if full else -1
            hit = self.index.get(h, -1)
            missed = missed or hit == -1 or self.content[hit] != tokens
            if missed:
                b = self._take(self.free[0])
            else:
                seq.num_cached_tokens += self.block_size
                b = hit
                if b in self.used:
                    self.ref[b] += 1
                else:
                    self._take(b)
            if full:
                self._seal(b, h, tokens)
            seq.block_table.append(b)
            prev = h

    def deallocate(self, seq) -> None:
        self._release(seq.block_table)
        seq.num_cached_tokens = 0
        seq.block_table.clear()

    def can_append(self, seq) -> bool:
        return len(self.free) >= int(len(seq) % self.block_size == 1)

    def may_append(self, seq) -> None:
        """Called once the sequence holds its newest token."""
        table = seq.block_table
        last = table[-1]
        pos = len(seq) % self.block_size
        if pos == 1:  # the token opened a new block
            assert self.hash[last] != -1
            table.append(self._take(self.free[0]))
        elif pos == 0:  # the token completed the last block
            assert self.hash[last] == -1
            prev = self.hash[table[-2]] if len(table) > 1 else -1
            tokens = seq.block(seq.num_blocks - 1)
            self._seal(last, chained_hash(tokens, prev), tokens)
        else:
            assert self.hash[last] == -1

    def truncate_blocks(self, seq, keep_blocks: int) -> None:
        if keep_blocks >= len(seq.block_table):
            return
        self._release(seq.block_table[keep_blocks:])
        seq.block_table = seq.block_table[:keep_blocks]
        seq.num_cached_tokens = min(seq.num_cached_tokens, keep_blocks * self.block_size)
        if seq.block_table:
            self.hash[seq.block_table[-1]] = -1

    def state(self) -> dict:
        """The comparable state: free list order, used set, reference counts
        and which blocks carry a hash."""
        return {"free": list(self.free), "used": sorted(self.used), "ref": list(self.ref),
                "hash_set": [h != -1 for h in self.hash]}
