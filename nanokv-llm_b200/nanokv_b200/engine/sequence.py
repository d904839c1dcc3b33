"""The per-request state the compression path reads and writes.

Field names and length semantics follow the reference's Sequence
(nanokvllm/engine/sequence.py:16-139): num_tokens is the PHYSICAL KV length
(it shrinks when a compression event is applied), rope_pos the logical
position that only grows, tail_uncompressed_len the generated tokens since
the last compression.
"""

from __future__ import annotations

from dataclasses import dataclass
from itertools import count


class Sequence:
    block_size = 256
    counter = count()

    def __init__(self, token_ids: list[int], max_tokens: int = 64, ignore_eos: bool = False,
                 temperature: float = 1.0):
        self.seq_id = next(Sequence.counter)
        self.token_ids = list(token_ids)
        self.last_token = self.token_ids[-1]
        self.num_tokens = len(self.token_ids)
        self.num_prompt_tokens = len(self.token_ids)
        self.num_cached_tokens = 0
        self.num_computed_tokens = 0
        self.block_table: list[int] = []
        self.temperature = temperature
        self.max_tokens = max_tokens
        self.ignore_eos = ignore_eos
        self.generated_completion_tokens = 0
        self.rope_pos = self.num_tokens - 1
        self.tail_uncompressed_len = 0

    def __len__(self) -> int:
        return self.num_tokens

    def __getitem__(self, key):
        return self.token_ids[key]

    @property
    def is_prefill_done(self) -> bool:
        return self.num_computed_tokens >= self.num_prompt_tokens

    @property
    def num_blocks(self) -> int:
        return (self.num_tokens + self.block_size - 1) // self.block_size

    @property
    def last_block_num_tokens(self) -> int:
        return self.num_tokens - (self.num_blocks - 1) * self.block_size

    def block(self, i: int) -> list[int]:
        assert 0 <= i < self.num_blocks
        return self.token_ids[i * self.block_size:(i + 1) * self.block_size]

    def append_token(self, token_id: int) -> None:
        self.token_ids.append(token_id)
        self.last_token = token_id
        self.num_tokens += 1
        self.generated_completion_tokens += 1
        self.rope_pos += 1
        self.tail_uncompressed_len += 1


@dataclass
class ScheduledSeq:
    seq: Sequence
    num_new_tokens: int
