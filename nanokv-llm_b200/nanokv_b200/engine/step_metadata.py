"""Per-step metadata of the unified scheduler (mixed prefill chunks + decode
rows in one batch), vectorised.

The reference builds it in ModelRunner.prepare_step
(nanokvllm/engine/model_runner.py:160-219) with Python loops over every new
token (positions, slot_mapping) and prepare_block_tables (:154-158); at
batch 256 with prefill chunks of 2,048 tokens that is tens of thousands of
Python iterations per step on the host. StepMetadata.build computes the same
arrays with numpy over the batch:

  input_ids       seq[start:end] of every row, concatenated (int64)
  positions       start..end-1 of every row (int64)
  cu_seqlens_q/k  prefix sums of the new tokens / of the end positions (int32)
  max_seqlen_q/k  largest new-token count / end position
  slot_mapping    block_table[pos // block_size] * block_size + pos % block_size (int32)
  context_lens    end = num_computed_tokens + num_new_tokens (int32)
  logits_indices  index of each row's last new token in the step (int64)
  block_tables    rows padded with -1 to the longest table (int32)

where start = seq.num_computed_tokens and end = start + num_new_tokens.
StepMetadata.set_context uploads them (pinned, non-blocking) and sets the
attention Context exactly as prepare_step does: context_lens on an
all-decode step, cu_seqlens_q/k otherwise.
"""

from __future__ import annotations

from dataclasses import dataclass
from itertools import chain

import numpy as np
import torch

from ..utils.context import set_context
from .compress_schedule import padded_block_tables


@dataclass
class StepMetadata:
    input_ids: np.ndarray
    positions: np.ndarray
    cu_seqlens_q: np.ndarray
    cu_seqlens_k: np.ndarray
    max_seqlen_q: int
    max_seqlen_k: int
    slot_mapping: np.ndarray
    context_lens: np.ndarray
    logits_indices: np.ndarray
    block_tables: np.ndarray

    @classmethod
    def build(cls, scheduled, block_size: int) -> "StepMetadata":
        """`scheduled`: items with `.seq` (a request: token_ids, num_computed_tokens,
        block_table) and `.num_new_tokens`."""
        n = len(scheduled)
        seqs = [s.seq for s in scheduled]
        news = np.fromiter((s.num_new_tokens for s in scheduled), dtype=np.int64, count=n)
        starts = np.fromiter((s.num_computed_tokens for s in seqs), dtype=np.int64, count=n)
        ends = starts + news
        cu_q = np.zeros(n + 1, dtype=np.int64)
        np.cumsum(news, out=cu_q[1:])
        cu_k = np.zeros(n + 1, dtype=np.int64)
        np.cumsum(ends, out=cu_k[1:])
        total = int(cu_q[-1])
        rows = np.repeat(np.arange(n), news)
        positions = np.arange(total, dtype=np.int64) - np.repeat(cu_q[:-1] - starts, news)

        bt, widths = padded_block_tables(seqs)
        blk = positions // block_size
        # the reference indexes seq.block_table[pos // block_size] and fails
        # past its end
        if total and not bool((blk < widths[rows]).all()):
            raise IndexError("a new token lies past its sequence's block table")
        slots = bt[rows, blk].astype(np.int64) * block_size + positions % block_size

        input_ids = np.fromiter(
            chain.from_iterable(s.token_ids[int(a):int(b)] for s, a, b in zip(seqs, starts, ends)),
            dtype=np.int64, count=total)
        return cls(
            input_ids=input_ids,
            positions=positions,
            cu_seqlens_q=cu_q.astype(np.int32),
            cu_seqlens_k=cu_k.astype(np.int32),
            max_seqlen_q=int(news.max()) if n else 0,
            max_seqlen_k=int(ends.max()) if n else 0,
            slot_mapping=slots.astype(np.int32),
            context_lens=ends.astype(np.int32),
            logits_indices=cu_q[1:] - 1,
            block_tables=bt,
        )

    def set_context(self, all_decode: bool, device, pin: bool = True):
        """Uploads the step's tensors and sets the Context as prepare_step
        does; returns (input_ids, positions, logits_indices) on `device`."""
        def t(a):
            x = torch.from_numpy(np.ascontiguousarray(a))
            if pin and torch.cuda.is_available():
                x = x.pin_memory()
            return x.to(device, non_blocking=True)

        input_ids, positions, logits_indices = t(self.input_ids), t(self.positions), \
            t(self.logits_indices)
        slot_mapping, block_tables = t(self.slot_mapping), t(self.block_tables)
        if all_decode:
            context_lens, cu_q, cu_k = t(self.context_lens), None, None
        else:
            context_lens, cu_q, cu_k = None, t(self.cu_seqlens_q), t(self.cu_seqlens_k)
        set_context(all_decode, cu_q, cu_k, self.max_seqlen_q, self.max_seqlen_k, slot_mapping,
                    context_lens, block_tables)
        return input_ids, positions, logits_indices
