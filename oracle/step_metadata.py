"""Restatement of the unified scheduler's per-step metadata -- TEST
INFRASTRUCTURE ONLY (see the package header).

prepare_step_ref follows ModelRunner.prepare_step
(nanokvllm/engine/model_runner.py:160-219) and prepare_block_tables
(:154-158) token by token, in plain Python lists, returning host values
instead of uploading them; its outputs on three batches are pinned to the
reference's own prepare_step by tests/golden/step_metadata.json.
"""

from __future__ import annotations


def prepare_step_ref(scheduled, block_size: int) -> dict:
    """`scheduled`: items with `.seq` (token_ids, num_computed_tokens,
    block_table) and `.num_new_tokens`."""
    input_ids, positions, slot_mapping, context_lens, logits_indices = [], [], [], [], []
    cu_q, cu_k = [0], [0]
    max_q = max_k = 0
    offset = 0
    for sched in scheduled:  # model_runner.py:179-198
        seq = sched.seq
        new = sched.num_new_tokens
        start = seq.num_computed_tokens
        end = start + new
        input_ids.extend(seq.token_ids[start:end])
        positions.extend(range(start, end))
        cu_q.append(cu_q[-1] + new)
        cu_k.append(cu_k[-1] + end)
        max_q = max(max_q, new)
        max_k = max(max_k, end)
        for pos in range(start, end):
            block_id = seq.block_table[pos // block_size]
            slot_mapping.append(block_id * block_size + pos % block_size)
        context_lens.append(end)
        offset += new
        logits_indices.append(offset - 1)
    width = max(len(s.seq.block_table) for s in scheduled)  # :154-158
    block_tables = [s.seq.block_table + [-1] * (width - len(s.seq.block_table))
                    for s in scheduled]
    return {"input_ids": input_ids, "positions": positions, "cu_seqlens_q": cu_q,
            "cu_seqlens_k": cu_k, "max_seqlen_q": max_q, "max_seqlen_k": max_k,
            "slot_mapping": slot_mapping, "context_lens": context_lens,
            "logits_indices": logits_indices, "block_tables": block_tables}
