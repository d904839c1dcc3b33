"""Host-side scheduling of KV compression and application of its events.

* DecodeMetadata.build: per-step decode metadata with the semantics of the
  reference's prepare_decode (nanokvllm/engine/model_runner.py:265-285):
  positions are rope_pos (logical, never shrink), slots and context_lens come
  from the PHYSICAL length len(seq), so they stay right after compression.
  The per-sequence Python loops are replaced by numpy over the batch.
* PeriodicCompressScheduler: the periodic selection of prepare_decode
  (model_runner.py:291-332): a step counter, the eligibility rule
  (tail_len != block_size-1, tail_uncompressed_len >= window tokens,
  full_blocks >= window_blocks) and the FIRST kv_compress_topk eligible
  sequences in batch order. It also fills the device/host companions of the
  Context so the compress step needs no per-layer host work or syncs.
* prepare_threshold_context: KvChat's prepare_compression_context
  (KvChat/engine/model_runner.py:304-339).
* apply_window_events / apply_threshold_events: the event half of
  Scheduler.postprocess (nanokvllm/engine/scheduler.py:103-125 and
  KvChat/engine/scheduler.py:73-87).
"""

from __future__ import annotations

from dataclasses import dataclass
from itertools import chain

import numpy as np
import torch

from ..utils.context import Context


def padded_block_tables(seqs) -> tuple[np.ndarray, np.ndarray]:
    """The reference's prepare_block_tables (nanokvllm/engine/model_runner.py:154-158)
    on the host: rows padded with -1 to the longest table, int32; one
    scatter of all tables instead of a copy per row. Also returns the
    widths."""
    tables = [s.block_table for s in seqs]
    n = len(tables)
    widths = np.fromiter(map(len, tables), dtype=np.int64, count=n)
    mb = int(widths.max()) if n else 0
    bt = np.full((n, mb), -1, dtype=np.int32)
    if n:
        bt[np.arange(mb) < widths[:, None]] = np.fromiter(
            chain.from_iterable(tables), dtype=np.int32, count=int(widths.sum()))
    return bt, widths


@dataclass
class DecodeMetadata:
    input_ids: np.ndarray
    positions: np.ndarray
    slot_mapping: np.ndarray
    context_lens: np.ndarray
    block_tables: np.ndarray

    @classmethod
    def build(cls, seqs, block_size: int) -> "DecodeMetadata":
        n = len(seqs)
        lens = np.fromiter((s.num_tokens for s in seqs), dtype=np.int64, count=n)
        bt, widths = padded_block_tables(seqs)
        last_blk = bt[np.arange(n), np.maximum(widths - 1, 0)].astype(np.int64)
        last_cnt = lens - (((lens + block_size - 1) // block_size) - 1) * block_size
        slots = last_blk * block_size + last_cnt - 1
        return cls(
            input_ids=np.fromiter((s.last_token for s in seqs), dtype=np.int64, count=n),
            positions=np.fromiter((s.rope_pos for s in seqs), dtype=np.int64, count=n),
            slot_mapping=slots.astype(np.int32),
            context_lens=lens.astype(np.int32),
            block_tables=bt,
        )

    def to_device(self, device, pin: bool = True):
        def t(a):
            x = torch.from_numpy(a)
            if pin and torch.cuda.is_available():
                x = x.pin_memory()
            return x.to(device, non_blocking=True)
        return (t(self.input_ids), t(self.positions), t(self.slot_mapping), t(self.context_lens),
                t(self.block_tables))


class PeriodicCompressScheduler:
    def __init__(self, config, block_size: int):
        self.block_size = block_size
        self.period = config.kv_compress_period
        self.topk = config.kv_compress_topk
        self.window_blocks = config.kv_compress_window_blocks
        self.decode_step_counter = 0

    def select(self, seqs) -> tuple[bool, list[int], list[int]]:
        B = self.block_size
        window_tokens = self.window_blocks * B
        self.decode_step_counter += 1
        is_step = self.decode_step_counter % self.period == 0
        sel, ids = [], []
        if is_step:
            for i, seq in enumerate(seqs):
                L = len(seq)
                if L % B == B - 1:
                    continue
                if seq.tail_uncompressed_len >= window_tokens and L // B >= self.window_blocks:
                    sel.append(i)
                    ids.append(seq.seq_id)
                    if len(sel) == self.topk:
                        break
        return is_step, sel, ids

    def fill_context(self, ctx: Context, seqs, meta: DecodeMetadata | None = None) -> None:
        """Writes the compression fields of `ctx` for this step (the Context's
        context_lens must already be on the device)."""
        is_step, sel, ids = self.select(seqs)
        ctx.compress_need_mask = None
        # True on a step that compresses, so ModelRunner.run_model takes the
        # eager path (its graphs were captured without compression); the
        # reference leaves this False and would replay a graph instead.
        ctx.compress_any = bool(is_step and sel)
        ctx.is_compress_step = is_step
        ctx.compress_selected_batch_indices = sel
        ctx.compress_selected_seq_ids = ids
        if is_step and sel:
            ctx.compress_base_context_lens = ctx.context_lens.clone()
            dev = ctx.context_lens.device
            ctx.compress_selected_t = torch.tensor(sel, dtype=torch.int32).to(dev, non_blocking=True)
            if meta is not None:
                ctx.compress_base_context_lens_host = meta.context_lens.tolist()
                ctx.block_tables_host = meta.block_tables.tolist()
        else:
            ctx.compress_base_context_lens = None

    # ---------------------------------------------------------- device-side selection
    def device_buffers(self, batch: int, device) -> dict:
        """Static buffers of a graph-captured compression step (allocate once
        per captured batch size)."""
        pin = torch.cuda.is_available()
        return {
            "selected": torch.full((self.topk,), -1, dtype=torch.int32, device=device),
            "base_lens": torch.zeros(batch, dtype=torch.int32, device=device),
            "tail_uncompressed": torch.zeros(batch, dtype=torch.int32, device=device),
            "selected_host": torch.full((self.topk,), -1, dtype=torch.int32).pin_memory()
            if pin else torch.full((self.topk,), -1, dtype=torch.int32),
        }

    def fill_context_device(self, ctx: Context, seqs, buffers: dict) -> bool:
        """Like fill_context, but leaves the choice of rows to the device
        (nkv_window_select inside the step), so the compression step can be
        replayed from a CUDA graph captured once: only the per-sequence
        tail_uncompressed counters are uploaded. Returns is_compress_step;
        on such a step the runner replays its compression graph (captured
        with this context) instead of the plain decode graph, and calls
        events_from_device after the step."""
        self.decode_step_counter += 1
        is_step = self.decode_step_counter % self.period == 0
        ctx.compress_need_mask = None
        ctx.compress_any = False
        ctx.is_compress_step = is_step
        ctx.compress_selected_batch_indices = []
        ctx.compress_selected_seq_ids = []
        ctx.compress_device_select = True
        ctx.compress_topk = self.topk
        ctx.compress_selected_t = buffers["selected"]
        ctx.compress_base_context_lens = buffers["base_lens"][: len(seqs)]
        tail = buffers["tail_uncompressed"]
        if is_step:
            host = torch.tensor([s.tail_uncompressed_len for s in seqs], dtype=torch.int32)
            if tail.is_cuda and torch.cuda.is_available():
                host = host.pin_memory()
            tail[: len(seqs)].copy_(host, non_blocking=True)
        ctx.compress_tail_uncompressed_t = tail[: len(seqs)]
        ctx.compress_selected_host = buffers["selected_host"]
        return is_step

    def events_from_device(self, selected_host, base_lens_host, block_tables_host,
                           keep_blocks: int, keep_extra_tokens: int,
                           num_layers: int) -> list[dict]:
        """The events of a device-selected compression step, built after the
        step from the selection it copied back (the same events
        MyCompressCompact builds on a host-selected step)."""
        B = self.block_size
        window_tokens = self.window_blocks * B
        keep_tokens = keep_blocks * B + keep_extra_tokens
        events = []
        for b in [int(x) for x in selected_host if int(x) >= 0]:
            new_len = int(base_lens_host[b]) - window_tokens + keep_tokens
            keep_after = (new_len + B - 1) // B
            events.append({
                "batch_index": b,
                "layer": num_layers - 1,
                "new_context_len": new_len,
                "keep_blocks": keep_after,
                "freed_block_ids": [int(x) for x in block_tables_host[b][keep_after:] if int(x) >= 0],
                "tail_uncompressed_len_after": 0,
            })
        return events


def prepare_threshold_context(ctx: Context, seqs, config, query_window_manager) -> None:
    """KvChat's per-step trigger (KvChat/engine/model_runner.py:304-339): a
    sequence compresses when len == prompt + S; its query window is active
    for the W steps before (S_i - W < len <= S_i). S and R for the whole batch
    come from the FIRST sequence, as in the reference."""
    W = config.query_window_size
    active_idx, active_ids, seq_ids, need = [], [], [], []
    rS = rR = 0
    for i, seq in enumerate(seqs):
        seq_ids.append(seq.seq_id)
        S_i = seq.num_prompt_tokens + config.kv_compress_S
        R_i = seq.num_prompt_tokens + config.kv_compress_R
        if rS == 0:
            rS, rR = S_i, R_i
        L = len(seq)
        need.append(L == S_i)
        if S_i - W < L <= S_i:
            active_idx.append(i)
            active_ids.append(seq.seq_id)
            if not query_window_manager.has(seq.seq_id):
                query_window_manager.activate(seq.seq_id)
        elif query_window_manager.has(seq.seq_id):
            query_window_manager.free(seq.seq_id)
    ctx.compress_need_mask = need
    ctx.compress_any = any(need)
    ctx.q_window_active_indices = active_idx
    ctx.q_window_active_seq_ids = active_ids
    ctx.seq_ids = seq_ids
    ctx.runtime_compress_S = rS
    ctx.runtime_compress_R = rR


def _seq(x):
    return getattr(x, "seq", x)


def apply_window_events(seqs, events, block_manager) -> None:
    """nanokvllm Scheduler.postprocess, event part: the last event per batch
    index wins; truncate blocks, set the physical length, reset the counter."""
    if not events:
        return
    dedup = {}
    for ev in events:
        b = ev["batch_index"]
        if 0 <= b < len(seqs):
            dedup[b] = ev
    for b, ev in dedup.items():
        seq = _seq(seqs[b])
        block_manager.truncate_blocks(seq, ev["keep_blocks"])
        seq.num_tokens = ev["new_context_len"]
        seq.tail_uncompressed_len = ev.get("tail_uncompressed_len_after", 0)


def apply_threshold_events(seqs, events, block_manager) -> None:
    """KvChat Scheduler.postprocess, event part (no de-duplication)."""
    if not events:
        return
    for ev in events:
        b = ev["batch_index"]
        if b < 0 or b >= len(seqs):
            continue
        seq = _seq(seqs[b])
        block_manager.truncate_blocks(seq, ev["keep_blocks"])
        seq.num_tokens = ev["R"]
