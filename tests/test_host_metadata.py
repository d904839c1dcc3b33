"""Host-side compression metadata vs traces recorded from the reference
(tests/golden/host_metadata.json, made by tests/golden/make_golden.py):
Scheduler.postprocess event application (the product's apply_window_events
/ apply_threshold_events driving a block manager's truncate_blocks), the
periodic selection of ModelRunner.prepare_decode, and KvChat's
prepare_compression_context. The requests and the block manager are the
oracle's models (oracle/host_state.py), which the same traces pin to the
reference's Sequence and BlockManager; in deployment the product drives the
reference's own objects. CPU only."""

import json
import types
from itertools import count

import numpy as np
import pytest

from nanokv_b200.engine.compress_schedule import (DecodeMetadata, PeriodicCompressScheduler,
                                                  apply_threshold_events, apply_window_events,
                                                  prepare_threshold_context)
from nanokv_b200.engine.query_window import QueryWindowManager
from nanokv_b200.utils.context import Context
from oracle.host_state import BlockPool, Scheduled, SeqState


@pytest.fixture(scope="module")
def trace(golden_dir):
    return json.loads((golden_dir / "host_metadata.json").read_text())


def _seq_state(s):
    return {"seq_id": s.seq_id, "num_tokens": s.num_tokens, "block_table": list(s.block_table),
            "num_cached_tokens": s.num_cached_tokens, "tail_uncompressed_len": s.tail_uncompressed_len,
            "rope_pos": s.rope_pos}


def _bm_state(bm):
    return bm.state()


def _replay_block_manager(trace, check: bool):
    tr = trace["block_manager"]
    rng = np.random.default_rng(5)
    shared = rng.integers(0, 50000, 512).tolist()
    prompts = [shared + rng.integers(0, 50000, 300).tolist(),
               shared + rng.integers(0, 50000, 40).tolist(),
               rng.integers(0, 50000, 1100).tolist(),
               rng.integers(0, 50000, 255).tolist()]
    assert prompts == tr["prompts"]
    SeqState.counter = count()
    bm = BlockPool(num_blocks=40, block_size=256)
    seqs = [SeqState(p, max_tokens=10**6, ignore_eos=True) for p in prompts]
    for s in seqs:
        bm.allocate(s)
        s.num_computed_tokens = s.num_prompt_tokens
    recorded = iter(tr["steps"])
    first = next(recorded)
    assert [_seq_state(s) for s in seqs] == first["seqs"]
    assert _bm_state(bm) == first["bm"]
    checked = 1
    for step in range(300):
        for s in seqs:
            bm.may_append(s)
        token_ids = rng.integers(0, 50000, len(seqs)).tolist()
        events = None
        if step in (120, 260):
            events = []
            for bi in (0, 2):
                s = seqs[bi]
                new_len = len(s) - 1024 + 513
                kb = (new_len + 255) // 256
                events.append({"batch_index": bi, "layer": 0, "new_context_len": new_len,
                               "keep_blocks": kb,
                               "freed_block_ids": [x for x in s.block_table[kb:] if x >= 0],
                               "tail_uncompressed_len_after": 0})
            events.append(dict(events[0]))
        apply_window_events(seqs, events, bm)
        for s, t in zip(seqs, token_ids):
            s.num_computed_tokens += 1
            s.append_token(t)
        if check and (events or step % 50 == 0):
            rec = next(recorded)
            assert rec["op"] == f"step{step}"
            assert rec["events"] == events
            assert [_seq_state(s) for s in seqs] == rec["seqs"], f"seq state at step {step}"
            assert _bm_state(bm) == rec["bm"], f"block manager at step {step}"
            checked += 1
    assert not check or checked == len(tr["steps"])
    return bm, seqs


def test_block_manager_and_events_replay(trace):
    _replay_block_manager(trace, check=True)


def test_block_manager_release_and_prefix_reuse(trace):
    """After the replay: can_append, deallocate of a sequence sharing prefix
    blocks, can_allocate / allocate of a new prompt that hits the prefix
    cache, and two more deallocations, against the reference's BlockManager
    (nanokvllm/engine/block_manager.py:55-96)."""
    bm, seqs = _replay_block_manager(trace, check=False)
    rel = iter(trace["block_manager_release"]["steps"])
    rec = next(rel)
    assert [bm.can_append(s) for s in seqs] == rec["value"]
    bm.deallocate(seqs[1])
    rec = next(rel)
    assert [_seq_state(s) for s in seqs] == rec["seqs"] and _bm_state(bm) == rec["bm"]
    new = SeqState(trace["block_manager_release"]["new_prompt"], max_tokens=10**6, ignore_eos=True)
    assert bm.can_allocate(new) == next(rel)["value"]
    bm.allocate(new)
    rec = next(rel)
    assert _seq_state(new) == rec["seq"] and _bm_state(bm) == rec["bm"]
    bm.deallocate(seqs[3])
    bm.deallocate(new)
    rec = next(rel)
    assert [_seq_state(s) for s in seqs] == rec["seqs"] and _seq_state(new) == rec["new"]
    assert _bm_state(bm) == rec["bm"]


def test_periodic_selection_matches_prepare_decode(trace):
    tr = trace["periodic_selection"]
    SeqState.counter = count()
    seqs = []
    for L, t in zip(tr["lens"], tr["tails"]):
        s = SeqState(list(range(L)))
        s.block_table = list(range(100, 100 + (L + 255) // 256))
        s.tail_uncompressed_len = t
        s.rope_pos = L + 17
        seqs.append(s)
    cfg = types.SimpleNamespace(kv_compress_period=tr["period"], kv_compress_topk=tr["topk"],
                                kv_compress_window_blocks=4)
    sched = PeriodicCompressScheduler(cfg, 256)
    for rec in tr["steps"]:
        meta = DecodeMetadata.build(seqs, 256)
        is_step, sel, ids = sched.select(seqs)
        assert sched.decode_step_counter == rec["step"]
        assert is_step == rec["is_compress_step"]
        assert sel == rec["selected"] and ids == rec["seq_ids"]
        assert meta.positions.tolist() == rec["positions"]
        assert meta.slot_mapping.tolist() == rec["slot_mapping"]
        assert meta.context_lens.tolist() == rec["context_lens"]
        if rec["base_lens"] is not None:
            assert meta.context_lens.tolist() == rec["base_lens"]
        for s in seqs:
            s.append_token(1)


def test_periodic_fill_context_host_companions():
    import torch

    SeqState.counter = count()
    seqs = [SeqState(list(range(L))) for L in (1500, 900, 2000)]
    for s, t in zip(seqs, (1024, 2000, 1100)):
        s.block_table = list(range(len(s.block_table), len(s.block_table) + s.num_blocks))
        s.tail_uncompressed_len = t
    cfg = types.SimpleNamespace(kv_compress_period=1, kv_compress_topk=20, kv_compress_window_blocks=4)
    sched = PeriodicCompressScheduler(cfg, 256)
    meta = DecodeMetadata.build(seqs, 256)
    ctx = Context(use_decode_kernel=True, context_lens=torch.from_numpy(meta.context_lens))
    sched.fill_context(ctx, seqs, meta)
    assert ctx.is_compress_step and ctx.compress_selected_batch_indices == [0, 2]
    assert ctx.compress_any  # compression steps run eagerly
    assert ctx.compress_selected_t.tolist() == [0, 2]
    assert ctx.compress_base_context_lens_host == [1500, 900, 2000]
    assert ctx.block_tables_host[1][:4] == seqs[1].block_table


def test_kvchat_context_decisions(trace):
    tr = trace["kvchat_context"]
    cfg = types.SimpleNamespace(kv_compress_S=511, kv_compress_R=257, query_window_size=50)
    qwm = QueryWindowManager(1, 50, 2, 128, device="cpu")
    SeqState.counter = count()
    seqs = [SeqState(list(range(p))) for p in tr["prompts"]]
    for rec in tr["decisions"]:
        for s in seqs:
            s.num_tokens = s.num_prompt_tokens + rec["extra"]
        ctx = Context()
        prepare_threshold_context(ctx, seqs, cfg, qwm)
        assert ctx.compress_need_mask == rec["need"]
        assert ctx.compress_any == rec["any"]
        assert ctx.q_window_active_indices == rec["active"]
        assert (ctx.runtime_compress_S, ctx.runtime_compress_R) == (rec["S"], rec["R"])
        assert [qwm.has(s.seq_id) for s in seqs] == rec["has"]


def test_threshold_events_truncate():
    SeqState.counter = count()
    bm = BlockPool(8, 256)
    s = SeqState(list(range(767)))
    bm.allocate(s)
    apply_threshold_events([s], [{"batch_index": 0, "layer": 27, "R": 513, "keep_blocks": 3,
                                  "freed_block_ids": []}], bm)
    assert s.num_tokens == 513 and len(s.block_table) == 3
    assert list(bm.free)[-1] == 3 or 3 in bm.free


def test_device_select_host_half_matches_host_selection():
    """The host half of the graph-captured compression step: fill_context_device
    uploads only the tail counters, and events_from_device, given the -1-padded
    list the device selection copies back, builds the same events as the
    host-selected path (oracle.window_compress.compression_events)."""
    import torch

    from oracle.window_compress import compression_events

    SeqState.counter = count()
    lens = (1500, 900, 2000, 1279, 3000)
    tails = (1024, 2000, 1100, 1024, 5)
    seqs = [SeqState(list(range(L))) for L in lens]
    nxt = 0
    for s, t in zip(seqs, tails):
        s.block_table = list(range(nxt, nxt + s.num_blocks))
        nxt += s.num_blocks
        s.tail_uncompressed_len = t
    cfg = types.SimpleNamespace(kv_compress_period=2, kv_compress_topk=4, kv_compress_window_blocks=4)
    host_sched = PeriodicCompressScheduler(cfg, 256)
    dev_sched = PeriodicCompressScheduler(cfg, 256)
    bufs = dev_sched.device_buffers(8, "cpu")
    meta = DecodeMetadata.build(seqs, 256)
    for step in (1, 2):
        is_step, sel, _ = host_sched.select(seqs)
        ctx = Context(use_decode_kernel=True, context_lens=torch.from_numpy(meta.context_lens))
        assert dev_sched.fill_context_device(ctx, seqs, bufs) == is_step
        assert ctx.compress_device_select and not ctx.compress_any
        assert ctx.compress_selected_t is bufs["selected"] and ctx.compress_topk == 4
        if not is_step:
            continue
        # 1279 % 256 == 255 and the last tail is short: rows 0 and 2 only
        assert sel == [0, 2]
        assert ctx.compress_tail_uncompressed_t.tolist() == list(tails)
        selected_host = sel + [-1] * (cfg.kv_compress_topk - len(sel))
        window_tokens, keep_tokens = 4 * 256, 2 * 256 + 1
        new_lens = torch.tensor([lens[b] - window_tokens + keep_tokens for b in sel])
        events = dev_sched.events_from_device(selected_host, list(lens), meta.block_tables.tolist(),
                                              keep_blocks=2, keep_extra_tokens=1, num_layers=28)
        assert events == compression_events(torch.from_numpy(meta.block_tables), sel, new_lens,
                                            256, 27)


def test_step_metadata_matches_prepare_step(golden_dir):
    """StepMetadata (vectorised) against the reference's own prepare_step
    (nanokvllm/engine/model_runner.py:160-219) on mixed prefill-chunk +
    decode, all-decode and single-prefill batches
    (tests/golden/step_metadata.json): every array and the Context it sets."""
    import torch

    from nanokv_b200.engine.step_metadata import StepMetadata
    from nanokv_b200.utils.context import get_context, reset_context

    tr = json.loads((golden_dir / "step_metadata.json").read_text())
    bs = tr["block_size"]
    for rec in tr["batches"]:
        SeqState.counter = count()
        sched = []
        for r in rec["seqs"]:
            s = SeqState(r["token_ids"])
            s.num_computed_tokens = r["num_computed_tokens"]
            s.block_table = list(r["block_table"])
            sched.append(Scheduled(s, r["num_new_tokens"]))
        meta = StepMetadata.build(sched, bs)
        ids, pos, logits_idx = meta.set_context(rec["all_decode"], "cpu")
        c = get_context()
        name = rec["name"]
        assert ids.tolist() == rec["input_ids"], name
        assert ids.dtype == torch.int64 and pos.dtype == torch.int64
        assert pos.tolist() == rec["positions"], name
        assert logits_idx.tolist() == rec["logits_indices"], name
        assert c.use_decode_kernel == rec["use_decode_kernel"], name
        assert c.slot_mapping.tolist() == rec["slot_mapping"] and c.slot_mapping.dtype == torch.int32
        assert c.block_tables.tolist() == rec["block_tables"], name
        assert (c.max_seqlen_q, c.max_seqlen_k) == (rec["max_seqlen_q"], rec["max_seqlen_k"])
        for key in ("cu_seqlens_q", "cu_seqlens_k", "context_lens"):
            got = getattr(c, key)
            assert (None if got is None else got.tolist()) == rec[key], (name, key)
            assert got is None or got.dtype == torch.int32
        reset_context()


def test_step_metadata_rejects_token_past_block_table():
    from nanokv_b200.engine.step_metadata import StepMetadata

    SeqState.counter = count()
    s = SeqState(list(range(300)))
    s.block_table = [7]  # 300 tokens need two 256-token blocks
    with pytest.raises(IndexError):
        StepMetadata.build([Scheduled(s, 300)], 256)


def test_step_metadata_oracle_pinned_and_random_batches(golden_dir):
    """The oracle's token-by-token prepare_step restatement reproduces the
    reference's own outputs (golden), and StepMetadata equals it on 200
    random mixed batches (prefill chunks of 1..2,100 tokens, decode rows,
    ragged block tables, 64- and 256-token blocks)."""
    from nanokv_b200.engine.step_metadata import StepMetadata
    from oracle.step_metadata import prepare_step_ref

    tr = json.loads((golden_dir / "step_metadata.json").read_text())
    for rec in tr["batches"]:
        SeqState.counter = count()
        sched = []
        for r in rec["seqs"]:
            s = SeqState(r["token_ids"])
            s.num_computed_tokens = r["num_computed_tokens"]
            s.block_table = list(r["block_table"])
            sched.append(Scheduled(s, r["num_new_tokens"]))
        ref = prepare_step_ref(sched, tr["block_size"])
        for key in ("input_ids", "positions", "slot_mapping", "logits_indices", "block_tables",
                    "max_seqlen_q", "max_seqlen_k"):
            assert ref[key] == rec[key], (rec["name"], key)
        if rec["all_decode"]:
            assert ref["context_lens"] == rec["context_lens"]
        else:
            assert (ref["cu_seqlens_q"], ref["cu_seqlens_k"]) == (rec["cu_seqlens_q"],
                                                                 rec["cu_seqlens_k"])

    rng = np.random.default_rng(23)
    for trial in range(200):
        bs = int(rng.choice([64, 256]))
        SeqState.counter = count()
        sched, next_block = [], 0
        for _ in range(int(rng.integers(1, 12))):
            total = int(rng.integers(1, 6000))
            computed = int(rng.integers(0, total))
            new = 1 if rng.random() < 0.5 else int(rng.integers(1, min(2100, total - computed) + 1))
            new = min(new, total - computed)
            s = SeqState(rng.integers(0, 1000, total).tolist())
            s.num_computed_tokens = computed
            nb = (computed + new + bs - 1) // bs + int(rng.integers(0, 3))  # spare blocks too
            s.block_table = (rng.permutation(nb) + next_block).tolist()
            next_block += nb
            sched.append(Scheduled(s, new))
        ref = prepare_step_ref(sched, bs)
        m = StepMetadata.build(sched, bs)
        assert m.input_ids.tolist() == ref["input_ids"], trial
        assert m.positions.tolist() == ref["positions"], trial
        assert m.slot_mapping.tolist() == ref["slot_mapping"], trial
        assert m.cu_seqlens_q.tolist() == ref["cu_seqlens_q"], trial
        assert m.cu_seqlens_k.tolist() == ref["cu_seqlens_k"], trial
        assert m.context_lens.tolist() == ref["context_lens"], trial
        assert m.logits_indices.tolist() == ref["logits_indices"], trial
        assert m.block_tables.tolist() == ref["block_tables"], trial
        assert (m.max_seqlen_q, m.max_seqlen_k) == (ref["max_seqlen_q"], ref["max_seqlen_k"])
