"""Tensor-parallel sharding of the path by KV head, on CPU with gloo ranks.

Under TP each rank holds Hk/N kv heads and their Hq/N q heads of every layer
(nanokvllm/models/qwen3.py:53-59, engine/model_runner.py:140). Properties the
multi-GPU path relies on, checked with world_size 2:
  * decode shards, concatenated over heads, equal the unsharded decode
    (CPU oracle);
  * after a compression step every rank reports the same new lengths,
    keep_blocks and freed blocks (rank 0's events drive the host metadata),
    although each rank ranks tokens by its local heads only (CPU oracle);
  * the product's host path under TP -- PeriodicCompressScheduler selecting
    the rows, the step's events built from the host copies, rank 0's events
    applied through apply_window_events to the block manager -- leaves every
    rank with the same block tables, lengths and free list, equal to what
    each rank's own compaction wrote, over several decode steps and two
    compression steps (nanokvllm/engine/model_runner.py:381-397,
    scheduler.py:103-125);
  * a rank that dies between steps is detected through the group's timeout;
  * RowParallelOProj's default path equals the unsharded product.
"""

import os
import socket
from itertools import count

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, repo, out_q):
    import sys
    sys.path[:0] = [repo]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle.attention import paged_decode_ref, store_kvcache_ref
        from oracle.inputs import make_paged_batch
        from oracle.window_compress import compression_events, window_compress_ref

        Hq, Hk = 16, 8
        pb = make_paged_batch(seed=5, lens=[300, 1300, 2100, 1500], Hq=Hq, Hk=Hk)
        hk, hq = Hk // world, Hq // world
        ks, vs = slice(rank * hk, (rank + 1) * hk), slice(rank * hq, (rank + 1) * hq)
        kc = pb.k_cache[:, :, ks].contiguous()
        vc = pb.v_cache[:, :, ks].contiguous()
        q = pb.q[:, vs].contiguous()
        store_kvcache_ref(pb.k_new[:, ks].contiguous(), pb.v_new[:, ks].contiguous(), kc, vc,
                          pb.slot_mapping)
        dec = paged_decode_ref(q, kc, vc, pb.block_tables, pb.context_lens, 128 ** -0.5)
        sel = [1, 2, 3]
        cl = pb.context_lens.clone()
        keep, new_lens = window_compress_ref(q, kc, vc, pb.block_tables, pb.context_lens.clone(), cl,
                                             sel, 256, 4, 2, 1)
        ev = compression_events(pb.block_tables, sel, new_lens, 256, 0)
        gathered = [None] * world
        dist.all_gather_object(gathered, {"dec": dec, "events": ev, "lens": cl.tolist(),
                                          "keep": keep})
        if rank == 0:
            out_q.put(gathered)
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_two_rank_kv_head_sharding():
    from oracle.attention import paged_decode_ref, store_kvcache_ref
    from oracle.inputs import make_paged_batch

    world = 2
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, repo, q)) for r in range(world)]
    for p in procs:
        p.start()
    gathered = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # decode: per-rank head shards concatenate to the unsharded result
    pb = make_paged_batch(seed=5, lens=[300, 1300, 2100, 1500], Hq=16, Hk=8)
    kc, vc = pb.k_cache.clone(), pb.v_cache.clone()
    store_kvcache_ref(pb.k_new, pb.v_new, kc, vc, pb.slot_mapping)
    full = paged_decode_ref(pb.q, kc, vc, pb.block_tables, pb.context_lens, 128 ** -0.5)
    cat = torch.cat([g["dec"] for g in gathered], dim=1)
    assert torch.allclose(cat, full, atol=1e-5)
    # compression metadata agrees across ranks
    assert gathered[0]["events"] == gathered[1]["events"]
    assert gathered[0]["lens"] == gathered[1]["lens"] == [300, 789, 1589, 989]
    assert gathered[0]["keep"].shape == gathered[1]["keep"].shape


def _host_path_rank_main(rank, world, port, repo, out_q):
    import sys
    sys.path[:0] = [repo, os.path.join(repo, "nanokv-llm_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import types

        from nanokv_b200.engine.compress_schedule import (DecodeMetadata,
                                                          PeriodicCompressScheduler,
                                                          apply_window_events)
        from nanokv_b200.utils.context import Context
        from oracle.host_state import BlockPool, SeqState
        from oracle.window_compress import window_compress_ref

        Hq, Hk, D, BS, NB = 16, 8, 128, 256, 96
        hq, hk = Hq // world, Hk // world
        # every rank holds the same request state (the engine ships it to the
        # workers each step); the caches hold this rank's kv heads only
        SeqState.counter = count()
        rng = np.random.default_rng(8)
        lens = [300, 1300, 2100, 1500, 2700, 1279]
        seqs = [SeqState(rng.integers(0, 50000, L).tolist()) for L in lens]
        bm = BlockPool(NB, BS)
        for s_ in seqs:
            bm.allocate(s_)
            s_.num_computed_tokens = len(s_)
            s_.tail_uncompressed_len = 1100
        g = torch.Generator().manual_seed(9)
        k_all = torch.randn(NB, BS, Hk, D, generator=g).to(torch.bfloat16)
        v_all = torch.randn(NB, BS, Hk, D, generator=g).to(torch.bfloat16)
        kc = k_all[:, :, rank * hk:(rank + 1) * hk].contiguous()
        vc = v_all[:, :, rank * hk:(rank + 1) * hk].contiguous()
        cfg = types.SimpleNamespace(kv_compress_period=3, kv_compress_topk=3,
                                    kv_compress_window_blocks=4)
        sched = PeriodicCompressScheduler(cfg, BS)
        log = []
        for step in range(7):
            meta = DecodeMetadata.build(seqs, BS)
            ctx = Context(use_decode_kernel=True, context_lens=torch.from_numpy(meta.context_lens))
            sched.fill_context(ctx, seqs, meta)
            events = None
            local_lens = None
            if ctx.compress_any:
                sel = ctx.compress_selected_batch_indices
                q = torch.randn(len(seqs), Hq, D, generator=g).to(torch.bfloat16)
                q_local = q[:, rank * hq:(rank + 1) * hq].contiguous()
                cl = torch.from_numpy(meta.context_lens.copy())
                window_compress_ref(q_local, kc, vc, torch.from_numpy(meta.block_tables),
                                    cl.clone(), cl, sel, BS, 4, 2, 1)
                local_lens = [int(cl[b]) for b in sel]
                # the step's events from the host copies (the product's builder),
                # then rank 0's events go to every rank
                selected = sel + [-1] * (cfg.kv_compress_topk - len(sel))
                events = sched.events_from_device(selected, ctx.compress_base_context_lens_host,
                                                  ctx.block_tables_host, keep_blocks=2,
                                                  keep_extra_tokens=1, num_layers=28)
                box = [events if rank == 0 else None]
                dist.broadcast_object_list(box, src=0)
                events = box[0]
            apply_window_events(seqs, events, bm)
            if local_lens is not None:
                applied = [seqs[ev["batch_index"]].num_tokens for ev in events]
                assert applied == local_lens, (rank, step, applied, local_lens)
            for s_ in seqs:  # a decode step: each request takes one token
                s_.append_token(int(rng.integers(0, 50000)))
                bm.may_append(s_)
                s_.num_computed_tokens += 1
            log.append({"events": events, "tables": [list(s_.block_table) for s_ in seqs],
                        "lens": [len(s_) for s_ in seqs], "bm": bm.state()})
        gathered = [None] * world
        dist.all_gather_object(gathered, log)
        if rank == 0:
            out_q.put(gathered)
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_two_rank_product_host_path_agrees():
    world = 2
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_host_path_rank_main, args=(r, world, port, repo, q))
             for r in range(world)]
    for p in procs:
        p.start()
    gathered = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    log0, log1 = gathered
    assert log0 == log1
    steps_with_events = [i for i, rec in enumerate(log0) if rec["events"]]
    assert steps_with_events == [2, 5], steps_with_events  # period 3
    # the first compression step takes the first three eligible rows in batch
    # order; 300 tokens is below the window, 1279 % 256 == 255 is skipped
    assert [ev["batch_index"] for ev in log0[2]["events"]] == [1, 2, 3]


def _faulty_rank_main(rank, world, port, repo, out_q):
    """Rank 1 fails (raises) before the step's metadata exchange; rank 0 must
    learn it from the collective -- an error within the group's short
    timeout -- instead of blocking forever."""
    import datetime
    import sys
    sys.path[:0] = [repo]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    from oracle.inputs import make_paged_batch
    from oracle.window_compress import compression_events, window_compress_ref

    pb = make_paged_batch(seed=5, lens=[300, 1300, 2100, 1500], Hq=16, Hk=8)
    hk, hq = 8 // world, 16 // world
    ks, qs = slice(rank * hk, (rank + 1) * hk), slice(rank * hq, (rank + 1) * hq)
    kc, vc = pb.k_cache[:, :, ks].contiguous(), pb.v_cache[:, :, ks].contiguous()
    cl = pb.context_lens.clone()
    _, new_lens = window_compress_ref(pb.q[:, qs].contiguous(), kc, vc, pb.block_tables,
                                      pb.context_lens.clone(), cl, [1, 2], 256, 4, 2, 1)
    ev = compression_events(pb.block_tables, [1, 2], new_lens, 256, 0)
    if rank == 1:
        raise SystemExit(3)  # dies between steps, with no collective in flight
    import time
    t0 = time.monotonic()
    try:
        got = [None] * world
        dist.all_gather_object(got, ev)
        out_q.put(("no error", time.monotonic() - t0))
    except Exception as exc:  # noqa: BLE001 - any collective error is the detection
        out_q.put(("detected", time.monotonic() - t0, type(exc).__name__))


@pytest.mark.timeout(300)
def test_dead_rank_is_detected_not_waited_for():
    world = 2
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_faulty_rank_main, args=(r, world, port, repo, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
    assert res[0] == "detected", res
    assert res[1] < 60, res  # well inside the group's timeout plus set-up slack
    assert procs[1].exitcode == 3


def _oproj_rank_main(rank, world, port, repo, out_q):
    import sys
    sys.path[:0] = [repo, os.path.join(repo, "nanokv-llm_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from nanokv_b200.layers.linear import RowParallelOProj

        g = torch.Generator().manual_seed(40)
        x_full = torch.randn(8, 64, generator=g)
        w_full = torch.randn(32, 64, generator=g)
        k = 64 // world  # the rank's shard of the input dim (RowParallelLinear)
        layer = RowParallelOProj(w_full[:, rank * k:(rank + 1) * k].contiguous())
        assert layer.fused is None  # opt-in only
        y = layer(x_full[:, rank * k:(rank + 1) * k].contiguous())
        if rank == 0:
            out_q.put((y, x_full @ w_full.T))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_row_parallel_oproj_default_path_two_ranks():
    """RowParallelOProj without fusion is the reference's RowParallelLinear
    forward (nanokvllm/layers/linear.py:151-155): each rank's F.linear of its
    input shard, then dist.all_reduce -- two gloo ranks on the CPU give the
    unsharded product."""
    world = 2
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_oproj_rank_main, args=(r, world, port, repo, q))
             for r in range(world)]
    for p in procs:
        p.start()
    y, ref = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert torch.allclose(y, ref, atol=1e-4, rtol=1e-5)
