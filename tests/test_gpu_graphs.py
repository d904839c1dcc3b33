"""The decode-step kernels inside a captured CUDA graph, as the reference's
ModelRunner replays them (nanokvllm/engine/model_runner.py:366-379, :401-441):
static input buffers are refilled before every replay and results must match
the CPU oracle. Covers store + paged decode and the KvChat query-window
append (whose device index tensors make it capturable)."""

import numpy as np
import pytest
import torch

from oracle.attention import paged_decode_ref, store_kvcache_ref
from oracle.inputs import bf16, make_paged_batch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_store_and_decode_replayed_from_graph(cuda_lib):
    from nanokv_b200 import _lib, ops

    Hq, Hk, D = 32, 8, 128
    lens = [700, 3000, 1, 4100, 256, 1900]
    pb = make_paged_batch(seed=60, lens=lens, Hq=Hq, Hk=Hk, num_blocks=64)
    B, mb = len(lens), 20
    kc, vc = pb.k_cache.to(DEV), pb.v_cache.to(DEV)
    bt = torch.full((B, mb), -1, dtype=torch.int32, device=DEV)
    bt[:, :pb.block_tables.size(1)] = pb.block_tables.to(DEV)
    cl = torch.zeros(B, dtype=torch.int32, device=DEV)
    sm = torch.full((B,), -1, dtype=torch.int32, device=DEV)
    qkv = torch.zeros(B, (Hq + 2 * Hk) * D, dtype=torch.bfloat16, device=DEV)
    q, k, v = qkv.split([Hq * D, Hk * D, Hk * D], dim=-1)
    q, k, v = q.view(B, Hq, D), k.view(B, Hk, D), v.view(B, Hk, D)
    out = torch.empty(B, Hq, D, dtype=torch.bfloat16, device=DEV)
    ws = ops.decode_workspace(torch.device(DEV), B, Hq, Hk, D, mb, 256)

    def step():
        ops.store_kvcache(k, v, kc, vc, sm)
        ops.paged_decode(q, kc, vc, bt, cl, D ** -0.5, out=out, workspace=ws)

    step()  # eager warm-up outside capture (library load, attributes)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    rng = np.random.default_rng(61)
    ref_k, ref_v = pb.k_cache.clone(), pb.v_cache.clone()
    cur = list(lens)
    for it in range(3):
        new = bf16(rng.standard_normal((B, (Hq + 2 * Hk) * D), dtype=np.float32))
        slots = []
        for b in range(B):
            pos = cur[b] - 1
            slots.append(int(pb.block_tables[b, pos // 256]) * 256 + pos % 256)
        qkv.copy_(new.to(DEV))
        cl.copy_(torch.tensor(cur, dtype=torch.int32))
        sm.copy_(torch.tensor(slots, dtype=torch.int32))
        graph.replay()
        torch.cuda.synchronize()
        nq, nk, nv = new.split([Hq * D, Hk * D, Hk * D], dim=-1)
        store_kvcache_ref(nk.reshape(B, Hk, D), nv.reshape(B, Hk, D), ref_k, ref_v,
                          torch.tensor(slots, dtype=torch.int32))
        ref = paged_decode_ref(nq.reshape(B, Hq, D), ref_k, ref_v, pb.block_tables,
                               torch.tensor(cur, dtype=torch.int32), D ** -0.5)
        assert (out.float().cpu() - ref).abs().max().item() <= 2e-2
        assert torch.equal(kc.cpu().view(torch.int16), ref_k.view(torch.int16))
        # grow sequences that still fit their last block (slot stays mapped)
        cur = [L + 1 if (L % 256) != 0 else L for L in cur]
    assert _lib.read_device_error(clear=True) == 0


def test_query_window_append_replayed_from_graph(cuda_lib):
    from nanokv_b200 import ops

    Hq, D, W, L = 16, 128, 5, 2
    ring = torch.zeros(3, L, W, Hq, D, dtype=torch.bfloat16, device=DEV)
    q = torch.zeros(4, Hq, D, dtype=torch.bfloat16, device=DEV)
    bidx = torch.tensor([1, 3], dtype=torch.int32, device=DEV)
    slot = torch.tensor([2, 0], dtype=torch.int32, device=DEV)
    pos = torch.zeros(2, dtype=torch.int32, device=DEV)
    ops.query_window_append(q, ring, 1, bidx, slot, pos)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ops.query_window_append(q, ring, 1, bidx, slot, pos)
    for step in range(W):
        q.copy_(torch.full((4, Hq, D), float(step + 1), dtype=torch.bfloat16))
        pos.fill_(step)
        graph.replay()
    torch.cuda.synchronize()
    r = ring.float().cpu()
    for step in range(W):
        assert torch.all(r[2, 1, step] == step + 1) and torch.all(r[0, 1, step] == step + 1)
    assert torch.all(r[1] == 0) and torch.all(r[:, 0] == 0)


def test_graph_replay_with_padding_rows(cuda_lib):
    """The reference's graph replay for a batch smaller than the captured
    one (nanokvllm/engine/model_runner.py:370-376): rows past the batch get
    slot_mapping -1 and context_lens 0. The fused decode step must skip
    their store, give them a defined (zero) output instead of NaNs, and
    leave the live rows and the cache exactly as for the unpadded batch."""
    from nanokv_b200 import _lib, ops

    Hq, Hk, D = 32, 8, 128
    lens = [700, 3000, 1900, 260]
    live = 2  # the step's real batch; rows 2 and 3 are padding
    pb = make_paged_batch(seed=62, lens=lens, Hq=Hq, Hk=Hk, num_blocks=64)
    B = len(lens)
    kc, vc = pb.k_cache.to(DEV), pb.v_cache.to(DEV)
    bt = pb.block_tables.to(DEV).clone()
    cl = torch.zeros(B, dtype=torch.int32, device=DEV)
    sm = torch.full((B,), -1, dtype=torch.int32, device=DEV)
    qkv = torch.zeros(B, (Hq + 2 * Hk) * D, dtype=torch.bfloat16, device=DEV)
    q, k, v = qkv.split([Hq * D, Hk * D, Hk * D], dim=-1)
    q, k, v = q.view(B, Hq, D), k.view(B, Hk, D), v.view(B, Hk, D)
    out = torch.empty(B, Hq, D, dtype=torch.bfloat16, device=DEV)
    ws = ops.decode_workspace(torch.device(DEV), B, Hq, Hk, D, bt.size(1), 256)

    def step():
        ops.decode_step(q, k, v, kc, vc, sm, bt, cl, D ** -0.5, out=out, workspace=ws)

    step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    new = bf16(np.random.default_rng(63).standard_normal((B, (Hq + 2 * Hk) * D),
                                                          dtype=np.float32))
    qkv.copy_(new.to(DEV))
    slots = [int(pb.block_tables[b, (lens[b] - 1) // 256]) * 256 + (lens[b] - 1) % 256
             for b in range(live)]
    # as the reference fills its graph inputs: -1 slots and zero lengths past bs
    sm.fill_(-1)
    sm[:live] = torch.tensor(slots, dtype=torch.int32)
    cl.zero_()
    cl[:live] = torch.tensor(lens[:live], dtype=torch.int32)
    out.fill_(float("nan"))
    graph.replay()
    torch.cuda.synchronize()
    assert _lib.read_device_error(clear=True) == 0
    nq, nk, nv = new.split([Hq * D, Hk * D, Hk * D], dim=-1)
    ref_k, ref_v = pb.k_cache.clone(), pb.v_cache.clone()
    store_kvcache_ref(nk[:live].reshape(live, Hk, D), nv[:live].reshape(live, Hk, D), ref_k, ref_v,
                      torch.tensor(slots, dtype=torch.int32))
    ref = paged_decode_ref(nq[:live].reshape(live, Hq, D), ref_k, ref_v, pb.block_tables[:live],
                           torch.tensor(lens[:live], dtype=torch.int32), D ** -0.5)
    got = out.float().cpu()
    assert (got[:live] - ref).abs().max().item() <= 2e-2
    assert torch.equal(got[live:], torch.zeros_like(got[live:]))  # defined, not NaN
    assert torch.equal(kc.cpu().view(torch.int16), ref_k.view(torch.int16))
    assert torch.equal(vc.cpu().view(torch.int16), ref_v.view(torch.int16))
