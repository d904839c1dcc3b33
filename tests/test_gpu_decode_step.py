"""The fused decode step (nkv_decode_step): slot write [+ KvChat query-window
append] + paged decode in one launch must equal the separate launches
(store_kvcache, query_window_append, paged_decode) on the same inputs, with
the reference's graph padding rows (slot -1, length 0) and a refused row
whose slot is not its current position."""

import numpy as np
import pytest
import torch

from oracle.attention import paged_decode_ref, store_kvcache_ref
from oracle.inputs import bf16, make_paged_batch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _qkv(B, Hq, Hk, seed):
    rng = np.random.default_rng(seed)
    qkv = bf16(rng.standard_normal((B, (Hq + 2 * Hk) * 128), dtype=np.float32)).to(DEV)
    q, k, v = qkv.split([Hq * 128, Hk * 128, Hk * 128], dim=-1)
    return q.view(B, Hq, 128), k.view(B, Hk, 128), v.view(B, Hk, 128)


@pytest.mark.parametrize("metadata_ready", [False, True])
@pytest.mark.parametrize("Hq,Hk", [(32, 8), (16, 8), (4, 1), (64, 8)])
def test_decode_step_equals_store_then_decode(cuda_lib, Hq, Hk, metadata_ready):
    # metadata_ready: the kernel launched just before (paged_decode) writes
    # none of the metadata, so reading it before the dependency wait is valid
    from nanokv_b200 import _lib, ops

    lens = [1, 300, 0, 4097, 128, 2500, 0, 7000]
    pb = make_paged_batch(seed=90 + Hq, lens=lens, Hq=Hq, Hk=Hk)
    q, k, v = _qkv(len(lens), Hq, Hk, 91)
    sm = pb.slot_mapping.to(DEV)  # -1 for the empty rows (graph padding)
    bt, cl = pb.block_tables.to(DEV), pb.context_lens.to(DEV)
    ka, va = pb.k_cache.to(DEV), pb.v_cache.to(DEV)
    kb, vb = ka.clone(), va.clone()
    ops.store_kvcache(k, v, ka, va, sm)
    sep = ops.paged_decode(q, ka, va, bt, cl, 128 ** -0.5)
    fused = ops.decode_step(q, k, v, kb, vb, sm, bt, cl, 128 ** -0.5, metadata_ready=metadata_ready)
    torch.cuda.synchronize()
    assert torch.equal(ka.view(torch.int16), kb.view(torch.int16))
    assert torch.equal(va.view(torch.int16), vb.view(torch.int16))
    assert torch.equal(sep.view(torch.int16), fused.view(torch.int16))
    assert _lib.read_device_error(clear=True) == 0
    # and against the oracle
    kc, vc = pb.k_cache.clone(), pb.v_cache.clone()
    store_kvcache_ref(k.cpu(), v.cpu(), kc, vc, pb.slot_mapping)
    ref = paged_decode_ref(q.cpu(), kc, vc, pb.block_tables, pb.context_lens, 128 ** -0.5)
    assert (fused.float().cpu() - ref).abs().max().item() <= 2e-2


def test_decode_step_refuses_slot_that_is_not_the_current_position(cuda_lib):
    from nanokv_b200 import _lib, ops

    pb = make_paged_batch(seed=95, lens=[600, 900], Hq=16, Hk=8)
    q, k, v = _qkv(2, 16, 8, 96)
    sm = pb.slot_mapping.clone()
    wrong = int(pb.block_tables[1, 0]) * 256 + 5  # a slot of row 1's first block
    sm[1] = wrong
    kd, vd = pb.k_cache.to(DEV), pb.v_cache.to(DEV)
    ops.decode_step(q, k, v, kd, vd, sm.to(DEV), pb.block_tables.to(DEV),
                    pb.context_lens.to(DEV), 128 ** -0.5)
    torch.cuda.synchronize()
    assert _lib.read_device_error(clear=True) & 0x1
    flat = kd.cpu().view(-1, 8 * 128)
    assert torch.equal(flat[wrong].view(torch.int16), pb.k_cache.view(-1, 8 * 128)[wrong].view(torch.int16))
    good = int(pb.slot_mapping[0])
    assert torch.equal(flat[good], k[0].cpu().reshape(-1))


def test_decode_step_appends_query_window(cuda_lib):
    from nanokv_b200 import ops

    B, Hq, Hk, W, L = 4, 16, 8, 6, 3
    pb = make_paged_batch(seed=97, lens=[700, 300, 1500, 80], Hq=Hq, Hk=Hk)
    q, k, v = _qkv(B, Hq, Hk, 98)
    ring_a = torch.zeros(3, L, W, Hq, 128, dtype=torch.bfloat16, device=DEV)
    ring_b = ring_a.clone()
    slot_of_row = torch.tensor([2, -1, 0, 1], dtype=torch.int32, device=DEV)
    pos_of_row = torch.tensor([4, 0, 1, 5], dtype=torch.int32, device=DEV)
    kd, vd = pb.k_cache.to(DEV), pb.v_cache.to(DEV)
    ops.decode_step(q, k, v, kd, vd, pb.slot_mapping.to(DEV), pb.block_tables.to(DEV),
                    pb.context_lens.to(DEV), 128 ** -0.5, ring=ring_a, layer_id=1,
                    ring_slot_of_row=slot_of_row, ring_pos_of_row=pos_of_row)
    active = torch.tensor([0, 2, 3], dtype=torch.int32, device=DEV)
    ops.query_window_append(q, ring_b, 1, active, slot_of_row[[0, 2, 3]].contiguous(),
                            pos_of_row[[0, 2, 3]].contiguous())
    torch.cuda.synchronize()
    assert torch.equal(ring_a.view(torch.int16), ring_b.view(torch.int16))
    assert torch.count_nonzero(ring_a[:, [0, 2]]) == 0


def test_decode_step_replayed_from_graph(cuda_lib):
    from nanokv_b200 import ops

    Hq, Hk = 32, 8
    lens = [700, 3000, 2, 1900]
    pb = make_paged_batch(seed=99, lens=lens, Hq=Hq, Hk=Hk)
    B = len(lens)
    kd, vd = pb.k_cache.to(DEV), pb.v_cache.to(DEV)
    bt, cl, sm = pb.block_tables.to(DEV), pb.context_lens.to(DEV), pb.slot_mapping.to(DEV)
    q = torch.zeros(B, Hq, 128, dtype=torch.bfloat16, device=DEV)
    k = torch.zeros(B, Hk, 128, dtype=torch.bfloat16, device=DEV)
    v = torch.zeros_like(k)
    out = torch.empty(B, Hq, 128, dtype=torch.bfloat16, device=DEV)
    ws = ops.decode_workspace(torch.device(DEV), B, Hq, Hk, 128, bt.size(1), 256)
    ops.decode_step(q, k, v, kd, vd, sm, bt, cl, 128 ** -0.5, out=out, workspace=ws,
                    metadata_ready=True)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ops.decode_step(q, k, v, kd, vd, sm, bt, cl, 128 ** -0.5, out=out, workspace=ws,
                        metadata_ready=True)
    ref_k, ref_v = pb.k_cache.clone(), pb.v_cache.clone()
    for it in range(3):
        nq, nk, nv = _qkv(B, Hq, Hk, 200 + it)
        q.copy_(nq), k.copy_(nk), v.copy_(nv)
        g.replay()
        torch.cuda.synchronize()
        store_kvcache_ref(nk.cpu(), nv.cpu(), ref_k, ref_v, pb.slot_mapping)
        ref = paged_decode_ref(nq.cpu(), ref_k, ref_v, pb.block_tables, pb.context_lens, 128 ** -0.5)
        assert (out.float().cpu() - ref).abs().max().item() <= 2e-2
        assert torch.equal(kd.cpu().view(torch.int16), ref_k.view(torch.int16))


@pytest.mark.parametrize("lens", [[640], [767, 300, 1025], [5000, 12]])
def test_decode_step_chain_with_metadata_ready(cuda_lib, lens):
    """Layers' fused steps launched back to back, each reading its metadata
    before waiting on the previous launch (metadata_ready, as the layers
    call it), at small batches that split rows over thread-block clusters,
    with the KvChat ring: every layer's output, cache rows and ring rows
    must equal the oracle's / the separate append's."""
    from nanokv_b200 import _lib, ops

    Hq, Hk, W, L = 16, 8, 5, 6
    B = len(lens)
    pb = make_paged_batch(seed=300 + B, lens=lens, Hq=Hq, Hk=Hk)
    bt, cl, sm = pb.block_tables.to(DEV), pb.context_lens.to(DEV), pb.slot_mapping.to(DEV)
    caches = [(pb.k_cache.to(DEV), pb.v_cache.to(DEV)) for _ in range(L)]
    steps = [_qkv(B, Hq, Hk, 310 + i) for i in range(L)]
    ring = torch.zeros(2, L, W, Hq, 128, dtype=torch.bfloat16, device=DEV)
    ring_ref = ring.clone()
    slot_of_row = torch.tensor([i % 2 for i in range(B)], dtype=torch.int32, device=DEV)
    pos_of_row = torch.tensor([(3 * i + 1) % W for i in range(B)], dtype=torch.int32, device=DEV)
    outs = [torch.empty(B, Hq, 128, dtype=torch.bfloat16, device=DEV) for _ in range(L)]
    ws = ops.decode_workspace(torch.device(DEV), B, Hq, Hk, 128, bt.size(1), 256)
    torch.cuda.synchronize()
    for layer in range(L):
        q, k, v = steps[layer]
        ops.decode_step(q, k, v, caches[layer][0], caches[layer][1], sm, bt, cl, 128 ** -0.5,
                        out=outs[layer], ring=ring, layer_id=layer, ring_slot_of_row=slot_of_row,
                        ring_pos_of_row=pos_of_row, workspace=ws, metadata_ready=True)
    torch.cuda.synchronize()
    assert _lib.read_device_error(clear=True) == 0
    active = torch.arange(B, dtype=torch.int32, device=DEV)
    for layer in range(L):
        q, k, v = steps[layer]
        ops.query_window_append(q, ring_ref, layer, active, slot_of_row, pos_of_row)
        kc, vc = pb.k_cache.clone(), pb.v_cache.clone()
        store_kvcache_ref(k.cpu(), v.cpu(), kc, vc, pb.slot_mapping)
        assert torch.equal(caches[layer][0].cpu().view(torch.int16), kc.view(torch.int16))
        assert torch.equal(caches[layer][1].cpu().view(torch.int16), vc.view(torch.int16))
        ref = paged_decode_ref(q.cpu(), kc, vc, pb.block_tables, pb.context_lens, 128 ** -0.5)
        assert (outs[layer].float().cpu() - ref).abs().max().item() <= 2e-2, f"layer {layer}"
    torch.cuda.synchronize()
    assert torch.equal(ring.view(torch.int16), ring_ref.view(torch.int16))


def test_decode_step_chain_one_item_per_cta_without_clusters(cuda_lib):
    """16 short rows x 8 kv heads: 128 (row, kv head) pairs, each one split,
    too many for thread-block clusters, so every CTA of the plain launch
    has exactly one item -- the case where a launch with metadata_ready
    requests its first K/V tile before waiting on the previous launch. Three
    layers launched back to back: outputs and cache rows equal the oracle's
    and the same steps without metadata_ready."""
    from nanokv_b200 import _lib, ops

    Hq, Hk, L = 32, 8, 3
    lens = [1 + (37 * i) % 1000 for i in range(16)]
    pb = make_paged_batch(seed=400, lens=lens, Hq=Hq, Hk=Hk)
    B = len(lens)
    bt, cl, sm = pb.block_tables.to(DEV), pb.context_lens.to(DEV), pb.slot_mapping.to(DEV)
    steps = [_qkv(B, Hq, Hk, 410 + i) for i in range(L)]
    ws = ops.decode_workspace(torch.device(DEV), B, Hq, Hk, 128, bt.size(1), 256)
    results = {}
    for ready in (True, False):
        caches = [(pb.k_cache.to(DEV), pb.v_cache.to(DEV)) for _ in range(L)]
        outs = [torch.empty(B, Hq, 128, dtype=torch.bfloat16, device=DEV) for _ in range(L)]
        torch.cuda.synchronize()
        for layer in range(L):
            q, k, v = steps[layer]
            ops.decode_step(q, k, v, caches[layer][0], caches[layer][1], sm, bt, cl, 128 ** -0.5,
                            out=outs[layer], workspace=ws, metadata_ready=ready)
        torch.cuda.synchronize()
        assert _lib.read_device_error(clear=True) == 0
        results[ready] = (caches, outs)
    for layer in range(L):
        q, k, v = steps[layer]
        kc, vc = pb.k_cache.clone(), pb.v_cache.clone()
        store_kvcache_ref(k.cpu(), v.cpu(), kc, vc, pb.slot_mapping)
        ref = paged_decode_ref(q.cpu(), kc, vc, pb.block_tables, pb.context_lens, 128 ** -0.5)
        caches, outs = results[True]
        assert torch.equal(caches[layer][0].cpu().view(torch.int16), kc.view(torch.int16))
        assert torch.equal(caches[layer][1].cpu().view(torch.int16), vc.view(torch.int16))
        assert (outs[layer].float().cpu() - ref).abs().max().item() <= 2e-2, f"layer {layer}"
        assert torch.equal(outs[layer].view(torch.int16), results[False][1][layer].view(torch.int16))
