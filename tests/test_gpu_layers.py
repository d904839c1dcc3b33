"""End-to-end GPU parity of the drop-in layers: Attention.forward(q, k, v,
Layer) driven through the Context contract for several layers and steps
(store -> periodic compression -> decode; KvChat store -> query window ->
threshold compression -> decode), against the CPU oracle pipeline."""

import types

import numpy as np
import pytest
import torch

from oracle.attention import paged_decode_ref, store_kvcache_ref
from oracle.inputs import bf16, make_paged_batch
from oracle.snapkv import snapkv_keep
from oracle.threshold_compress import QueryWindowRef, threshold_compress_ref
from oracle.window_compress import compression_events, window_compress_ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _cfg(**kw):
    base = dict(kv_compress_enabled=True, kv_compress_window_blocks=4, kv_compress_keep_blocks=2,
                kv_compress_keep_extra_tokens=1)
    base.update(kw)
    return types.SimpleNamespace(**base)


def test_attention_layers_periodic_compress_step(cuda_lib):
    from nanokv_b200.layers.attention import Attention
    from nanokv_b200.utils.context import get_context, reset_context, set_context

    L, Hq, Hk, D = 3, 32, 8, 128
    lens = [1300, 2100, 700, 1800]
    pb = make_paged_batch(seed=70, lens=lens, Hq=Hq, Hk=Hk)
    rng = np.random.default_rng(71)
    caches = [(bf16(rng.standard_normal(pb.k_cache.shape, dtype=np.float32)),
               bf16(rng.standard_normal(pb.k_cache.shape, dtype=np.float32))) for _ in range(L)]
    qkv = [bf16(rng.standard_normal((4, (Hq + 2 * Hk) * D), dtype=np.float32)) for _ in range(L)]
    selected = [0, 1, 3]

    # ---- device path through the drop-in modules
    layers = []
    for i in range(L):
        a = Attention(Hq, D, D ** -0.5, Hk, _cfg(), L)
        a.k_cache, a.v_cache = caches[i][0].to(DEV), caches[i][1].to(DEV)
        layers.append(a)
    cl = pb.context_lens.to(DEV)
    set_context(True, slot_mapping=pb.slot_mapping.to(DEV), context_lens=cl,
                block_tables=pb.block_tables.to(DEV))
    ctx = get_context()
    ctx.is_compress_step = True
    ctx.compress_selected_batch_indices = selected
    ctx.compress_base_context_lens = cl.clone()
    outs = []
    for i in range(L):
        q, k, v = qkv[i].to(DEV).split([Hq * D, Hk * D, Hk * D], dim=-1)
        o = layers[i].forward(q.view(4, Hq, D), k.view(4, Hk, D), v.view(4, Hk, D), i)
        outs.append(o)
    torch.cuda.synchronize()
    events = ctx.compression_events
    reset_context()

    # ---- oracle pipeline; each layer's kept set is taken from the device
    # result only where the oracle's own choice is within the tie band
    clc = pb.context_lens.clone()
    base = pb.context_lens.clone()
    for i in range(L):
        kc, vc = caches[i][0].clone(), caches[i][1].clone()
        q, k, v = qkv[i].split([Hq * D, Hk * D, Hk * D], dim=-1)
        q = q.reshape(4, Hq, D)
        store_kvcache_ref(k.reshape(4, Hk, D), v.reshape(4, Hk, D), kc, vc, pb.slot_mapping)
        keep_o, _ = window_compress_ref(q, kc.clone(), vc.clone(), pb.block_tables, base,
                                        clc.clone(), selected, 256, 4, 2, 1)
        # compaction with the oracle's kept set must equal the device cache
        # unless a tie-band swap happened; compare against the device bytes
        window_compress_ref(q, kc, vc, pb.block_tables, base, clc, selected, 256, 4, 2, 1,
                            keep_idx_override=keep_o)
        same = torch.equal(layers[i].k_cache.cpu().view(torch.int16), kc.view(torch.int16))
        ref = paged_decode_ref(q, kc, vc, pb.block_tables, clc, D ** -0.5)
        o = outs[i].float().cpu().view(4, Hq, D)
        if same:
            assert torch.equal(layers[i].v_cache.cpu().view(torch.int16), vc.view(torch.int16))
            assert (o - ref).abs().max().item() <= 2e-2
        else:  # a one-ulp tie at the cut: only the swapped rows may differ
            diff_rows = (layers[i].k_cache.cpu().view(-1, Hk * D).view(torch.int16)
                         != kc.view(-1, Hk * D).view(torch.int16)).any(-1).sum().item()
            assert diff_rows <= 8, f"layer {i}: {diff_rows} rows differ"
    assert cl.cpu().tolist() == clc.tolist() == [1300 - 1024 + 513, 2100 - 1024 + 513, 700,
                                                 1800 - 1024 + 513]
    assert events == compression_events(pb.block_tables, selected,
                                        torch.tensor([789, 1589, 1289]), 256, L - 1)


def test_attention_decode_only_matches_oracle(cuda_lib):
    """No compression: the layer is store + decode; output shape [B, 1, Hq, D]."""
    from nanokv_b200.layers.attention import Attention
    from nanokv_b200.utils.context import reset_context, set_context

    pb = make_paged_batch(seed=72, lens=[1, 257, 3000, 4096], Hq=16, Hk=8)
    a = Attention(16, 128, 128 ** -0.5, 8, _cfg(kv_compress_enabled=False), 1)
    a.k_cache, a.v_cache = pb.k_cache.to(DEV), pb.v_cache.to(DEV)
    set_context(True, slot_mapping=pb.slot_mapping.to(DEV), context_lens=pb.context_lens.to(DEV),
                block_tables=pb.block_tables.to(DEV))
    o = a.forward(pb.q.to(DEV), pb.k_new.to(DEV), pb.v_new.to(DEV), 0)
    torch.cuda.synchronize()
    reset_context()
    assert o.shape == (4, 1, 16, 128)
    kc, vc = pb.k_cache.clone(), pb.v_cache.clone()
    store_kvcache_ref(pb.k_new, pb.v_new, kc, vc, pb.slot_mapping)
    ref = paged_decode_ref(pb.q, kc, vc, pb.block_tables, pb.context_lens, 128 ** -0.5)
    assert (o[:, 0].float().cpu() - ref).abs().max().item() <= 2e-2


def test_kvchat_attention_threshold_cycle(cuda_lib):
    """KvChat: W decode steps append queries, the last one compresses S -> R."""
    from nanokv_b200.engine.compress_schedule import prepare_threshold_context
    from nanokv_b200.engine.query_window import QueryWindowManager
    from oracle.host_state import SeqState as Sequence
    from nanokv_b200.layers.kvchat import Attention
    from nanokv_b200.utils.context import get_context, reset_context, set_kvchat_context

    P, Hq, Hk, D, W, L = 64, 16, 8, 128, 50, 2
    S, R = P + 511, P + 257
    cfg = types.SimpleNamespace(kv_compress_enabled=True, kv_compress_N=4, kv_compress_S=511,
                                kv_compress_R=257, query_window_size=W)
    pb = make_paged_batch(seed=80, lens=[S], Hq=Hq, Hk=Hk)
    qwm = QueryWindowManager(L, W, Hq, D, device=DEV)
    layers = []
    for i in range(L):
        a = Attention(Hq, D, D ** -0.5, Hk, cfg, L)
        a.query_window_manager = qwm
        a.k_cache, a.v_cache = pb.k_cache.clone().to(DEV), pb.v_cache.clone().to(DEV)
        layers.append(a)
    seq = Sequence(list(range(P)))
    rng = np.random.default_rng(81)
    qs = bf16(rng.standard_normal((W, L, 1, Hq, D), dtype=np.float32))
    kn = bf16(rng.standard_normal((W, L, 1, Hk, D), dtype=np.float32))
    ref_qwm = QueryWindowRef(L, W, Hq, D)
    ref_caches = [(pb.k_cache.clone(), pb.v_cache.clone()) for _ in range(L)]
    bs = 256
    for step in range(W):
        length = S - W + 1 + step  # lengths S-W+1 .. S: the active window
        seq.num_tokens = length
        cl = torch.tensor([length], dtype=torch.int32)
        slot = torch.tensor([int(pb.block_tables[0, (length - 1) // bs]) * bs + (length - 1) % bs],
                            dtype=torch.int32)
        set_kvchat_context(False, slot_mapping=slot.to(DEV), context_lens=cl.to(DEV),
                           block_tables=pb.block_tables.to(DEV))
        ctx = get_context()
        prepare_threshold_context(ctx, [seq], cfg, qwm)
        if step == 0:
            ref_qwm.activate(seq.seq_id)
        for i in range(L):
            layers[i].forward(qs[step, i].to(DEV), kn[step, i].to(DEV), kn[step, i].to(DEV), i)
            store_kvcache_ref(kn[step, i], kn[step, i], ref_caches[i][0], ref_caches[i][1], slot)
            ref_qwm.append([seq.seq_id], i, qs[step, i])
            if ctx.compress_any:
                keep = threshold_compress_ref(ref_qwm.gather([seq.seq_id], i), ref_caches[i][0],
                                              ref_caches[i][1], pb.block_tables, cl, [0], S, R, W)
        torch.cuda.synchronize()
        events = ctx.compression_events
        reset_context()
    assert [e["R"] for e in events] == [R] and events[0]["keep_blocks"] == (R + 255) // 256
    assert not qwm.has(seq.seq_id)  # freed after the compressing step
    for i in range(L):
        dk = layers[i].k_cache.cpu().view(torch.int16)
        rk = ref_caches[i][0].view(torch.int16)
        ndiff = (dk.view(-1, Hk * D) != rk.view(-1, Hk * D)).any(-1).sum().item()
        assert ndiff <= 8, f"layer {i}: {ndiff} cache rows differ (beyond a tie swap)"
