"""Periodic compression steps selected on the device and replayed from a
CUDA graph (the graph-captured compression step): nkv_window_select against
the reference's host selection rule, and a captured step replayed on two
different steps against the eager, host-selected path of the same layers
(itself checked against the oracle in test_gpu_layers.py)."""

import types

import numpy as np
import pytest
import torch

from oracle.inputs import bf16, make_paged_batch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _deverr():
    from nanokv_b200 import _lib
    return _lib.read_device_error(clear=True)


class _Seq:
    def __init__(self, seq_id, n, tail):
        self.seq_id, self._n, self.tail_uncompressed_len = seq_id, n, tail

    def __len__(self):
        return self._n


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_window_select_matches_host_rule(cuda_lib, seed):
    from nanokv_b200 import ops
    from nanokv_b200.engine.compress_schedule import PeriodicCompressScheduler

    rng = np.random.default_rng(90 + seed)
    Bsz, bs, wb, topk = 300, 256, 4, 8
    lens = rng.integers(1, 9000, size=Bsz)
    lens[rng.choice(Bsz, 20, replace=False)] = rng.integers(4, 30, 20) * bs + bs - 1  # skip rule
    tails = rng.integers(0, 2 * wb * bs, size=Bsz)
    if seed == 2:
        tails[:] = 0  # nobody eligible
    seqs = [_Seq(i, int(L), int(t)) for i, (L, t) in enumerate(zip(lens, tails))]
    sch = PeriodicCompressScheduler(types.SimpleNamespace(kv_compress_period=1, kv_compress_topk=topk,
                                                          kv_compress_window_blocks=wb), bs)
    _, sel_host, _ = sch.select(seqs)
    cl = torch.tensor(lens, dtype=torch.int32, device=DEV)
    tl = torch.tensor(tails, dtype=torch.int32, device=DEV)
    cnt = torch.zeros(1, dtype=torch.int32, device=DEV)
    base = torch.zeros(Bsz, dtype=torch.int32, device=DEV)
    sel = ops.window_select(cl, tl, bs, wb, topk, out_count=cnt, out_base_lens=base)
    torch.cuda.synchronize()
    got = [int(x) for x in sel.cpu() if int(x) >= 0]
    assert got == sel_host
    assert int(cnt.item()) == len(sel_host)
    assert torch.equal(base.cpu(), cl.cpu())


def test_compression_step_replayed_from_cuda_graph(cuda_lib):
    """Capture store + device-selected compression + decode of 3 layers once,
    replay it for two steps with different eligible rows, and compare caches,
    lengths, outputs and events with the eager host-selected path."""
    from nanokv_b200.engine.compress_schedule import PeriodicCompressScheduler
    from nanokv_b200.layers.attention import Attention
    from nanokv_b200.utils.context import Context, get_context, reset_context, set_context

    L, Hq, Hk, D, bs = 3, 32, 8, 128, 256
    wb, kb, ke, topk = 4, 2, 1, 2
    lens = [1300, 2100, 700, 1800, 1200, 2600]
    Bsz = len(lens)
    pb = make_paged_batch(seed=91, lens=lens, Hq=Hq, Hk=Hk)
    rng = np.random.default_rng(92)
    caches0 = [(bf16(rng.standard_normal(pb.k_cache.shape, dtype=np.float32)),
                bf16(rng.standard_normal(pb.k_cache.shape, dtype=np.float32))) for _ in range(L)]
    cfg = types.SimpleNamespace(kv_compress_enabled=True, kv_compress_window_blocks=wb,
                                kv_compress_keep_blocks=kb, kv_compress_keep_extra_tokens=ke,
                                kv_compress_period=1, kv_compress_topk=topk)
    sch = PeriodicCompressScheduler(cfg, bs)
    # two steps: different tails -> different selections
    step_tails = [[0, 2000, 0, 1500, 1100, 2000], [1500, 0, 0, 0, 1100, 1100]]
    step_qkv = [[bf16(rng.standard_normal((Bsz, (Hq + 2 * Hk) * D), dtype=np.float32))
                 for _ in range(L)] for _ in step_tails]

    def make_layers():
        out = []
        for i in range(L):
            a = Attention(Hq, D, D ** -0.5, Hk, cfg, L)
            a.k_cache, a.v_cache = caches0[i][0].to(DEV), caches0[i][1].to(DEV)
            out.append(a)
        return out

    # ---- eager, host-selected (reference path of the drop-in layers)
    eager = []
    for tails, qkvs in zip(step_tails, step_qkv):
        layers = make_layers()
        seqs = [_Seq(i, n, t) for i, (n, t) in enumerate(zip(lens, tails))]
        cl = pb.context_lens.to(DEV)
        set_context(True, slot_mapping=pb.slot_mapping.to(DEV), context_lens=cl,
                    block_tables=pb.block_tables.to(DEV))
        ctx = get_context()
        _, sel, ids = sch.select(seqs)
        ctx.is_compress_step, ctx.compress_selected_batch_indices = True, sel
        ctx.compress_selected_seq_ids = ids
        ctx.compress_base_context_lens = cl.clone()
        outs = []
        for i in range(L):
            q, k, v = qkvs[i].to(DEV).split([Hq * D, Hk * D, Hk * D], dim=-1)
            outs.append(layers[i].forward(q.view(Bsz, Hq, D), k.view(Bsz, Hk, D),
                                          v.view(Bsz, Hk, D), i).clone())
        torch.cuda.synchronize()
        eager.append(dict(outs=outs, lens=cl.cpu().clone(), events=list(ctx.compression_events),
                          caches=[(a.k_cache.cpu(), a.v_cache.cpu()) for a in layers]))
        reset_context()
    assert eager[0]["events"] and eager[1]["events"]
    assert [e["batch_index"] for e in eager[0]["events"]] != [e["batch_index"] for e in eager[1]["events"]]

    # ---- graph: static buffers, device selection, captured once
    layers = make_layers()
    bufs = sch.device_buffers(Bsz, DEV)
    cl = pb.context_lens.to(DEV)
    sm = pb.slot_mapping.to(DEV)
    bt = pb.block_tables.to(DEV)
    qkv_static = [torch.empty(Bsz, (Hq + 2 * Hk) * D, dtype=torch.bfloat16, device=DEV)
                  for _ in range(L)]
    out_static = []

    def run_layers():
        out_static.clear()
        for i in range(L):
            q, k, v = qkv_static[i].split([Hq * D, Hk * D, Hk * D], dim=-1)
            out_static.append(layers[i].forward(q.view(Bsz, Hq, D), k.view(Bsz, Hk, D),
                                                v.view(Bsz, Hk, D), i))

    def set_step_context(tails):
        set_context(True, slot_mapping=sm, context_lens=cl, block_tables=bt)
        seqs = [_Seq(i, n, t) for i, (n, t) in enumerate(zip(lens, tails))]
        sch.decode_step_counter = 0  # period 1: every step compresses
        assert sch.fill_context_device(get_context(), seqs, bufs)

    def reset_state(step):
        for i in range(L):
            layers[i].k_cache.copy_(caches0[i][0].to(DEV))
            layers[i].v_cache.copy_(caches0[i][1].to(DEV))
            qkv_static[i].copy_(step_qkv[step][i].to(DEV))
        cl.copy_(pb.context_lens.to(DEV))

    # warm up on a side stream, then capture
    set_step_context(step_tails[0])
    reset_state(0)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        run_layers()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    reset_state(0)
    with torch.cuda.graph(graph):
        run_layers()
    torch.cuda.synchronize()
    for step, tails in enumerate(step_tails):
        set_step_context(tails)  # uploads this step's tail counters into the static buffer
        reset_state(step)
        torch.cuda.synchronize()
        graph.replay()
        torch.cuda.synchronize()
        assert _deverr() == 0
        ref = eager[step]
        events = sch.events_from_device(bufs["selected_host"].tolist(), pb.context_lens.tolist(),
                                        pb.block_tables.tolist(), kb, ke, L)
        assert events == ref["events"], f"step {step}"
        assert torch.equal(cl.cpu(), ref["lens"])
        for i in range(L):
            assert torch.equal(out_static[i].cpu().view(torch.int16),
                               ref["outs"][i].cpu().view(torch.int16)), f"step {step} layer {i}"
            assert torch.equal(layers[i].k_cache.cpu().view(torch.int16),
                               ref["caches"][i][0].view(torch.int16))
            assert torch.equal(layers[i].v_cache.cpu().view(torch.int16),
                               ref["caches"][i][1].view(torch.int16))
    del graph
    reset_context()
