"""Generates the golden vectors under tests/golden/ by running the REFERENCE's
own Python functions (nano-kvllm, imported from a read-only checkout) on the
CPU. Run from the repo root:

    python tests/golden/make_golden.py /path/to/nanokv-llm

What is recorded (inputs are regenerated from seeds by oracle/inputs.py, so
only their sha256 digests are stored):

  snapkv.npz          reference SnapKV (nanokvllm/layers/CompressMethod.py) on
                      seeded Q/K: its bf16 key_importance (captured at its
                      torch.topk call) and final_idx, for several shapes.
  window_compress.npz reference MyCompressCompact (nanokvllm/layers/compress_utils.py)
                      on BASELINE config 1 and a GQA-4 multi-sequence case:
                      kept indices, new context_lens, events, cache digests.
  threshold.npz       reference KvChat MyCompressCompact + QueryWindowManager
                      (KvChat/layers/compress_utils.py, KvChat/engine/query_window_manager.py).
                      The Triton gather TritonGetKVForComp cannot run on a CPU;
                      it is replaced by oracle.threshold_compress.gather_first_positions,
                      a torch restatement of the same gather.
  host_metadata.json  reference BlockManager / Scheduler.postprocess traces,
                      ModelRunner.prepare_decode periodic selection, and KvChat
                      prepare_compression_context decisions.
  step_metadata.json  reference ModelRunner.prepare_step (the unified
                      scheduler's per-step metadata) on mixed prefill-chunk +
                      decode batches, an all-decode batch and a single prefill.

The store that precedes compression is the reference's Triton kernel (CUDA
only); the script applies it with oracle.attention.store_kvcache_ref, which
is a plain indexed copy.
"""

from __future__ import annotations

import json
import os
import sys
import types
from collections import deque
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))

from oracle.attention import store_kvcache_ref  # noqa: E402
from oracle.cases import SNAPKV_CASES, THRESHOLD_CASES, WINDOW_CASES, snapkv_inputs, threshold_inputs  # noqa: E402
from oracle.inputs import digest, make_paged_batch  # noqa: E402
from oracle.threshold_compress import gather_first_positions  # noqa: E402

OUT = Path(__file__).resolve().parent


class _Recorder:
    """Wraps torch.topk / SnapKV to capture what the reference computes."""

    def __init__(self):
        self.topk_inputs = []
        self.snapkv_outputs = []


def _patched_topk(rec: _Recorder):
    real = torch.topk

    def topk(input, *args, **kwargs):
        rec.topk_inputs.append(input.detach().clone())
        return real(input, *args, **kwargs)

    return real, topk


# ------------------------------------------------------------------ SnapKV
def gen_snapkv(ref):
    from nanokvllm.layers.CompressMethod import SnapKV
    out = {}
    for name, seed, m, Hq, Hk, L, window, num_keep, outlier in SNAPKV_CASES:
        Q, K = snapkv_inputs(seed, m, Hq, Hk, L, window, outlier)
        rec = _Recorder()
        real, fake = _patched_topk(rec)
        torch.topk = fake
        try:
            final = SnapKV(Q, K, K, num_keep=num_keep, window=window)
        finally:
            torch.topk = real
        imp = rec.topk_inputs[0].view(m, -1)
        out[f"{name}/importance_bits"] = imp.view(torch.int16).numpy()
        out[f"{name}/final_idx"] = final.numpy().astype(np.int32)
        out[f"{name}/q_digest"] = np.array(digest(Q))
        out[f"{name}/k_digest"] = np.array(digest(K))
    np.savez_compressed(OUT / "snapkv.npz", **out)
    print("snapkv.npz:", len(SNAPKV_CASES), "cases")


# ------------------------------------------------------------------ window compression
def gen_window(ref):
    import nanokvllm.layers.compress_utils as cu
    from nanokvllm.utils.context import Context
    out, meta = {}, {}
    for name, kw, selected, wb, kb, ke in WINDOW_CASES:
        pb = make_paged_batch(**kw)
        out[f"{name}/k_cache_in_digest"] = np.array(digest(pb.k_cache))
        out[f"{name}/v_cache_in_digest"] = np.array(digest(pb.v_cache))
        out[f"{name}/q_digest"] = np.array(digest(pb.q))
        k_cache, v_cache = pb.k_cache.clone(), pb.v_cache.clone()
        store_kvcache_ref(pb.k_new, pb.v_new, k_cache, v_cache, pb.slot_mapping)
        out[f"{name}/k_cache_stored_digest"] = np.array(digest(k_cache))
        ctx = Context(use_decode_kernel=True, context_lens=pb.context_lens.clone(),
                      block_tables=pb.block_tables.clone(), compression_events=[],
                      is_compress_step=True, compress_selected_batch_indices=list(selected),
                      compress_base_context_lens=pb.context_lens.clone())
        rec = _Recorder()
        real_snap = cu.SnapKV

        def snap(*a, **k):
            r = real_snap(*a, **k)
            rec.snapkv_outputs.append(r.clone())
            return r

        real, fake = _patched_topk(rec)
        cu.SnapKV, torch.topk = snap, fake
        try:
            ok = cu.MyCompressCompact(pb.q, k_cache, v_cache, layer_id=0, block_size=pb.block_size,
                                      window_blocks=wb, keep_blocks=kb, keep_extra_tokens=ke,
                                      num_layers=1, context=ctx)
        finally:
            cu.SnapKV, torch.topk = real_snap, real
        assert ok is True
        out[f"{name}/keep_idx"] = rec.snapkv_outputs[0].numpy().astype(np.int32)
        out[f"{name}/importance_bits"] = rec.topk_inputs[0].view(len(selected), -1).view(torch.int16).numpy()
        out[f"{name}/context_lens_after"] = ctx.context_lens.numpy()
        out[f"{name}/k_cache_out_digest"] = np.array(digest(k_cache))
        out[f"{name}/v_cache_out_digest"] = np.array(digest(v_cache))
        meta[name] = {"selected": list(selected), "window_blocks": wb, "keep_blocks": kb,
                      "keep_extra_tokens": ke, "events": ctx.compression_events}
    out["meta_json"] = np.array(json.dumps(meta))
    np.savez_compressed(OUT / "window_compress.npz", **out)
    print("window_compress.npz:", list(meta))


# ------------------------------------------------------------------ KvChat threshold
def gen_threshold(ref):
    import KvChat.layers.compress_utils as kcu
    from KvChat.engine.query_window_manager import QueryWindowManager
    from KvChat.utils.context import Context
    out, meta = {}, {}
    for name, seed, P, Hq, Hk, W, S_cfg, R_cfg, L, layer in THRESHOLD_CASES:
        S, R = P + S_cfg, P + R_cfg
        pb, qsteps = threshold_inputs(seed, P, Hq, Hk, W, S_cfg, L)
        out[f"{name}/qsteps_digest"] = np.array(digest(qsteps))
        k_cache, v_cache = pb.k_cache.clone(), pb.v_cache.clone()
        qwm = QueryWindowManager(num_layers=L, window_size=W, num_heads=Hq, head_dim=128,
                                 device="cpu", dtype=torch.bfloat16)
        seq_id = 0
        qwm.activate(seq_id)
        for step in range(W):
            # the last step's append of the compressing layer precedes compression
            upto = L if step < W - 1 else layer + 1
            for l in range(upto):
                qwm.append([seq_id], l, qsteps[step, l])
        ctx = Context(is_prefill=False, context_lens=pb.context_lens.clone(),
                      block_tables=pb.block_tables.clone(), slot_mapping=pb.slot_mapping.clone(),
                      compression_events=[], compress_need_mask=[True], compress_any=True,
                      seq_ids=[seq_id], q_window_active_indices=[0], q_window_active_seq_ids=[seq_id],
                      runtime_compress_S=S, runtime_compress_R=R)
        rec = _Recorder()
        real_snap, real_gather = kcu.SnapKV, kcu.TritonGetKVForComp

        def snap(*a, **k):
            r = real_snap(*a, **k)
            rec.snapkv_outputs.append(r.clone())
            return r

        def gather(k_cache, v_cache, block_tables, seq_idxs, S, chunk_size=128):
            return gather_first_positions(k_cache, v_cache, block_tables, seq_idxs.tolist(), S)

        real, fake = _patched_topk(rec)
        kcu.SnapKV, kcu.TritonGetKVForComp, torch.topk = snap, gather, fake
        try:
            ok = kcu.MyCompressCompact(qwm, k_cache, v_cache, layer_id=layer, block_size=256, S=S,
                                       R=R, query_window_size=W, num_layers=L, context=ctx)
        finally:
            kcu.SnapKV, kcu.TritonGetKVForComp, torch.topk = real_snap, real_gather, real
        assert ok is True
        out[f"{name}/keep_idx"] = rec.snapkv_outputs[0].numpy().astype(np.int32)
        out[f"{name}/importance_bits"] = rec.topk_inputs[0].view(1, -1).view(torch.int16).numpy()
        out[f"{name}/context_lens_after"] = ctx.context_lens.numpy()
        out[f"{name}/k_cache_out_digest"] = np.array(digest(k_cache))
        out[f"{name}/v_cache_out_digest"] = np.array(digest(v_cache))
        meta[name] = {"prompt": P, "S": S, "R": R, "W": W, "num_layers": L, "layer": layer,
                      "Hq": Hq, "Hk": Hk, "events": ctx.compression_events}
    out["meta_json"] = np.array(json.dumps(meta))
    np.savez_compressed(OUT / "threshold.npz", **out)
    print("threshold.npz:", list(meta))


# ------------------------------------------------------------------ host metadata
class _TorchNoPin(types.ModuleType):
    """torch proxy whose tensor() ignores pin_memory (CPU-only host)."""

    def __init__(self):
        super().__init__("torch_nopin")

    def __getattr__(self, name):
        return getattr(torch, name)

    @staticmethod
    def tensor(*a, **k):
        k.pop("pin_memory", None)
        return torch.tensor(*a, **k)


def _seq_state(seq):
    return {"seq_id": seq.seq_id, "num_tokens": seq.num_tokens, "block_table": list(seq.block_table),
            "num_cached_tokens": seq.num_cached_tokens,
            "tail_uncompressed_len": getattr(seq, "tail_uncompressed_len", None),
            "rope_pos": getattr(seq, "rope_pos", None)}


def _bm_state(bm):
    return {"free": list(bm.free_block_ids), "used": sorted(bm.used_block_ids),
            "ref": [b.ref_count for b in bm.blocks], "hash_set": [b.hash != -1 for b in bm.blocks]}


def gen_host(ref):
    from nanokvllm.engine.block_manager import BlockManager
    from nanokvllm.engine.model_runner import ModelRunner
    import nanokvllm.engine.model_runner as mr
    from nanokvllm.engine.scheduler import Scheduler
    from nanokvllm.engine.sequence import ScheduledSeq, Sequence
    from nanokvllm.sampling_params import SamplingParams
    from nanokvllm.utils.context import get_context
    trace = {}

    # --- BlockManager + Scheduler.postprocess with compression events
    rng = np.random.default_rng(5)
    Sequence.counter = iter(range(10**6))
    bm = BlockManager(num_blocks=40, block_size=256)
    shared = rng.integers(0, 50000, 512).tolist()
    prompts = [shared + rng.integers(0, 50000, 300).tolist(),
               shared + rng.integers(0, 50000, 40).tolist(),
               rng.integers(0, 50000, 1100).tolist(),
               rng.integers(0, 50000, 255).tolist()]
    sp = SamplingParams(max_tokens=10**6, ignore_eos=True)
    seqs = [Sequence(p, sp) for p in prompts]
    steps = []
    for s in seqs:
        bm.allocate(s)
        s.num_computed_tokens = s.num_prompt_tokens
    steps.append({"op": "allocate", "seqs": [_seq_state(s) for s in seqs], "bm": _bm_state(bm)})
    sched = Scheduler.__new__(Scheduler)
    sched.block_manager, sched.eos, sched.running = bm, -1, deque(seqs)
    for step in range(300):
        for s in seqs:
            bm.may_append(s)
        token_ids = rng.integers(0, 50000, len(seqs)).tolist()
        events = None
        if step in (120, 260):
            # events shaped exactly like compress_utils.py:280-288 for seqs 0 and 2
            events = []
            for bi in (0, 2):
                s = seqs[bi]
                new_len = len(s) - 1024 + 513
                kb = (new_len + 255) // 256
                events.append({"batch_index": bi, "layer": 0, "new_context_len": new_len,
                               "keep_blocks": kb,
                               "freed_block_ids": [x for x in s.block_table[kb:] if x >= 0],
                               "tail_uncompressed_len_after": 0})
            events.append(dict(events[0]))  # duplicate: postprocess keeps the last per seq
        sched.postprocess([ScheduledSeq(s, 1) for s in seqs], token_ids, events)
        if events or step % 50 == 0:
            steps.append({"op": f"step{step}", "events": events, "token_ids": token_ids,
                          "seqs": [_seq_state(s) for s in seqs], "bm": _bm_state(bm)})
    trace["block_manager"] = {"prompts": prompts, "steps": steps}

    # --- then release and reuse: can_append, deallocate (shared prefix
    # blocks), can_allocate / allocate of a new prompt sharing the prefix
    rel = [{"op": "can_append", "value": [bm.can_append(s) for s in seqs]}]
    bm.deallocate(seqs[1])
    rel.append({"op": "deallocate1", "seqs": [_seq_state(s) for s in seqs], "bm": _bm_state(bm)})
    new_prompt = shared + rng.integers(0, 50000, 700).tolist()
    new = Sequence(new_prompt, sp)
    rel.append({"op": "can_allocate", "value": bm.can_allocate(new)})
    bm.allocate(new)
    rel.append({"op": "allocate_new", "seq": _seq_state(new), "bm": _bm_state(bm)})
    bm.deallocate(seqs[3])
    bm.deallocate(new)
    rel.append({"op": "deallocate3_new", "seqs": [_seq_state(s) for s in seqs],
                "new": _seq_state(new), "bm": _bm_state(bm)})
    trace["block_manager_release"] = {"new_prompt": new_prompt, "steps": rel}

    # --- periodic selection: ModelRunner.prepare_decode (model_runner.py:265-333)
    cfg = types.SimpleNamespace(kv_compress_window_blocks=4, kv_compress_topk=2,
                                kv_compress_period=3)
    stub = types.SimpleNamespace(block_size=256, kv_compress_enabled=True, decode_step_counter=0,
                                 config=cfg)
    stub.prepare_block_tables = lambda seqs: ModelRunner.prepare_block_tables(stub, seqs)
    Sequence.counter = iter(range(10**6))
    lens = [1200, 1279, 1535, 2000, 800, 1790, 3000]
    tails = [1100, 1024, 1500, 1023, 900, 1200, 1024]
    sel_seqs = []
    for L, t in zip(lens, tails):
        s = Sequence(list(range(L)), sp)
        s.block_table = list(range(100, 100 + (L + 255) // 256))
        s.tail_uncompressed_len = t
        s.rope_pos = L + 17
        sel_seqs.append(s)
    real_cuda = torch.Tensor.cuda
    torch.Tensor.cuda = lambda self, *a, **k: self
    mr_torch = mr.torch
    mr.torch = _TorchNoPin()
    picks = []
    try:
        for step in range(7):
            ids, pos = ModelRunner.prepare_decode(stub, sel_seqs)
            ctx = get_context()
            picks.append({"step": step + 1, "is_compress_step": ctx.is_compress_step,
                          "selected": ctx.compress_selected_batch_indices,
                          "seq_ids": ctx.compress_selected_seq_ids,
                          "base_lens": None if ctx.compress_base_context_lens is None
                          else ctx.compress_base_context_lens.tolist(),
                          "positions": pos.tolist(), "slot_mapping": ctx.slot_mapping.tolist(),
                          "context_lens": ctx.context_lens.tolist()})
            for s in sel_seqs:  # grow by one token between steps
                s.append_token(1)
    finally:
        torch.Tensor.cuda = real_cuda
        mr.torch = mr_torch
    trace["periodic_selection"] = {"lens": lens, "tails": tails, "period": 3, "topk": 2,
                                   "steps": picks}

    # --- KvChat prepare_compression_context (KvChat/engine/model_runner.py:304-339)
    from KvChat.engine.model_runner import ModelRunner as KModelRunner
    from KvChat.engine.query_window_manager import QueryWindowManager
    from KvChat.engine.sequence import Sequence as KSequence
    from KvChat.utils.context import get_context as kget, set_context as kset
    kcfg = types.SimpleNamespace(kv_compress_S=511, kv_compress_R=257, query_window_size=50)
    qwm = QueryWindowManager(1, 50, 2, 128, device="cpu", dtype=torch.bfloat16)
    kstub = types.SimpleNamespace(config=kcfg, query_window_manager=qwm)
    KSequence.counter = iter(range(10**6))
    kseqs = [KSequence(list(range(p))) for p in (100, 100, 40)]
    decisions = []
    for L_extra in (450, 461, 462, 500, 511, 512):
        for s in kseqs:
            s.num_tokens = s.num_prompt_tokens + L_extra
        kset(False)
        KModelRunner.prepare_compression_context(kstub, kseqs)
        c = kget()
        decisions.append({"extra": L_extra, "need": c.compress_need_mask, "any": c.compress_any,
                          "active": c.q_window_active_indices, "S": c.runtime_compress_S,
                          "R": c.runtime_compress_R, "has": [qwm.has(s.seq_id) for s in kseqs]})
    trace["kvchat_context"] = {"prompts": [100, 100, 40], "decisions": decisions}
    (OUT / "host_metadata.json").write_text(json.dumps(trace))
    print("host_metadata.json written")


def gen_step(ref):
    """The unified scheduler's per-step metadata: ModelRunner.prepare_step
    (nanokvllm/engine/model_runner.py:160-219) on mixed prefill-chunk +
    decode batches, an all-decode batch and a single prefill, run on the CPU
    (tensor uploads stubbed out as in gen_host)."""
    from nanokvllm.engine.model_runner import ModelRunner
    import nanokvllm.engine.model_runner as mr
    from nanokvllm.engine.sequence import ScheduledSeq, Sequence
    from nanokvllm.sampling_params import SamplingParams
    from nanokvllm.utils.context import get_context, reset_context
    rng = np.random.default_rng(17)
    sp = SamplingParams(max_tokens=10**6, ignore_eos=True)
    Sequence.counter = iter(range(10**6))
    stub = types.SimpleNamespace(block_size=256)
    stub.prepare_block_tables = lambda seqs: ModelRunner.prepare_block_tables(stub, seqs)
    pool = rng.permutation(4096).tolist()

    def make(prompt_len, computed, generated=0):
        s = Sequence(rng.integers(0, 100, prompt_len).tolist(), sp)  # small ids: small file
        for t in rng.integers(0, 100, generated).tolist():
            s.append_token(int(t))
        s.num_computed_tokens = computed
        nb = (len(s) + 255) // 256
        s.block_table = [pool.pop() for _ in range(nb)]
        return s

    batches = []
    # mixed: decode rows, a first chunk, a middle chunk, a one-token last chunk
    d0, d1 = make(300, 304, 5), make(1800, 1800 + 40, 41)
    c0, c1, c2 = make(5000, 0), make(5000, 2048), make(2049, 2048)
    batches.append(("mixed", [ScheduledSeq(d0, 1), ScheduledSeq(c0, 2048), ScheduledSeq(d1, 1),
                              ScheduledSeq(c1, 1000), ScheduledSeq(c2, 1)], False))
    dec = [make(int(n), int(n) + 7, 8) for n in rng.integers(200, 3000, 6)]
    batches.append(("all_decode", [ScheduledSeq(s, 1) for s in dec], True))
    batches.append(("single_prefill", [ScheduledSeq(make(300, 0), 300)], False))
    real_cuda = torch.Tensor.cuda
    torch.Tensor.cuda = lambda self, *a, **k: self
    mr_torch = mr.torch
    mr.torch = _TorchNoPin()
    out = []
    try:
        for name, sched, all_decode in batches:
            ids, pos, logits_idx = ModelRunner.prepare_step(stub, sched, all_decode)
            c = get_context()
            t = lambda x: None if x is None else x.tolist()
            out.append({"name": name, "all_decode": all_decode,
                        "seqs": [{"token_ids": list(s.seq.token_ids),
                                  "num_computed_tokens": s.seq.num_computed_tokens,
                                  "block_table": list(s.seq.block_table),
                                  "num_new_tokens": s.num_new_tokens} for s in sched],
                        "input_ids": ids.tolist(), "positions": pos.tolist(),
                        "logits_indices": logits_idx.tolist(),
                        "use_decode_kernel": c.use_decode_kernel,
                        "cu_seqlens_q": t(c.cu_seqlens_q), "cu_seqlens_k": t(c.cu_seqlens_k),
                        "max_seqlen_q": c.max_seqlen_q, "max_seqlen_k": c.max_seqlen_k,
                        "slot_mapping": t(c.slot_mapping), "context_lens": t(c.context_lens),
                        "block_tables": t(c.block_tables)})
            reset_context()
    finally:
        torch.Tensor.cuda = real_cuda
        mr.torch = mr_torch
    (OUT / "step_metadata.json").write_text(json.dumps({"block_size": 256, "batches": out}))
    print("step_metadata.json written")


def main():
    arg = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("NANOKV_REFERENCE")
    if not arg:
        raise SystemExit(f"usage: python {Path(__file__).name} /path/to/nanokv-llm checkout "
                         "(or set NANOKV_REFERENCE)")
    ref = Path(arg).resolve()
    sys.path.insert(0, str(ref))
    torch.set_num_threads(8)
    gen_snapkv(ref)
    gen_window(ref)
    gen_threshold(ref)
    gen_host(ref)
    gen_step(ref)


if __name__ == "__main__":
    main()
