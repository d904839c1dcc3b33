"""GPU parity of nkv_qk_norm_rope_store -- q/k RMSNorm + rotary embedding +
slot write in one launch, replacing nanokvllm/models/qwen3.py:109-113 and
nanokvllm/layers/attention.py:72-73 -- against the CPU oracle, which
tests/golden/norm_rope.npz pins bit for bit to the reference's own modules.

Tolerance: v rows and untouched slots bit-exact; rotated q / k within one
bf16 ulp per element with at least 99 % of elements bit-identical (the mean
of squares is summed in a different order and rsqrt is the device's, so a
value at a bf16 rounding boundary can land on the neighbouring bf16).
"""

import types

import numpy as np
import pytest
import torch

from oracle.attention import paged_decode_ref, varlen_attention_ref
from oracle.cases import NORM_ROPE_CASES, norm_rope_inputs
from oracle.inputs import make_paged_batch, make_varlen_batch
from oracle.norm_rope import qk_norm_rope_store_ref, rope_cache

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ops():
    from nanokv_b200 import ops
    return ops


def _deverr():
    from nanokv_b200 import _lib
    return _lib.read_device_error(clear=True)


def _ulp_close(ours: torch.Tensor, ref: torch.Tensor, what: str) -> None:
    a = ours.cpu().float()
    b = ref.cpu().float()
    diff = (a - b).abs()
    # one bf16 ulp of the larger magnitude (7 explicit mantissa bits)
    ulp = torch.ldexp(torch.ones_like(b), torch.frexp(torch.maximum(a.abs(), b.abs()))[1] - 8)
    assert bool((diff <= ulp).all()), f"{what}: max diff {diff.max().item()} beyond one bf16 ulp"
    exact = (a == b).float().mean().item()
    assert exact >= 0.99, f"{what}: only {exact:.4f} bit-identical"


@pytest.mark.parametrize("case", NORM_ROPE_CASES, ids=[c[0] for c in NORM_ROPE_CASES])
def test_norm_rope_store_matches_oracle(cuda_lib, case):
    ops = _ops()
    name, seed, T, Hq, Hk, max_pos, base, eps = case
    qkv, pos, qw, kw, slots = norm_rope_inputs(seed, T, Hq, Hk, max_pos)
    cs = rope_cache(max_pos, base)
    num_slots = T * 4
    sentinel = torch.full((num_slots, Hk, 128), 3.0, dtype=torch.bfloat16)
    kc_ref, vc_ref = sentinel.clone(), sentinel.clone()
    q_ref, k_ref, _ = qk_norm_rope_store_ref(qkv, pos, cs, qw, kw, eps, Hq, Hk, kc_ref, vc_ref,
                                             slots)
    kc, vc = sentinel.clone().to(DEV), sentinel.clone().to(DEV)
    k_out = torch.empty(T, Hk, 128, dtype=torch.bfloat16, device=DEV)
    q, v, k = ops.qk_norm_rope_store(qkv.to(DEV), pos.to(DEV), cs.view(max_pos, 1, 128).to(DEV),
                                     qw.to(DEV), kw.to(DEV), eps, Hq, Hk, k_cache=kc, v_cache=vc,
                                     slot_mapping=slots.to(DEV), k_out=k_out)
    torch.cuda.synchronize()
    assert _deverr() == 0
    _ulp_close(q, q_ref, f"{name} q")
    _ulp_close(k, k_ref, f"{name} k")
    # v is a copy; slots of -1 and unused slots keep the sentinel
    assert torch.equal(vc.cpu().view(torch.int16), vc_ref.view(torch.int16))
    _ulp_close(kc, kc_ref, f"{name} k cache")
    live = slots[slots >= 0].long()
    untouched = torch.ones(num_slots, dtype=torch.bool)
    untouched[live] = False
    assert torch.equal(kc.cpu()[untouched].view(torch.int16), sentinel[untouched].view(torch.int16))


def test_norm_rope_out_of_range_position_is_flagged(cuda_lib):
    from nanokv_b200 import _lib
    ops = _ops()
    qkv, pos, qw, kw, _ = norm_rope_inputs(64, 4, 16, 8, 128)
    pos[2] = 500  # outside the 128-position cache: clamped to 127 and flagged
    cs = rope_cache(128, 10000.0)
    q, _, _ = ops.qk_norm_rope_store(qkv.to(DEV), pos.to(DEV), cs.to(DEV), qw.to(DEV),
                                     kw.to(DEV), 1e-6, 16, 8)
    torch.cuda.synchronize()
    assert _deverr() & _lib.DEVERR_ROPE_POSITION
    pos_c = pos.clone()
    pos_c[2] = 127
    q_ref, _, _ = qk_norm_rope_store_ref(qkv, pos_c, cs, qw, kw, 1e-6, 16, 8)
    _ulp_close(q, q_ref, "clamped position")


def _layer_weights(seed):
    rng = np.random.default_rng(seed)
    qw = torch.from_numpy(rng.normal(1.0, 0.3, 128).astype(np.float32)).to(torch.bfloat16)
    kw = torch.from_numpy(rng.normal(1.0, 0.3, 128).astype(np.float32)).to(torch.bfloat16)
    return qw, kw


def test_attention_forward_qkv_decode_step(cuda_lib):
    """Attention.forward_qkv on a decode step (norm + RoPE + store, then the
    decode kernel) against the oracle sequence (norm, RoPE, store, decode)."""
    from nanokv_b200.layers.attention import Attention
    from nanokv_b200.utils.context import reset_context, set_context

    Hq, Hk, D = 32, 8, 128
    pb = make_paged_batch(seed=81, lens=[300, 1500, 4097, 2], Hq=Hq, Hk=Hk)
    B = 4
    rng = np.random.default_rng(82)
    qkv = torch.from_numpy(rng.standard_normal((B, (Hq + 2 * Hk) * D), dtype=np.float32)
                           ).to(torch.bfloat16)
    positions = (pb.context_lens - 1).to(torch.int64)
    cs = rope_cache(8192, 1000000.0)
    qw, kw = _layer_weights(83)
    a = Attention(Hq, D, D ** -0.5, Hk, types.SimpleNamespace(kv_compress_enabled=False), 1)
    a.k_cache, a.v_cache = pb.k_cache.clone().to(DEV), pb.v_cache.clone().to(DEV)
    set_context(True, slot_mapping=pb.slot_mapping.to(DEV), context_lens=pb.context_lens.to(DEV),
                block_tables=pb.block_tables.to(DEV))
    o = a.forward_qkv(qkv.to(DEV), positions.to(DEV), qw.to(DEV), kw.to(DEV),
                      cs.view(8192, 1, D).to(DEV), 1e-6, 0)
    torch.cuda.synchronize()
    reset_context()
    assert _deverr() == 0
    kc, vc = pb.k_cache.clone(), pb.v_cache.clone()
    q_ref, _, _ = qk_norm_rope_store_ref(qkv, positions, cs, qw, kw, 1e-6, Hq, Hk, kc, vc,
                                         pb.slot_mapping)
    ref = paged_decode_ref(q_ref, kc, vc, pb.block_tables, pb.context_lens, D ** -0.5)
    out = o[:, 0].float().cpu()
    assert (out - ref).abs().max().item() <= 2e-2
    assert ((out - ref).norm() / ref.norm()).item() <= 1e-2
    _ulp_close(a.k_cache, kc, "stored k")
    assert torch.equal(a.v_cache.cpu().view(torch.int16), vc.view(torch.int16))


def test_attention_forward_qkv_prefill_step(cuda_lib):
    """forward_qkv on a prefill step without cached prefix (keys from the
    step's rows) and on a chunk with a cached prefix (keys from the cache)."""
    from nanokv_b200.layers.attention import Attention
    from nanokv_b200.utils.context import reset_context, set_context

    Hq, Hk, D = 16, 8, 128
    cs = rope_cache(8192, 1000000.0)
    qw, kw = _layer_weights(84)
    rng = np.random.default_rng(85)
    for paged in (False, True):
        q_lens = [37, 200]
        k_lens = [37, 200] if not paged else [500, 1200]
        vb = make_varlen_batch(seed=86, q_lens=q_lens, k_lens=k_lens, Hq=Hq, Hk=Hk, paged=paged)
        T = sum(q_lens)
        qkv = torch.from_numpy(rng.standard_normal((T, (Hq + 2 * Hk) * D), dtype=np.float32)
                               ).to(torch.bfloat16)
        positions = torch.cat([torch.arange(lk - lq, lk) for lq, lk in zip(q_lens, k_lens)])
        a = Attention(Hq, D, D ** -0.5, Hk, types.SimpleNamespace(kv_compress_enabled=False), 1)
        if paged:
            a.k_cache, a.v_cache = vb.k_cache.clone().to(DEV), vb.v_cache.clone().to(DEV)
            slots, bt = vb.slot_mapping, vb.block_tables.to(DEV)
        else:
            slots, bt = torch.full((T,), -1, dtype=torch.int32), None
        set_context(False, vb.cu_seqlens_q.to(DEV), vb.cu_seqlens_k.to(DEV), vb.max_seqlen_q,
                    vb.max_seqlen_k, slots.to(DEV), None, bt)
        o = a.forward_qkv(qkv.to(DEV), positions.to(DEV), qw.to(DEV), kw.to(DEV), cs.to(DEV),
                          1e-6, 0)
        torch.cuda.synchronize()
        reset_context()
        assert _deverr() == 0
        if paged:
            kc, vc = vb.k_cache.clone(), vb.v_cache.clone()
            q_ref, _, _ = qk_norm_rope_store_ref(qkv, positions, cs, qw, kw, 1e-6, Hq, Hk, kc, vc,
                                                 vb.slot_mapping)
            ref = varlen_attention_ref(q_ref, kc, vc, vb.cu_seqlens_q, vb.cu_seqlens_k,
                                       D ** -0.5, True, vb.block_tables)
        else:
            q_ref, k_ref, v_ref = qk_norm_rope_store_ref(qkv, positions, cs, qw, kw, 1e-6, Hq, Hk)
            ref = varlen_attention_ref(q_ref, k_ref, v_ref, vb.cu_seqlens_q, vb.cu_seqlens_k,
                                       D ** -0.5, True, None)
        out = o.float().cpu()
        assert (out - ref).abs().max().item() <= 2e-2, f"paged={paged}"
        assert ((out - ref).norm() / ref.norm()).item() <= 1e-2, f"paged={paged}"


def test_kvchat_forward_qkv_decode_step_with_query_window(cuda_lib):
    """KvChat's Attention.forward_qkv on a decode step inside the query
    window (S - W < len <= S, no compression yet): q/k norm + RoPE + slot
    write in one launch, then this step's rotated queries appended to the
    window ring, then decode -- against the oracle sequence (norm, RoPE,
    store, the reference's QueryWindowManager.append, decode)."""
    from nanokv_b200.engine.compress_schedule import prepare_threshold_context
    from nanokv_b200.engine.query_window import QueryWindowManager
    from oracle.host_state import SeqState as Sequence
    from nanokv_b200.layers.kvchat import Attention as KvChatAttention
    from nanokv_b200.utils.context import get_context, reset_context, set_kvchat_context

    P, Hq, Hk, D, W = 64, 16, 8, 128, 50
    S = P + 511
    length = S - W + 5
    cfg = types.SimpleNamespace(kv_compress_enabled=True, kv_compress_N=4, kv_compress_S=511,
                                kv_compress_R=257, query_window_size=W)
    pb = make_paged_batch(seed=87, lens=[length], Hq=Hq, Hk=Hk)
    qwm = QueryWindowManager(1, W, Hq, D, device=DEV)
    a = KvChatAttention(Hq, D, D ** -0.5, Hk, cfg, 1)
    a.query_window_manager = qwm
    a.k_cache, a.v_cache = pb.k_cache.clone().to(DEV), pb.v_cache.clone().to(DEV)
    seq = Sequence(list(range(P)))
    seq.num_tokens = length
    rng = np.random.default_rng(88)
    qkv = torch.from_numpy(rng.standard_normal((1, (Hq + 2 * Hk) * D), dtype=np.float32)
                           ).to(torch.bfloat16)
    positions = torch.tensor([length - 1], dtype=torch.int64)
    cs = rope_cache(4096, 1000000.0)
    qw, kw = _layer_weights(89)
    set_kvchat_context(False, slot_mapping=pb.slot_mapping.to(DEV),
                       context_lens=pb.context_lens.to(DEV), block_tables=pb.block_tables.to(DEV))
    ctx = get_context()
    prepare_threshold_context(ctx, [seq], cfg, qwm)
    assert ctx.q_window_active_indices == [0] and not ctx.compress_any
    slot = qwm.slot_of(seq.seq_id)
    o = a.forward_qkv(qkv.to(DEV), positions.to(DEV), qw.to(DEV), kw.to(DEV), cs.to(DEV), 1e-6, 0)
    torch.cuda.synchronize()
    reset_context()
    assert _deverr() == 0
    kc, vc = pb.k_cache.clone(), pb.v_cache.clone()
    q_ref, _, _ = qk_norm_rope_store_ref(qkv, positions, cs, qw, kw, 1e-6, Hq, Hk, kc, vc,
                                         pb.slot_mapping)
    ref = paged_decode_ref(q_ref, kc, vc, pb.block_tables, pb.context_lens, D ** -0.5)
    out = o[:, 0].float().cpu()
    assert (out - ref).abs().max().item() <= 2e-2
    assert ((out - ref).norm() / ref.norm()).item() <= 1e-2
    _ulp_close(qwm.ring[slot, 0, 0].cpu(), q_ref[0], "query window row")
    assert qwm.buffers[seq.seq_id][1] == 1  # the write position moved on
    _ulp_close(a.k_cache, kc, "stored k")
    assert torch.equal(a.v_cache.cpu().view(torch.int16), vc.view(torch.int16))
