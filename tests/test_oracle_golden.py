"""Pins the CPU oracle to the reference: every golden vector under
tests/golden/ was produced by the reference's own functions
(tests/golden/make_golden.py, on the CPU) or, for decode attention, by the
reference's decode kernel flash_attn_with_kvcache on a B200
(tests/golden/make_golden_flashattn.py). CPU only."""

import json

import numpy as np
import pytest
import torch

from oracle.attention import paged_decode_ref, store_kvcache_ref
from oracle.cases import SNAPKV_CASES, THRESHOLD_CASES, WINDOW_CASES, snapkv_inputs, threshold_inputs
from oracle.inputs import digest, make_paged_batch
from oracle.snapkv import snapkv_importance, snapkv_keep, tie_band_ok
from oracle.threshold_compress import QueryWindowRef, threshold_compress_ref
from oracle.window_compress import compression_events, window_compress_ref


def _npz(golden_dir, name):
    return np.load(golden_dir / name, allow_pickle=False)


def _bits_to_float(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits.astype(np.int16)).view(torch.bfloat16).float()


@pytest.mark.parametrize("case", SNAPKV_CASES, ids=[c[0] for c in SNAPKV_CASES])
def test_snapkv_matches_reference(golden_dir, case):
    name, seed, m, Hq, Hk, L, window, num_keep, outlier = case
    g = _npz(golden_dir, "snapkv.npz")
    Q, K = snapkv_inputs(seed, m, Hq, Hk, L, window, outlier)
    assert digest(Q) == str(g[f"{name}/q_digest"]), "input generator drifted"
    assert digest(K) == str(g[f"{name}/k_digest"]), "input generator drifted"
    imp = snapkv_importance(Q, K, window)
    # importance: bit-identical to the reference's bf16 key_importance
    ref_imp = torch.from_numpy(g[f"{name}/importance_bits"]).view(torch.bfloat16)
    assert torch.equal(imp.view(torch.int16), ref_imp.view(torch.int16))
    final, _ = snapkv_keep(Q, K, num_keep, window)
    ref_final = torch.from_numpy(g[f"{name}/final_idx"]).long()
    assert final.shape == ref_final.shape
    # bos and the observation window are fixed; kept sets agree up to swaps
    # inside the exact-tie group at the cut (torch.topk's tie order is unspecified)
    assert torch.equal(final[:, 0], ref_final[:, 0])
    assert torch.equal(final[:, 1 + num_keep:], ref_final[:, 1 + num_keep:])
    for i in range(m):
        ok, why = tie_band_ok(imp[i], final[i, 1:1 + num_keep], ref_final[i, 1:1 + num_keep],
                              num_keep, band=0.0)
        assert ok, why
        assert torch.all(ref_final[i, 1:1 + num_keep].diff() > 0)


@pytest.mark.parametrize("case", SNAPKV_CASES + [("config3_event",)],
                         ids=[c[0] for c in SNAPKV_CASES] + ["config3_event"])
def test_exact_score_importance_differs_only_at_cpu_rounding_keys(golden_dir, case):
    """The exact-score variant of the oracle (q.k rounded once from its exact
    value, the definition libnkv's window kernel implements) against the
    reference's computation on this CPU: on the golden cases it equals the
    reference's importance bit for bit; on config 3's 20-sequence event the
    two differ only at keys where torch's CPU bf16 matmul rounded some head's
    score differently from the exact value."""
    if case[0] == "config3_event":
        from oracle.window_compress import window_importance, window_score_rounding_keys
        lens = np.random.default_rng(33).integers(1100, 4397, 20).tolist()
        pb = make_paged_batch(seed=34, lens=lens, Hq=32, Hk=8, outlier_sigma=4.0,
                              outlier_frac=0.05)
        args = (pb.q, pb.k_cache, pb.block_tables, pb.context_lens, list(range(20)), 256, 4)
        exact = window_importance(*args, exact_scores=True)
        cpu = window_importance(*args)
        keys = window_score_rounding_keys(*args)
        differ = exact.view(torch.int16) != cpu.view(torch.int16)
        assert not bool((differ & ~keys).any())
        assert int(keys.sum()) <= 5e-3 * keys.numel()  # 38 of 20,460 keys here
        return
    name, seed, m, Hq, Hk, L, window, num_keep, outlier = case
    g = _npz(golden_dir, "snapkv.npz")
    Q, K = snapkv_inputs(seed, m, Hq, Hk, L, window, outlier)
    exact = snapkv_importance(Q, K, window, exact_scores=True)
    ref_imp = torch.from_numpy(g[f"{name}/importance_bits"]).view(torch.bfloat16)
    assert torch.equal(exact.view(torch.int16), ref_imp.view(torch.int16))


@pytest.mark.parametrize("case", WINDOW_CASES, ids=[c[0] for c in WINDOW_CASES])
def test_window_compress_matches_reference(golden_dir, case):
    name, kw, selected, wb, kb, ke = case
    g = _npz(golden_dir, "window_compress.npz")
    meta = json.loads(str(g["meta_json"]))[name]
    pb = make_paged_batch(**kw)
    assert digest(pb.k_cache) == str(g[f"{name}/k_cache_in_digest"])
    assert digest(pb.q) == str(g[f"{name}/q_digest"])
    k0, v0 = pb.k_cache.clone(), pb.v_cache.clone()
    store_kvcache_ref(pb.k_new, pb.v_new, k0, v0, pb.slot_mapping)
    assert digest(k0) == str(g[f"{name}/k_cache_stored_digest"])

    # 1. oracle selection vs the reference's (tie swaps only)
    k1, v1, cl1 = k0.clone(), v0.clone(), pb.context_lens.clone()
    keep_idx, new_lens = window_compress_ref(pb.q, k1, v1, pb.block_tables, pb.context_lens.clone(),
                                             cl1, selected, pb.block_size, wb, kb, ke)
    ref_keep = torch.from_numpy(g[f"{name}/keep_idx"]).long()
    imp = _bits_to_float(g[f"{name}/importance_bits"])
    num_keep = kb * pb.block_size + ke - 2
    for i in range(len(selected)):
        ok, why = tie_band_ok(imp[i], keep_idx[i, 1:1 + num_keep], ref_keep[i, 1:1 + num_keep],
                              num_keep, band=0.0)
        assert ok, why
    assert cl1.tolist() == g[f"{name}/context_lens_after"].tolist()
    events = compression_events(pb.block_tables, selected, new_lens, pb.block_size, 0)
    assert events == meta["events"]

    # 2. given the reference's kept set, the compacted caches are bit-exact
    k2, v2, cl2 = k0.clone(), v0.clone(), pb.context_lens.clone()
    window_compress_ref(pb.q, k2, v2, pb.block_tables, pb.context_lens.clone(), cl2, selected,
                        pb.block_size, wb, kb, ke, keep_idx_override=ref_keep)
    assert digest(k2) == str(g[f"{name}/k_cache_out_digest"])
    assert digest(v2) == str(g[f"{name}/v_cache_out_digest"])


@pytest.mark.parametrize("case", THRESHOLD_CASES, ids=[c[0] for c in THRESHOLD_CASES])
def test_threshold_compress_matches_reference(golden_dir, case):
    name, seed, P, Hq, Hk, W, S_cfg, R_cfg, L, layer = case
    g = _npz(golden_dir, "threshold.npz")
    meta = json.loads(str(g["meta_json"]))[name]
    S, R = P + S_cfg, P + R_cfg
    pb, qsteps = threshold_inputs(seed, P, Hq, Hk, W, S_cfg, L)
    assert digest(qsteps) == str(g[f"{name}/qsteps_digest"])
    qwm = QueryWindowRef(L, W, Hq, 128)
    qwm.activate(0)
    for step in range(W):
        for lyr in range(L if step < W - 1 else layer + 1):
            qwm.append([0], lyr, qsteps[step, lyr])
    q_sub = qwm.gather([0], layer)
    ref_keep = torch.from_numpy(g[f"{name}/keep_idx"]).long()
    imp = _bits_to_float(g[f"{name}/importance_bits"])
    num_keep = R - W - 1

    k1, v1, cl1 = pb.k_cache.clone(), pb.v_cache.clone(), pb.context_lens.clone()
    keep = threshold_compress_ref(q_sub, k1, v1, pb.block_tables, cl1, [0], S, R, W)
    ok, why = tie_band_ok(imp[0], keep[0, 1:1 + num_keep], ref_keep[0, 1:1 + num_keep], num_keep)
    assert ok, why
    assert cl1.tolist() == g[f"{name}/context_lens_after"].tolist()

    k2, v2, cl2 = pb.k_cache.clone(), pb.v_cache.clone(), pb.context_lens.clone()
    threshold_compress_ref(q_sub, k2, v2, pb.block_tables, cl2, [0], S, R, W,
                           keep_idx_override=ref_keep)
    assert digest(k2) == str(g[f"{name}/k_cache_out_digest"])
    assert digest(v2) == str(g[f"{name}/v_cache_out_digest"])
    ev = meta["events"]
    if layer + 1 >= L:  # events are recorded on the last layer only
        assert len(ev) == 1 and ev[0]["R"] == R and ev[0]["keep_blocks"] == (R + 255) // 256
    else:
        assert ev == []


def test_decode_oracle_small_exact():
    """The fp32 decode restatement on a hand-checkable case: one sequence of
    3 tokens, Hq == Hk == 1, against an explicit softmax."""
    torch.manual_seed(0)
    D = 128
    k_cache = torch.randn(2, 256, 1, D).to(torch.bfloat16)
    v_cache = torch.randn(2, 256, 1, D).to(torch.bfloat16)
    q = torch.randn(1, 1, D).to(torch.bfloat16)
    bt = torch.tensor([[1, 0]], dtype=torch.int32)
    out = paged_decode_ref(q, k_cache, v_cache, bt, torch.tensor([3], dtype=torch.int32), 0.1)
    K = k_cache[1, :3, 0].float()
    V = v_cache[1, :3, 0].float()
    p = torch.softmax(q[0, 0].float() @ K.T * 0.1, -1)
    assert torch.allclose(out[0, 0], p @ V, atol=1e-5)
    zero = paged_decode_ref(q, k_cache, v_cache, bt, torch.tensor([0], dtype=torch.int32), 0.1)
    assert torch.count_nonzero(zero) == 0


def test_decode_oracle_matches_flash_attn_golden(golden_dir):
    """Pins the fp32 decode restatement to the reference's own decode kernel:
    flash_attn_with_kvcache outputs recorded on a B200
    (tests/golden/make_golden_flashattn.py). flash-attn rounds its output to
    bf16, so agreement is to bf16 resolution."""
    from tests.golden.make_golden_flashattn import DECODE_CASES

    g = np.load(golden_dir / "decode_flashattn.npz")
    assert str(g["flash_attn_version"]).startswith("2.")
    for name, kw in DECODE_CASES:
        pb = make_paged_batch(**kw)
        assert digest(pb.q) == str(g[f"{name}/q_digest"])
        assert digest(pb.k_cache) == str(g[f"{name}/k_digest"])
        ref = torch.from_numpy(g[f"{name}/out_bits"]).view(torch.bfloat16).float()
        ours = paged_decode_ref(pb.q, pb.k_cache, pb.v_cache, pb.block_tables, pb.context_lens,
                                kw["D"] ** -0.5)
        err = (ours - ref).abs()
        rel = (ours - ref).norm() / ref.norm().clamp_min(1e-12)
        # flash-attn feeds bf16 probabilities to its PV product and rounds the
        # output to bf16: measured agreement is <= 1.5e-3 abs and 0.2 % rel;
        # the bounds below are 2.5x that and 5x tighter than the kernel tests'.
        assert err.max().item() <= 4e-3, f"{name}: max abs {err.max().item()}"
        assert rel.item() <= 5e-3, f"{name}: rel {rel.item()}"
        zero_rows = pb.context_lens == 0
        assert torch.count_nonzero(ref[zero_rows]) == 0  # flash-attn writes zeros for empty rows


def test_varlen_oracle_pinned_to_flash_attn(golden_dir):
    """The prefill / mixed-batch oracle (varlen_attention_ref) against
    flash_attn_varlen_func's own outputs on the seeded VARLEN_CASES, recorded
    on a B200 (tests/golden/make_golden_flashattn_varlen.py)."""
    from oracle.attention import varlen_attention_ref
    from oracle.cases import VARLEN_CASES
    from oracle.inputs import make_varlen_batch

    g = np.load(golden_dir / "prefill_flashattn.npz")
    assert str(g["flash_attn_version"]).startswith("2.")
    for name, kw in VARLEN_CASES:
        vb = make_varlen_batch(**kw)
        paged = vb.block_tables is not None
        k = vb.k_cache if paged else vb.k_new
        v = vb.v_cache if paged else vb.v_new
        assert digest(vb.q) == str(g[f"{name}/q_digest"])
        assert digest(k) == str(g[f"{name}/k_digest"])
        rows = torch.from_numpy(g[f"{name}/rows"])
        ref = torch.from_numpy(g[f"{name}/out_bits"]).view(torch.bfloat16).float()
        ours = varlen_attention_ref(vb.q, k, v, vb.cu_seqlens_q, vb.cu_seqlens_k, 128 ** -0.5,
                                    True, vb.block_tables)[rows]
        # flash-attn rounds P to bf16 for its PV product and the output to
        # bf16; early causal rows attend to few keys, so outputs reach |4|
        # where one bf16 ulp is 1.6e-2. Bound: 4e-3 plus one ulp of |ref|
        # per element, 5e-3 relative overall (measured: <= 9.4e-3 abs at
        # |ref| ~ 4, 0.22 % rel).
        err = (ours - ref).abs()
        assert bool((err <= 4e-3 + ref.abs() * 2.0 ** -8).all()), f"{name}: max abs {err.max()}"
        rel = (ours - ref).norm() / ref.norm().clamp_min(1e-12)
        assert rel.item() <= 5e-3, f"{name}: rel {rel.item()}"
        # rows that see no key are all zeros in both
        assert torch.equal((ours == 0).all(-1), (ref == 0).all(-1))


def test_norm_rope_oracle_matches_reference_modules(golden_dir):
    """oracle.norm_rope restates q/k RMSNorm + RoPE; it must reproduce the
    reference's own RMSNorm / RotaryEmbedding modules (run eagerly on the
    CPU by tests/golden/make_golden_norm_rope.py) bit for bit."""
    from oracle.cases import NORM_ROPE_CASES, norm_rope_inputs
    from oracle.norm_rope import qk_norm_rope_store_ref, rope_cache

    g = np.load(golden_dir / "norm_rope.npz")
    for name, seed, T, Hq, Hk, max_pos, base, eps in NORM_ROPE_CASES:
        qkv, pos, qw, kw, _ = norm_rope_inputs(seed, T, Hq, Hk, max_pos)
        assert digest(qkv) == str(g[f"{name}/qkv_digest"])
        cs = rope_cache(max_pos, base)
        assert digest(cs.view(torch.int32)) == str(g[f"{name}/cos_sin_digest"])
        q, k, _ = qk_norm_rope_store_ref(qkv, pos, cs, qw, kw, eps, Hq, Hk)
        assert np.array_equal(q.view(torch.int16).numpy(), g[f"{name}/q_bits"]), name
        assert np.array_equal(k.view(torch.int16).numpy(), g[f"{name}/k_bits"]), name
