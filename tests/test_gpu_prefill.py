"""GPU parity of nkv_paged_prefill -- the replacement of the reference's
flash_attn_varlen_func call for prefill and chunked-prefill mixed batches
(nanokvllm/layers/attention.py:96-102) -- against the fp32 CPU oracle
(pinned to flash-attn's outputs by tests/golden/prefill_flashattn.npz) and,
at sizes the oracle would take minutes for, against flash-attn itself on the
same device. Every call goes through the C ABI via nanokv_b200.ops.

Tolerance (bf16 outputs vs fp32): max-abs 2e-2 and relative (Frobenius) 1e-2.
"""

import types

import numpy as np
import pytest
import torch

from oracle.attention import store_kvcache_ref, varlen_attention_ref
from oracle.cases import VARLEN_CASES
from oracle.inputs import bf16, make_varlen_batch

pytestmark = pytest.mark.gpu

DEV = "cuda"
ATOL = 2e-2
RTOL = 1e-2


def _ops():
    from nanokv_b200 import ops
    return ops


def _deverr():
    from nanokv_b200 import _lib
    return _lib.read_device_error(clear=True)


def _close(ours: torch.Tensor, ref: torch.Tensor, what: str) -> None:
    ours = ours.float().cpu()
    ref = ref.float().cpu()
    err = (ours - ref).abs().max().item() if ref.numel() else 0.0
    rel = ((ours - ref).norm() / ref.norm().clamp_min(1e-12)).item() if ref.numel() else 0.0
    assert err <= ATOL, f"{what}: max abs {err}"
    assert rel <= RTOL, f"{what}: rel {rel}"


def _kv(vb):
    paged = vb.block_tables is not None
    return (vb.k_cache, vb.v_cache) if paged else (vb.k_new, vb.v_new)


def _device_run(vb, causal=True, scale=128 ** -0.5):
    ops = _ops()
    k, v = _kv(vb)
    bt = vb.block_tables.to(DEV) if vb.block_tables is not None else None
    return ops.flash_attn_varlen_func(vb.q.to(DEV), k.to(DEV), v.to(DEV),
                                      cu_seqlens_q=vb.cu_seqlens_q.to(DEV),
                                      cu_seqlens_k=vb.cu_seqlens_k.to(DEV),
                                      max_seqlen_q=vb.max_seqlen_q, max_seqlen_k=vb.max_seqlen_k,
                                      softmax_scale=scale, causal=causal, block_table=bt)


@pytest.mark.parametrize("case", VARLEN_CASES, ids=[c[0] for c in VARLEN_CASES])
def test_prefill_matches_oracle(cuda_lib, case):
    name, kw = case
    vb = make_varlen_batch(**kw)
    out = _device_run(vb)
    torch.cuda.synchronize()
    assert _deverr() == 0
    k, v = _kv(vb)
    ref = varlen_attention_ref(vb.q, k, v, vb.cu_seqlens_q, vb.cu_seqlens_k, 128 ** -0.5, True,
                               vb.block_tables)
    _close(out, ref, name)
    assert torch.isfinite(out.float()).all()


def test_prefill_non_causal(cuda_lib):
    vb = make_varlen_batch(seed=51, q_lens=[100, 7], k_lens=[600, 300], Hq=32, Hk=8)
    out = _device_run(vb, causal=False, scale=0.07)
    torch.cuda.synchronize()
    assert _deverr() == 0
    ref = varlen_attention_ref(vb.q, vb.k_cache, vb.v_cache, vb.cu_seqlens_q, vb.cu_seqlens_k,
                               0.07, False, vb.block_tables)
    _close(out, ref, "non-causal")


def test_prefill_block_size_64(cuda_lib):
    vb = make_varlen_batch(seed=52, q_lens=[65, 200, 1], k_lens=[65, 333, 130], Hq=16, Hk=4,
                           block_size=64)
    out = _device_run(vb)
    torch.cuda.synchronize()
    assert _deverr() == 0
    ref = varlen_attention_ref(vb.q, vb.k_cache, vb.v_cache, vb.cu_seqlens_q, vb.cu_seqlens_k,
                               128 ** -0.5, True, vb.block_tables)
    _close(out, ref, "block 64")


def test_prefill_strided_qkv_rows(cuda_lib):
    """q/k/v as views into one fused qkv projection, as the model passes them
    when no prefix is cached (block_table None)."""
    ops = _ops()
    Hq, Hk, D = 32, 8, 128
    lens = [37, 512, 129]
    T = sum(lens)
    rng = np.random.default_rng(53)
    qkv = bf16(rng.standard_normal((T, (Hq + 2 * Hk) * D), dtype=np.float32)).to(DEV)
    q, k, v = qkv.split([Hq * D, Hk * D, Hk * D], dim=-1)
    q, k, v = q.view(T, Hq, D), k.view(T, Hk, D), v.view(T, Hk, D)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32)
    out = ops.flash_attn_varlen_func(q, k, v, cu.to(DEV), cu.to(DEV), max(lens), max(lens),
                                     softmax_scale=D ** -0.5, causal=True)
    torch.cuda.synchronize()
    assert _deverr() == 0
    ref = varlen_attention_ref(q.cpu(), k.cpu(), v.cpu(), cu, cu, D ** -0.5, True, None)
    _close(out, ref, "strided qkv")


def test_prefill_queries_longer_than_keys(cuda_lib):
    """Lq > Lk: with the bottom-right causal mask the first Lq - Lk queries
    see no key and are zeros (flash-attn's convention); Lk == 0 likewise."""
    ops = _ops()
    Hq, Hk, D = 16, 8, 128
    q_lens, k_lens = [10, 300, 4], [4, 100, 0]
    rng = np.random.default_rng(54)
    q = bf16(rng.standard_normal((sum(q_lens), Hq, D), dtype=np.float32))
    k = bf16(rng.standard_normal((sum(k_lens), Hk, D), dtype=np.float32))
    v = bf16(rng.standard_normal((sum(k_lens), Hk, D), dtype=np.float32))
    cq = torch.tensor(np.concatenate([[0], np.cumsum(q_lens)]), dtype=torch.int32)
    ck = torch.tensor(np.concatenate([[0], np.cumsum(k_lens)]), dtype=torch.int32)
    out = ops.flash_attn_varlen_func(q.to(DEV), k.to(DEV), v.to(DEV), cq.to(DEV), ck.to(DEV),
                                     max(q_lens), max(k_lens), softmax_scale=D ** -0.5, causal=True)
    torch.cuda.synchronize()
    assert _deverr() == 0
    ref = varlen_attention_ref(q, k, v, cq, ck, D ** -0.5, True, None)
    _close(out, ref, "Lq > Lk")
    o = out.cpu().float()
    assert torch.count_nonzero(o[0:6]) == 0 and torch.count_nonzero(o[10:210]) == 0
    assert torch.count_nonzero(o[310:314]) == 0


def test_prefill_bad_metadata_is_flagged_not_written(cuda_lib):
    """max_seqlen_q below a sequence's Lq, or cu_seqlens_q past the query
    rows: the kernel skips those sequences and sets NKV_DEVERR_PREFILL_RANGE;
    the other sequences are still computed."""
    from nanokv_b200 import _lib
    ops = _ops()
    vb = make_varlen_batch(seed=55, q_lens=[300, 20], k_lens=[300, 20], Hq=16, Hk=8, paged=False)
    out = torch.full((320, 16, 128), 7.0, dtype=torch.bfloat16, device=DEV)
    ops.paged_prefill(vb.q.to(DEV), vb.k_new.to(DEV), vb.v_new.to(DEV), vb.cu_seqlens_q.to(DEV),
                      vb.cu_seqlens_k.to(DEV), 64, 128 ** -0.5, out=out)
    torch.cuda.synchronize()
    assert _deverr() & _lib.DEVERR_PREFILL_RANGE
    assert (out[:300].float() == 7.0).all()  # sequence 0 (Lq 300 > 64) untouched
    ref = varlen_attention_ref(vb.q, vb.k_new, vb.v_new, vb.cu_seqlens_q, vb.cu_seqlens_k,
                               128 ** -0.5, True, None)
    _close(out[300:], ref[300:], "sequence 1")
    bad_cu = torch.tensor([0, 300, 400], dtype=torch.int32, device=DEV)  # 400 > 320 rows
    out2 = torch.full_like(out, 7.0)
    ops.paged_prefill(vb.q.to(DEV), vb.k_new.to(DEV), vb.v_new.to(DEV), bad_cu,
                      bad_cu, 300, 128 ** -0.5, out=out2)
    torch.cuda.synchronize()
    assert _deverr() & _lib.DEVERR_PREFILL_RANGE
    assert (out2[300:].float() == 7.0).all()
    _close(out2[:300], ref[:300], "sequence 0")


def _flash_attn():
    try:
        from flash_attn import flash_attn_varlen_func
    except Exception:  # pragma: no cover - flash-attn is in the image
        pytest.skip("flash-attn not importable")
    return flash_attn_varlen_func


@pytest.mark.parametrize("hq,hk,paged", [(32, 8, True), (64, 8, True), (32, 8, False),
                                         (16, 16, True)])
def test_prefill_matches_flash_attn_full_size(cuda_lib, hq, hk, paged):
    """Chunked prefill of 8 sequences (2048-token chunks over up to 8k of
    cached prefix) and mixed decode rows, compared with the reference's own
    kernel on the same device and inputs."""
    fa = _flash_attn()
    ops = _ops()
    D, bs = 128, 256
    rng = np.random.default_rng(56 + hq + hk + int(paged))
    if paged:
        q_lens = [2048, 2048, 1, 1, 2048, 977, 1, 2048]
        k_lens = [2048, 8192, 5000, 1, 4096, 977, 7000, 6144]
    else:
        q_lens = k_lens = [2048, 1, 4096, 333, 2048, 1500, 64, 3000]
    vb = make_varlen_batch(seed=int(rng.integers(1 << 30)), q_lens=q_lens, k_lens=k_lens,
                           Hq=hq, Hk=hk, block_size=bs, paged=paged)
    k, v = _kv(vb)
    args = (vb.q.to(DEV), k.to(DEV), v.to(DEV))
    kw = dict(cu_seqlens_q=vb.cu_seqlens_q.to(DEV), cu_seqlens_k=vb.cu_seqlens_k.to(DEV),
              max_seqlen_q=vb.max_seqlen_q, max_seqlen_k=vb.max_seqlen_k,
              softmax_scale=D ** -0.5, causal=True,
              block_table=vb.block_tables.to(DEV) if paged else None)
    ours = ops.flash_attn_varlen_func(*args, **kw)
    ref = fa(*args, **kw)
    torch.cuda.synchronize()
    assert _deverr() == 0
    _close(ours, ref, f"vs flash-attn hq{hq} hk{hk} paged={paged}")


def test_attention_layer_prefill_step(cuda_lib):
    """Attention.forward on a mixed step (use_decode_kernel False, block
    tables set, as the reference's prepare_step builds it): slot write of the
    step's rows, then varlen attention over the paged cache."""
    from nanokv_b200.layers.attention import Attention
    from nanokv_b200.utils.context import reset_context, set_context

    Hq, Hk, D = 32, 8, 128
    vb = make_varlen_batch(seed=57, q_lens=[1, 700, 1, 256], k_lens=[1500, 900, 3000, 256],
                           Hq=Hq, Hk=Hk)
    rng = np.random.default_rng(58)
    # the cache holds stale bytes at the step's slots until the layer stores
    kc, vc = vb.k_cache.clone(), vb.v_cache.clone()
    flat_k, flat_v = kc.view(-1, Hk, D), vc.view(-1, Hk, D)
    sl = vb.slot_mapping.long()
    flat_k[sl] = bf16(rng.standard_normal((sl.numel(), Hk, D), dtype=np.float32))
    flat_v[sl] = bf16(rng.standard_normal((sl.numel(), Hk, D), dtype=np.float32))
    a = Attention(Hq, D, D ** -0.5, Hk, types.SimpleNamespace(kv_compress_enabled=False), 1)
    a.k_cache, a.v_cache = kc.to(DEV), vc.to(DEV)
    set_context(False, vb.cu_seqlens_q.to(DEV), vb.cu_seqlens_k.to(DEV), vb.max_seqlen_q,
                vb.max_seqlen_k, vb.slot_mapping.to(DEV), None, vb.block_tables.to(DEV))
    o = a.forward(vb.q.to(DEV), vb.k_new.to(DEV), vb.v_new.to(DEV), 0)
    torch.cuda.synchronize()
    reset_context()
    assert _deverr() == 0
    kr, vr = kc.clone(), vc.clone()
    store_kvcache_ref(vb.k_new, vb.v_new, kr, vr, vb.slot_mapping)
    assert torch.equal(a.k_cache.cpu().view(torch.int16), kr.view(torch.int16))
    assert torch.equal(a.v_cache.cpu().view(torch.int16), vr.view(torch.int16))
    ref = varlen_attention_ref(vb.q, kr, vr, vb.cu_seqlens_q, vb.cu_seqlens_k, D ** -0.5, True,
                               vb.block_tables)
    _close(o, ref, "layer prefill")


def test_prefill_config4_full_chunk_sampled_rows(cuda_lib):
    """BASELINE config 4's last prefill chunk at full size for one layer: 16
    rows x 2,048 new tokens over 30,720 cached tokens, Qwen3-32B attention
    shapes (64 q / 8 kv heads), the cache in 256-token blocks (~1 GB each of
    K and V, generated on the device). Size-independent property: sampled
    query rows -- first, middle and last of the chunk of three sequences --
    equal the oracle attending over their own causal prefix."""
    ops = _ops()
    B, Hq, Hk, D, BS, chunk, L = 16, 64, 8, 128, 256, 2048, 32768
    nbs = L // BS
    nb = B * nbs
    g = torch.Generator(device=DEV).manual_seed(31)
    kc = torch.randn(nb, BS, Hk, D, device=DEV, generator=g, dtype=torch.bfloat16)
    vc = torch.randn(nb, BS, Hk, D, device=DEV, generator=g, dtype=torch.bfloat16)
    q = torch.randn(B * chunk, Hq, D, device=DEV, generator=g, dtype=torch.bfloat16)
    bt = torch.randperm(nb, generator=torch.Generator().manual_seed(32)).to(torch.int32).view(B, nbs)
    cu_q = torch.arange(B + 1, dtype=torch.int32) * chunk
    cu_k = torch.arange(B + 1, dtype=torch.int32) * L
    out = ops.paged_prefill(q, kc, vc, cu_q.to(DEV), cu_k.to(DEV), chunk, D ** -0.5,
                            block_table=bt.to(DEV))
    torch.cuda.synchronize()
    assert _deverr() == 0
    for b in (0, 9, 15):
        for i in (0, chunk // 2, chunk - 1):
            p = L - chunk + i  # absolute position; keys 0..p are visible
            nblk = p // BS + 1
            blocks = bt[b, :nblk].long().to(DEV)
            ks = kc[blocks].cpu().view(-1, Hk, D)[:p + 1]
            vs = vc[blocks].cpu().view(-1, Hk, D)[:p + 1]
            row = b * chunk + i
            ref = varlen_attention_ref(q[row:row + 1].cpu(), ks, vs,
                                       torch.tensor([0, 1], dtype=torch.int32),
                                       torch.tensor([0, p + 1], dtype=torch.int32), D ** -0.5,
                                       True, None)
            _close(out[row:row + 1], ref, f"seq {b} row {i}")
