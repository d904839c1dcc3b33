"""Torch-facing wrappers of the libnkv C ABI (include/nkv.h).

Every function here validates its tensors the way the reference does (the
same asserts as nanokvllm/layers/attention.py:33-40 for the store), passes raw
device pointers and the caller's current CUDA stream to the library, and
raises on a non-zero status. There is no CPU or Triton fallback: CPU tensors
are rejected.
"""

from __future__ import annotations

import math
import threading

import torch

from . import _lib

__all__ = [
    "store_kvcache",
    "flash_decode_with_kvcache",
    "paged_decode",
    "decode_step",
    "decode_workspace",
    "paged_prefill",
    "qk_norm_rope_store",
    "flash_attn_varlen_func",
    "window_compress",
    "window_select",
    "query_window_append",
    "threshold_compress",
]


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(name: str, *tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError(f"{name}: CUDA tensors required (libnkv has no CPU path)")


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


# ---------------------------------------------------------------- store
def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor,
                  v_cache: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    """Writes key/value rows into their cache slots (slot == -1 is skipped).

    Same contract and asserts as the reference's store_kvcache
    (nanokvllm/layers/attention.py:33-40).
    """
    N, num_heads, head_dim = key.shape
    D = num_heads * head_dim
    assert key.stride(-1) == 1 and value.stride(-1) == 1
    assert key.stride(1) == head_dim and value.stride(1) == head_dim
    assert k_cache.stride(1) == D and v_cache.stride(1) == D
    assert slot_mapping.numel() == N
    if N == 0 or k_cache.numel() == 0:
        return
    _require_cuda("store_kvcache", key, value, k_cache, v_cache, slot_mapping)
    assert key.dtype == torch.bfloat16 and k_cache.dtype == torch.bfloat16
    assert slot_mapping.dtype == torch.int32 and slot_mapping.is_contiguous()
    num_slots = k_cache.numel() // D
    lib = _lib.load()
    _lib.check("nkv_store_kvcache", lib.nkv_store_kvcache(
        key.data_ptr(), key.stride(0), value.data_ptr(), value.stride(0),
        k_cache.data_ptr(), v_cache.data_ptr(), num_slots,
        slot_mapping.data_ptr(), N, num_heads, head_dim, _stream(key.device)))


# ---------------------------------------------------------------- decode
class _WorkspacePool:
    """One zero-initialised decode workspace per device, grown on demand.

    The decode kernel leaves its workspace zeroed after every call, so a
    single buffer serves every layer, step and captured graph. Call
    `decode_workspace(...)` with the largest shape before capturing a graph so
    the capture never allocates.
    """

    def __init__(self):
        self._bufs: dict[int, torch.Tensor] = {}
        self._lock = threading.Lock()

    def get(self, device: torch.device, nbytes: int) -> torch.Tensor:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        with self._lock:
            buf = self._bufs.get(idx)
            if buf is None or buf.numel() < nbytes:
                buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=torch.device("cuda", idx))
                self._bufs[idx] = buf
            return buf


_WS = _WorkspacePool()


def decode_workspace_bytes(batch: int, num_q_heads: int, num_kv_heads: int, head_dim: int,
                           max_blocks: int, block_size: int) -> int:
    return int(_lib.load().nkv_paged_decode_workspace_size(
        batch, num_q_heads, num_kv_heads, head_dim, max_blocks, block_size))


def decode_workspace(device: torch.device, batch: int, num_q_heads: int, num_kv_heads: int,
                     head_dim: int, max_blocks: int, block_size: int) -> torch.Tensor:
    nbytes = decode_workspace_bytes(batch, num_q_heads, num_kv_heads, head_dim, max_blocks, block_size)
    return _WS.get(device, nbytes)


def paged_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                 block_tables: torch.Tensor, context_lens: torch.Tensor, softmax_scale: float,
                 out: torch.Tensor | None = None,
                 workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Decode attention for one query token per sequence over the paged cache.

    q: [B, Hq, D] bf16 (row stride free, head stride multiple of 8);
    k_cache/v_cache: [num_blocks, block_size, Hk, D]; block_tables [B, max_blocks]
    int32; context_lens [B] int32. Returns out [B, Hq, D] bf16.
    """
    _require_cuda("paged_decode", q, k_cache, v_cache, block_tables, context_lens)
    B, Hq, D = q.shape
    num_blocks, block_size, Hk, Dk = k_cache.shape
    assert Dk == D and v_cache.shape == k_cache.shape
    assert q.dtype == torch.bfloat16 and k_cache.dtype == torch.bfloat16 and v_cache.dtype == torch.bfloat16
    assert q.stride(-1) == 1
    assert k_cache.is_contiguous() and v_cache.is_contiguous()
    assert block_tables.dtype == torch.int32 and context_lens.dtype == torch.int32
    assert block_tables.dim() == 2 and block_tables.size(0) >= B and block_tables.stride(1) == 1
    assert context_lens.numel() >= B and context_lens.is_contiguous()
    max_blocks = block_tables.size(1)
    if block_tables.stride(0) != max_blocks:
        block_tables = block_tables.contiguous()
    if out is None:
        out = torch.empty(B, Hq, D, dtype=torch.bfloat16, device=q.device)
    assert out.stride(-1) == 1 and out.stride(1) == D
    if B == 0:
        return out
    if workspace is None:
        workspace = decode_workspace(q.device, B, Hq, Hk, D, max_blocks, block_size)
    lib = _lib.load()
    _lib.check("nkv_paged_decode", lib.nkv_paged_decode(
        q.data_ptr(), q.stride(0), q.stride(1), k_cache.data_ptr(), v_cache.data_ptr(), num_blocks,
        block_tables.data_ptr(), max_blocks, context_lens.data_ptr(), out.data_ptr(), out.stride(0),
        B, Hq, Hk, D, block_size, float(softmax_scale), workspace.data_ptr(),
        workspace.numel() * workspace.element_size(), _stream(q.device)))
    return out


def decode_step(q: torch.Tensor, key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor,
                v_cache: torch.Tensor, slot_mapping: torch.Tensor, block_tables: torch.Tensor,
                context_lens: torch.Tensor, softmax_scale: float, out: torch.Tensor | None = None,
                ring: torch.Tensor | None = None, layer_id: int = 0,
                ring_slot_of_row: torch.Tensor | None = None,
                ring_pos_of_row: torch.Tensor | None = None,
                workspace: torch.Tensor | None = None,
                metadata_ready: bool = False) -> torch.Tensor:
    """One fused launch of store_kvcache(key, value, slot_mapping) [+ the
    KvChat query-window append] + paged_decode for a decode step (one new
    token per row, slot_mapping[b] = -1 or the slot of position
    context_lens[b] - 1).

    metadata_ready: the caller vouches that the kernel launched just before
    this call on the stream does not write block_tables, context_lens,
    slot_mapping or the ring indices (host copies and earlier kernels are
    fine), so the launch may read them before it waits for that kernel --
    true of a decode step's layers, whose metadata the engine copies from
    the host; not of a decode right after a compression kernel."""
    _require_cuda("decode_step", q, key, value, k_cache, v_cache, slot_mapping, block_tables,
                  context_lens)
    B, Hq, D = q.shape
    num_blocks, block_size, Hk, Dk = k_cache.shape
    assert Dk == D and v_cache.shape == k_cache.shape
    assert key.shape == (B, Hk, D) and value.shape == (B, Hk, D)
    assert key.stride(-1) == 1 and value.stride(-1) == 1
    assert key.stride(1) == D and value.stride(1) == D
    assert q.stride(-1) == 1 and k_cache.is_contiguous() and v_cache.is_contiguous()
    assert slot_mapping.dtype == torch.int32 and slot_mapping.numel() == B
    assert block_tables.dtype == torch.int32 and context_lens.dtype == torch.int32
    max_blocks = block_tables.size(1)
    if block_tables.stride(0) != max_blocks:
        block_tables = block_tables.contiguous()
        metadata_ready = False  # the copy kernel just wrote it
    if out is None:
        out = torch.empty(B, Hq, D, dtype=torch.bfloat16, device=q.device)
    if B == 0:
        return out
    if workspace is None:
        workspace = decode_workspace(q.device, B, Hq, Hk, D, max_blocks, block_size)
    if ring is not None:
        slots, layers, W, Hr, Dr = ring.shape
        assert Hr == Hq and Dr == D and ring.is_contiguous()
        ring_args = (ring.data_ptr(), slots, layers, W, layer_id, ring_slot_of_row.data_ptr(),
                     ring_pos_of_row.data_ptr())
    else:
        ring_args = (None, 0, 0, 0, 0, None, None)
    lib = _lib.load()
    _lib.check("nkv_decode_step", lib.nkv_decode_step(
        q.data_ptr(), q.stride(0), q.stride(1), key.data_ptr(), key.stride(0), value.data_ptr(),
        value.stride(0), slot_mapping.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
        num_blocks, block_tables.data_ptr(), max_blocks, context_lens.data_ptr(), *ring_args,
        out.data_ptr(), out.stride(0), B, Hq, Hk, D, block_size, float(softmax_scale),
        1 if metadata_ready else 0,
        workspace.data_ptr(), workspace.numel() * workspace.element_size(), _stream(q.device)))
    return out


def flash_decode_with_kvcache(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                              cache_seqlens: torch.Tensor, block_table: torch.Tensor,
                              softmax_scale: float | None = None, causal: bool = True,
                              out: torch.Tensor | None = None) -> torch.Tensor:
    """Drop-in for the reference's flash_attn_with_kvcache decode call
    (nanokvllm/layers/attention.py:104-107): q is [B, 1, Hq, D], the result
    is [B, 1, Hq, D]. With one query token `causal` changes nothing."""
    assert q.dim() == 4 and q.size(1) == 1, "decode path: exactly one query token per sequence"
    if softmax_scale is None:
        softmax_scale = q.size(-1) ** -0.5
    o = paged_decode(q[:, 0], k_cache, v_cache, block_table, cache_seqlens, softmax_scale,
                     out=None if out is None else out[:, 0])
    return o.unsqueeze(1)


# ---------------------------------------------------------------- q/k norm + RoPE + store
def qk_norm_rope_store(qkv: torch.Tensor, positions: torch.Tensor, cos_sin_cache: torch.Tensor,
                       q_norm_weight: torch.Tensor, k_norm_weight: torch.Tensor, eps: float,
                       num_q_heads: int, num_kv_heads: int, k_cache: torch.Tensor | None = None,
                       v_cache: torch.Tensor | None = None,
                       slot_mapping: torch.Tensor | None = None,
                       q_out: torch.Tensor | None = None, k_out: torch.Tensor | None = None):
    """q_norm / k_norm + rotary_emb + store_kvcache of one layer in one launch
    (nkv_qk_norm_rope_store; the sequence at nanokvllm/models/qwen3.py:109-113
    and nanokvllm/layers/attention.py:72-73).

    qkv: [T, (Hq + 2 Hk) * 128] bf16 (the qkv projection output);
    positions: [T] int64; cos_sin_cache: the RotaryEmbedding module's fp32
    buffer ([max_pos, 1, 128] or [max_pos, 128]); norm weights [128] bf16.
    Returns (q [T, Hq, 128], v view [T, Hk, 128], k_out or None); k and v
    are written to the cache slots when k_cache is given.
    """
    _require_cuda("qk_norm_rope_store", qkv, positions, cos_sin_cache, q_norm_weight,
                  k_norm_weight, k_cache, v_cache, slot_mapping)
    T = qkv.size(0)
    D = 128
    assert qkv.dtype == torch.bfloat16 and qkv.stride(-1) == 1
    assert qkv.size(-1) == (num_q_heads + 2 * num_kv_heads) * D
    assert positions.dtype == torch.int64 and positions.is_contiguous() and positions.numel() == T
    cs = cos_sin_cache.reshape(-1, D)
    assert cs.dtype == torch.float32 and cs.is_contiguous()
    assert q_norm_weight.dtype == torch.bfloat16 and k_norm_weight.dtype == torch.bfloat16
    assert q_norm_weight.is_contiguous() and k_norm_weight.is_contiguous()
    if q_out is None:
        q_out = torch.empty(T, num_q_heads, D, dtype=torch.bfloat16, device=qkv.device)
    assert q_out.stride(-1) == 1 and q_out.stride(1) == D
    if k_out is not None:
        assert k_out.stride(-1) == 1 and k_out.stride(1) == D
    num_slots = 0
    if k_cache is not None:
        assert v_cache is not None and slot_mapping is not None
        assert k_cache.is_contiguous() and v_cache.is_contiguous() and v_cache.shape == k_cache.shape
        assert slot_mapping.dtype == torch.int32 and slot_mapping.numel() == T
        num_slots = k_cache.numel() // (num_kv_heads * D)
    v = qkv[:, (num_q_heads + num_kv_heads) * D:].view(T, num_kv_heads, D)
    if T == 0:
        return q_out, v, k_out
    lib = _lib.load()
    _lib.check("nkv_qk_norm_rope_store", lib.nkv_qk_norm_rope_store(
        qkv.data_ptr(), qkv.stride(0), T, positions.data_ptr(), cs.data_ptr(), cs.size(0),
        q_norm_weight.data_ptr(), k_norm_weight.data_ptr(), float(eps), q_out.data_ptr(),
        q_out.stride(0), _ptr(k_out), 0 if k_out is None else k_out.stride(0), _ptr(k_cache),
        _ptr(v_cache), num_slots, _ptr(slot_mapping), num_q_heads, num_kv_heads, D,
        _stream(qkv.device)))
    return q_out, v, k_out


# ---------------------------------------------------------------- prefill
def paged_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens_q: torch.Tensor,
                  cu_seqlens_k: torch.Tensor, max_seqlen_q: int, softmax_scale: float,
                  causal: bool = True, block_table: torch.Tensor | None = None,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """Variable-length attention of a prefill / mixed batch (nkv_paged_prefill).

    q: [T, Hq, D] bf16. With block_table ([B, max_blocks] int32) k / v are the
    paged caches [num_blocks, block_size, Hk, D]; without it they are the
    step's rows [Tk, Hk, D] addressed through cu_seqlens_k. cu_seqlens_* are
    int32 [B + 1] device tensors; causal masks bottom-right aligned.
    Returns out [T, Hq, D] bf16.
    """
    _require_cuda("paged_prefill", q, k, v, cu_seqlens_q, cu_seqlens_k, block_table)
    T, Hq, D = q.shape
    assert q.dtype == torch.bfloat16 and k.dtype == torch.bfloat16 and v.dtype == torch.bfloat16
    assert q.stride(-1) == 1 and k.stride(-1) == 1 and v.stride(-1) == 1
    assert cu_seqlens_q.dtype == torch.int32 and cu_seqlens_k.dtype == torch.int32
    assert cu_seqlens_q.is_contiguous() and cu_seqlens_k.is_contiguous()
    B = cu_seqlens_q.numel() - 1
    assert cu_seqlens_k.numel() == B + 1
    if block_table is not None:
        num_blocks, block_size, Hk, Dk = k.shape
        assert k.is_contiguous() and v.is_contiguous() and v.shape == k.shape
        assert block_table.dtype == torch.int32 and block_table.dim() == 2
        assert block_table.size(0) >= B
        if not block_table.is_contiguous():
            block_table = block_table.contiguous()
        rows, k_stride, v_stride = num_blocks * block_size, Hk * D, Hk * D
        max_blocks = block_table.size(1)
        bt_ptr = block_table.data_ptr()
    else:
        rows, Hk, Dk = k.shape
        assert v.shape == k.shape and k.stride(1) == D and v.stride(1) == D
        k_stride, v_stride = k.stride(0), v.stride(0)
        block_size = max_blocks = 0
        bt_ptr = None
    assert Dk == D
    if out is None:
        out = torch.empty(T, Hq, D, dtype=torch.bfloat16, device=q.device)
    assert out.stride(-1) == 1 and out.stride(1) == D and out.size(0) >= T
    if B <= 0 or T == 0 or max_seqlen_q <= 0:
        return out
    lib = _lib.load()
    _lib.check("nkv_paged_prefill", lib.nkv_paged_prefill(
        q.data_ptr(), q.stride(0), q.stride(1), T, k.data_ptr(), k_stride, v.data_ptr(), v_stride,
        rows, bt_ptr, max_blocks, block_size, cu_seqlens_q.data_ptr(), cu_seqlens_k.data_ptr(), B,
        int(max_seqlen_q), 1 if causal else 0, out.data_ptr(), out.stride(0), Hq, Hk, D,
        float(softmax_scale), _stream(q.device)))
    return out


def flash_attn_varlen_func(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                           cu_seqlens_q: torch.Tensor, cu_seqlens_k: torch.Tensor,
                           max_seqlen_q: int, max_seqlen_k: int,
                           softmax_scale: float | None = None, causal: bool = False,
                           block_table: torch.Tensor | None = None) -> torch.Tensor:
    """Drop-in for the reference's prefill / mixed-batch call of
    flash_attn_varlen_func (nanokvllm/layers/attention.py:96-102), with the
    keyword names and defaults of flash-attn's function. max_seqlen_k is
    accepted for the signature; the kernel reads each length from cu_seqlens_k.
    """
    del max_seqlen_k
    if softmax_scale is None:
        softmax_scale = q.size(-1) ** -0.5
    return paged_prefill(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, softmax_scale,
                         causal=causal, block_table=block_table)


def window_select(context_lens: torch.Tensor, tail_uncompressed: torch.Tensor, block_size: int,
                  window_blocks: int, topk: int, out_selected: torch.Tensor | None = None,
                  out_count: torch.Tensor | None = None,
                  out_base_lens: torch.Tensor | None = None) -> torch.Tensor:
    """Device-side periodic-compression selection (nkv_window_select): the
    first `topk` eligible rows by the reference's rule (model_runner.py:
    305-321) into out_selected[topk], -1 padded. All tensors int32 on the
    device; nothing is read back, so the call can sit inside a CUDA graph."""
    _require_cuda("window_select", context_lens, tail_uncompressed, out_selected, out_count,
                  out_base_lens)
    B = context_lens.numel()
    assert context_lens.dtype == torch.int32 and tail_uncompressed.dtype == torch.int32
    assert context_lens.is_contiguous() and tail_uncompressed.is_contiguous()
    assert tail_uncompressed.numel() >= B
    if out_selected is None:
        out_selected = torch.empty(topk, dtype=torch.int32, device=context_lens.device)
    assert out_selected.dtype == torch.int32 and out_selected.numel() >= topk
    lib = _lib.load()
    _lib.check("nkv_window_select", lib.nkv_window_select(
        context_lens.data_ptr(), tail_uncompressed.data_ptr(), B, block_size, window_blocks, topk,
        out_selected.data_ptr(), _ptr(out_count), _ptr(out_base_lens), _stream(context_lens.device)))
    return out_selected


# ---------------------------------------------------------------- window compression
def window_compress(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                    block_tables: torch.Tensor, base_context_lens: torch.Tensor,
                    context_lens: torch.Tensor, selected: torch.Tensor, window_blocks: int,
                    keep_tokens: int, obs_window: int = 1, softmax_scale: float | None = None,
                    out_keep_idx: torch.Tensor | None = None,
                    out_new_lens: torch.Tensor | None = None,
                    out_importance: torch.Tensor | None = None) -> None:
    """Periodic window compression of one layer (SnapKV scoring + compaction).

    `selected` is an int32 device tensor of batch indices; context_lens is
    updated in place. softmax_scale defaults to SnapKV's 1/sqrt(head_dim).
    out_importance (bf16 [m, window_blocks * block_size - obs_window]), if
    given, receives the importance SnapKV ranked.
    """
    _require_cuda("window_compress", q, k_cache, v_cache, block_tables, base_context_lens,
                  context_lens, selected)
    m = selected.numel()
    if m == 0:
        return
    num_blocks, block_size, Hk, D = k_cache.shape
    Hq = q.size(1)
    assert q.stride(-1) == 1 and q.stride(1) == D
    assert selected.dtype == torch.int32 and selected.is_contiguous()
    assert block_tables.dtype == torch.int32 and block_tables.is_contiguous()
    assert base_context_lens.dtype == torch.int32 and context_lens.dtype == torch.int32
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(D)
    if out_importance is not None:
        assert out_importance.dtype == torch.bfloat16 and out_importance.is_contiguous()
        assert out_importance.shape == (m, window_blocks * block_size - obs_window)
    lib = _lib.load()
    _lib.check("nkv_window_compress", lib.nkv_window_compress(
        q.data_ptr(), q.stride(0), k_cache.data_ptr(), v_cache.data_ptr(), num_blocks,
        block_tables.data_ptr(), block_tables.size(1), base_context_lens.data_ptr(),
        context_lens.data_ptr(), selected.data_ptr(), m, window_blocks, keep_tokens, obs_window,
        Hq, Hk, D, block_size, float(softmax_scale), _ptr(out_keep_idx), _ptr(out_new_lens),
        _ptr(out_importance), _stream(q.device)))


# ---------------------------------------------------------------- KvChat threshold path
def query_window_append(q: torch.Tensor, ring: torch.Tensor, layer_id: int,
                        batch_index: torch.Tensor, ring_slot: torch.Tensor,
                        ring_pos: torch.Tensor) -> None:
    """ring[ring_slot[j], layer_id, ring_pos[j]] = q[batch_index[j]] for every j."""
    _require_cuda("query_window_append", q, ring, batch_index, ring_slot, ring_pos)
    n = batch_index.numel()
    if n == 0:
        return
    slots, layers, W, Hq, D = ring.shape
    assert q.size(1) == Hq and q.size(2) == D and q.stride(-1) == 1 and q.stride(1) == D
    assert ring.is_contiguous()
    lib = _lib.load()
    _lib.check("nkv_query_window_append", lib.nkv_query_window_append(
        q.data_ptr(), q.stride(0), ring.data_ptr(), slots, layers, W, layer_id,
        batch_index.data_ptr(), ring_slot.data_ptr(), ring_pos.data_ptr(), n, Hq, D,
        _stream(q.device)))


def threshold_compress(ring: torch.Tensor, ring_slot_of_selected: torch.Tensor, layer_id: int,
                       k_cache: torch.Tensor, v_cache: torch.Tensor, block_tables: torch.Tensor,
                       context_lens: torch.Tensor, selected: torch.Tensor, S: int, R: int,
                       softmax_scale: float | None = None,
                       out_keep_idx: torch.Tensor | None = None,
                       out_importance: torch.Tensor | None = None) -> None:
    """KvChat threshold compression S -> R of one layer; context_lens[sel] = R.
    out_importance (bf16 [m, S - W]), if given, receives the importance
    SnapKV ranked."""
    _require_cuda("threshold_compress", ring, ring_slot_of_selected, k_cache, v_cache,
                  block_tables, context_lens, selected)
    m = selected.numel()
    if m == 0:
        return
    slots, layers, W, Hq, D = ring.shape
    num_blocks, block_size, Hk, Dk = k_cache.shape
    assert Dk == D and ring.is_contiguous() and block_tables.is_contiguous()
    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(D)
    if out_importance is not None:
        assert out_importance.dtype == torch.bfloat16 and out_importance.is_contiguous()
        assert out_importance.shape == (m, S - W)
    lib = _lib.load()
    _lib.check("nkv_threshold_compress", lib.nkv_threshold_compress(
        ring.data_ptr(), slots, layers, W, layer_id, ring_slot_of_selected.data_ptr(),
        k_cache.data_ptr(), v_cache.data_ptr(), num_blocks, block_tables.data_ptr(),
        block_tables.size(1), context_lens.data_ptr(), selected.data_ptr(), m, S, R, Hq, Hk, D,
        block_size, float(softmax_scale), _ptr(out_keep_idx), _ptr(out_importance),
        _stream(k_cache.device)))
