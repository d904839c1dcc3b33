// Per-head RMSNorm of q and k, rotary embedding, and the slot write of k and
// v, in one launch: the B200 replacement for the sequence
//   q = q_norm(q); k = k_norm(k)                 nanokvllm/models/qwen3.py:109-111
//   q, k = rotary_emb(positions, q, k)           qwen3.py:113
//   store_kvcache(k, v, k_cache, v_cache, slots) nanokvllm/layers/attention.py:72-73
// reading the fused qkv projection output once and writing the rotated q
// rows plus the cache slots, so k never makes a round trip through HBM
// before the store.
//
// Arithmetic follows the reference modules' rounding points
// (nanokvllm/layers/layernorm.py:16-25, rotary_embedding.py:7-15):
//   RMSNorm: x fp32, var = mean(x^2), y = bf16(x * rsqrt(var + eps)),
//            z = bf16(y * w) with w the bf16 weight;
//   RoPE (rotate-half, neox): x1 = z[0:64], x2 = z[64:128] in fp32,
//            out1 = bf16(x1*cos - x2*sin), out2 = bf16(x2*cos + x1*sin),
//            cos/sin read from the module's fp32 cos_sin_cache[position]
//            (cos in [0, D/2), sin in [D/2, D)), products rounded before
//            the subtraction / addition as in eager torch.
// One warp per (token, head): lane l holds dims {2l, 2l+1} and their
// rotate-half partners {64+2l, 64+2l+1}, so RoPE needs no shuffles and
// every load / store is a coalesced 128-byte half row.
#pragma once
#include "nkv_common.cuh"

namespace nkv {

constexpr int kNormRopeWarps = 8;  // warps (token-head rows) per CTA

struct NormRopeParams {
  const __nv_bfloat16* qkv;     // [T, (Hq + 2 Hk) * 128], row stride qkv_stride
  int64_t qkv_stride;
  const int64_t* positions;     // [T]
  const float* cos_sin;         // [max_positions, 128]
  int64_t max_positions;
  const __nv_bfloat16* q_weight;  // [128]
  const __nv_bfloat16* k_weight;  // [128]
  float eps;
  __nv_bfloat16* q_out;         // [T, Hq, 128], row stride q_out_stride
  int64_t q_out_stride;
  __nv_bfloat16* k_out;         // optional [T, Hk, 128]
  int64_t k_out_stride;
  __nv_bfloat16* k_cache;       // optional [num_slots, Hk, 128]
  __nv_bfloat16* v_cache;
  int64_t num_slots;
  const int32_t* slot_mapping;  // [T], -1 = no cache write
  int num_tokens;
  int num_q_heads;
  int num_kv_heads;
};

__device__ __forceinline__ float2 bf2_to_f2(uint32_t u) {
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}

__global__ void __launch_bounds__(kNormRopeWarps * 32)
qk_norm_rope_kernel(const NormRopeParams p) {
  const int lane = threadIdx.x & 31;
  const int heads = p.num_q_heads + 2 * p.num_kv_heads;
  const int64_t item = static_cast<int64_t>(blockIdx.x) * kNormRopeWarps + (threadIdx.x >> 5);
  if (item >= static_cast<int64_t>(p.num_tokens) * heads) return;
  const int t = static_cast<int>(item / heads);
  const int h = static_cast<int>(item - static_cast<int64_t>(t) * heads);
  const __nv_bfloat16* src = p.qkv + static_cast<int64_t>(t) * p.qkv_stride + h * 128;
  const uint32_t lo = *reinterpret_cast<const uint32_t*>(src + 2 * lane);
  const uint32_t hi = *reinterpret_cast<const uint32_t*>(src + 64 + 2 * lane);
  const bool is_v = h >= p.num_q_heads + p.num_kv_heads;
  const bool is_k = !is_v && h >= p.num_q_heads;
  const int kvh = is_v ? h - p.num_q_heads - p.num_kv_heads : h - p.num_q_heads;
  // slot_mapping is read only when there is a cache to write (it may be NULL
  // otherwise)
  const int32_t slot =
      ((is_k || is_v) && p.k_cache != nullptr) ? __ldg(p.slot_mapping + t) : -1;
  if (slot >= 0 && slot >= p.num_slots) {
    if (lane == 0) raise_error(NKV_DEVERR_STORE_SLOT);
  }
  const bool write_cache = p.k_cache != nullptr && slot >= 0 && slot < p.num_slots;
  if (is_v) {
    if (write_cache) {
      __nv_bfloat16* dst = p.v_cache + (static_cast<int64_t>(slot) * p.num_kv_heads + kvh) * 128;
      *reinterpret_cast<uint32_t*>(dst + 2 * lane) = lo;
      *reinterpret_cast<uint32_t*>(dst + 64 + 2 * lane) = hi;
    }
    return;
  }
  // ---- RMSNorm over the 128 dims of this head
  const float2 a = bf2_to_f2(lo), c = bf2_to_f2(hi);
  float ss = a.x * a.x + a.y * a.y + c.x * c.x + c.y * c.y;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float rinv = rsqrtf(ss * (1.f / 128.f) + p.eps);
  const __nv_bfloat16* w = is_k ? p.k_weight : p.q_weight;
  const float2 wl = bf2_to_f2(*reinterpret_cast<const uint32_t*>(w + 2 * lane));
  const float2 wh = bf2_to_f2(*reinterpret_cast<const uint32_t*>(w + 64 + 2 * lane));
  // y = bf16(x * r); z = bf16(y * w)
  const float x1a = round_bf16(round_bf16(a.x * rinv) * wl.x);
  const float x1b = round_bf16(round_bf16(a.y * rinv) * wl.y);
  const float x2a = round_bf16(round_bf16(c.x * rinv) * wh.x);
  const float x2b = round_bf16(round_bf16(c.y * rinv) * wh.y);
  // ---- rotary embedding (rotate-half), products rounded before the sum
  int64_t pos = __ldg(p.positions + t);
  if (pos < 0 || pos >= p.max_positions) {
    if (lane == 0) raise_error(NKV_DEVERR_ROPE_POSITION);
    pos = pos < 0 ? 0 : p.max_positions - 1;
  }
  const float* cs = p.cos_sin + pos * 128;
  const float2 cv = *reinterpret_cast<const float2*>(cs + 2 * lane);
  const float2 sv = *reinterpret_cast<const float2*>(cs + 64 + 2 * lane);
  const float o1a = __fsub_rn(__fmul_rn(x1a, cv.x), __fmul_rn(x2a, sv.x));
  const float o1b = __fsub_rn(__fmul_rn(x1b, cv.y), __fmul_rn(x2b, sv.y));
  const float o2a = __fadd_rn(__fmul_rn(x2a, cv.x), __fmul_rn(x1a, sv.x));
  const float o2b = __fadd_rn(__fmul_rn(x2b, cv.y), __fmul_rn(x1b, sv.y));
  const uint32_t olo = pack_bf16x2(o1a, o1b);
  const uint32_t ohi = pack_bf16x2(o2a, o2b);
  if (!is_k) {
    __nv_bfloat16* dst = p.q_out + static_cast<int64_t>(t) * p.q_out_stride + h * 128;
    *reinterpret_cast<uint32_t*>(dst + 2 * lane) = olo;
    *reinterpret_cast<uint32_t*>(dst + 64 + 2 * lane) = ohi;
    return;
  }
  if (p.k_out != nullptr) {
    __nv_bfloat16* dst = p.k_out + static_cast<int64_t>(t) * p.k_out_stride + kvh * 128;
    *reinterpret_cast<uint32_t*>(dst + 2 * lane) = olo;
    *reinterpret_cast<uint32_t*>(dst + 64 + 2 * lane) = ohi;
  }
  if (write_cache) {
    __nv_bfloat16* dst = p.k_cache + (static_cast<int64_t>(slot) * p.num_kv_heads + kvh) * 128;
    *reinterpret_cast<uint32_t*>(dst + 2 * lane) = olo;
    *reinterpret_cast<uint32_t*>(dst + 64 + 2 * lane) = ohi;
  }
}

}  // namespace nkv
