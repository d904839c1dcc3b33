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
// One warp per (token, run of heads): the token's position and cos / sin
// are loaded once into registers; the warp then works four heads at a time
// with 16-byte loads and stores -- lanes 8h'..8h'+7 take head h' of the
// four, lane m = lane % 8 holding dims [8m, 8m+8) and their rotate-half
// partners [64+8m, 64+8m+8), so RoPE needs no shuffles and the RMSNorm
// reduction is three shuffles within the 8 lanes.
#pragma once
#include "nkv_common.cuh"

namespace nkv {

constexpr int kNormRopeWarps = 8;  // warps per CTA

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
  const int32_t* slot_mapping;  // [T], -1 = no cache write (read only with a cache)
  int num_tokens;
  int num_q_heads;
  int num_kv_heads;
  int groups_per_warp;          // 4-head groups one warp handles
  int warps_per_token;
};

__device__ __forceinline__ void bf8_to_f8(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

__global__ void __launch_bounds__(kNormRopeWarps * 32)
qk_norm_rope_kernel(const NormRopeParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * kNormRopeWarps + (threadIdx.x >> 5);
  const int t = static_cast<int>(gw / p.warps_per_token);
  if (t >= p.num_tokens) return;
  const int part = static_cast<int>(gw - static_cast<int64_t>(t) * p.warps_per_token);
  const int heads = p.num_q_heads + 2 * p.num_kv_heads;
  const int m = lane & 7;     // dims [8m, 8m+8) and [64+8m, 64+8m+8)
  const int sub = lane >> 3;  // head within the group of four

  // ---- per token: position, cos / sin of this lane's dims, slot
  int64_t pos = __ldg(p.positions + t);
  if (pos < 0 || pos >= p.max_positions) {
    if (lane == 0 && part == 0) raise_error(NKV_DEVERR_ROPE_POSITION);
    pos = pos < 0 ? 0 : p.max_positions - 1;
  }
  const float4* cs4 = reinterpret_cast<const float4*>(p.cos_sin + pos * 128);
  float cv[8], sv[8];
  {
    const float4 c0 = __ldg(cs4 + 2 * m), c1 = __ldg(cs4 + 2 * m + 1);
    const float4 s0 = __ldg(cs4 + 16 + 2 * m), s1 = __ldg(cs4 + 16 + 2 * m + 1);
    cv[0] = c0.x; cv[1] = c0.y; cv[2] = c0.z; cv[3] = c0.w;
    cv[4] = c1.x; cv[5] = c1.y; cv[6] = c1.z; cv[7] = c1.w;
    sv[0] = s0.x; sv[1] = s0.y; sv[2] = s0.z; sv[3] = s0.w;
    sv[4] = s1.x; sv[5] = s1.y; sv[6] = s1.z; sv[7] = s1.w;
  }
  int32_t slot = -1;
  if (p.k_cache != nullptr) {
    slot = __ldg(p.slot_mapping + t);
    if (slot >= p.num_slots) {
      if (lane == 0 && part == 0) raise_error(NKV_DEVERR_STORE_SLOT);
      slot = -1;
    }
  }
  const __nv_bfloat16* row = p.qkv + static_cast<int64_t>(t) * p.qkv_stride;
  const int g0 = part * p.groups_per_warp;
  for (int gi = 0; gi < p.groups_per_warp; ++gi) {
    const int h = (g0 + gi) * 4 + sub;
    if (h >= heads) break;  // trailing lanes of the last group (uniform per 8 lanes)
    const __nv_bfloat16* src = row + h * 128;
    const uint4 lo = *reinterpret_cast<const uint4*>(src + 8 * m);
    const uint4 hi = *reinterpret_cast<const uint4*>(src + 64 + 8 * m);
    const bool is_v = h >= p.num_q_heads + p.num_kv_heads;
    const bool is_k = !is_v && h >= p.num_q_heads;
    const int kvh = is_v ? h - p.num_q_heads - p.num_kv_heads : h - p.num_q_heads;
    if (is_v) {
      if (slot >= 0) {
        __nv_bfloat16* dst = p.v_cache + (static_cast<int64_t>(slot) * p.num_kv_heads + kvh) * 128;
        *reinterpret_cast<uint4*>(dst + 8 * m) = lo;
        *reinterpret_cast<uint4*>(dst + 64 + 8 * m) = hi;
      }
      continue;
    }
    float x1[8], x2[8];
    bf8_to_f8(lo, x1);
    bf8_to_f8(hi, x2);
    // ---- RMSNorm: y = bf16(x * rsqrt(mean(x^2) + eps)), z = bf16(y * w)
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += x1[i] * x1[i] + x2[i] * x2[i];
    const unsigned gmask = 0xffu << (8 * sub);  // this head's 8 lanes, all on the same path
    ss += __shfl_xor_sync(gmask, ss, 1);
    ss += __shfl_xor_sync(gmask, ss, 2);
    ss += __shfl_xor_sync(gmask, ss, 4);
    const float rinv = rsqrtf(ss * (1.f / 128.f) + p.eps);
    const __nv_bfloat16* w = is_k ? p.k_weight : p.q_weight;
    float w1[8], w2[8];
    bf8_to_f8(__ldg(reinterpret_cast<const uint4*>(w + 8 * m)), w1);
    bf8_to_f8(__ldg(reinterpret_cast<const uint4*>(w + 64 + 8 * m)), w2);
    uint32_t olo[4], ohi[4];
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      float a[2], c[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float z1 = round_bf16(round_bf16(x1[i + e] * rinv) * w1[i + e]);
        const float z2 = round_bf16(round_bf16(x2[i + e] * rinv) * w2[i + e]);
        // ---- RoPE, products rounded before the sum (eager torch)
        a[e] = __fsub_rn(__fmul_rn(z1, cv[i + e]), __fmul_rn(z2, sv[i + e]));
        c[e] = __fadd_rn(__fmul_rn(z2, cv[i + e]), __fmul_rn(z1, sv[i + e]));
      }
      olo[i / 2] = pack_bf16x2(a[0], a[1]);
      ohi[i / 2] = pack_bf16x2(c[0], c[1]);
    }
    const uint4 vlo = make_uint4(olo[0], olo[1], olo[2], olo[3]);
    const uint4 vhi = make_uint4(ohi[0], ohi[1], ohi[2], ohi[3]);
    __nv_bfloat16* dst;
    if (!is_k) {
      dst = p.q_out + static_cast<int64_t>(t) * p.q_out_stride + h * 128;
      *reinterpret_cast<uint4*>(dst + 8 * m) = vlo;
      *reinterpret_cast<uint4*>(dst + 64 + 8 * m) = vhi;
      continue;
    }
    if (p.k_out != nullptr) {
      dst = p.k_out + static_cast<int64_t>(t) * p.k_out_stride + kvh * 128;
      *reinterpret_cast<uint4*>(dst + 8 * m) = vlo;
      *reinterpret_cast<uint4*>(dst + 64 + 8 * m) = vhi;
    }
    if (slot >= 0) {
      dst = p.k_cache + (static_cast<int64_t>(slot) * p.num_kv_heads + kvh) * 128;
      *reinterpret_cast<uint4*>(dst + 8 * m) = vlo;
      *reinterpret_cast<uint4*>(dst + 64 + 8 * m) = vhi;
    }
  }
}

}  // namespace nkv
