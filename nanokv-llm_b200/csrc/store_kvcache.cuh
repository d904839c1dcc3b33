// Paged KV slot write: the B200 replacement for the reference's Triton
// store_kvcache_kernel (nanokvllm/layers/attention.py:10-30).
//
// One warp per token. A token row is num_kv_heads*head_dim bf16 values
// (2 KiB at 8 kv heads x 128); each lane moves 16-byte vectors, so a warp
// streams 512 bytes per instruction and the K and V rows of a token are in
// flight together. slot == -1 (graph padding rows) is skipped exactly like the
// reference; any other slot outside [0, num_slots) is skipped and flagged.
#pragma once
#include "nkv_common.cuh"

namespace nkv {

constexpr int kStoreWarpsPerBlock = 8;

__global__ void __launch_bounds__(kStoreWarpsPerBlock * 32)
store_kvcache_kernel(const uint4* __restrict__ key, int64_t key_stride_vec,
                     const uint4* __restrict__ value, int64_t value_stride_vec,
                     uint4* __restrict__ k_cache, uint4* __restrict__ v_cache, int64_t num_slots,
                     const int32_t* __restrict__ slot_mapping, int32_t num_tokens,
                     int32_t row_vecs) {
  // The decode kernel that follows in the stream may be launched now; it
  // waits for this grid's completion before it reads the cache.
  allow_dependent_launch();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int token = blockIdx.x * kStoreWarpsPerBlock + warp;
  if (token >= num_tokens) return;
  const int32_t slot = __ldg(slot_mapping + token);
  if (slot == -1) return;
  if (slot < 0 || static_cast<int64_t>(slot) >= num_slots) {
    if (lane == 0) raise_error(NKV_DEVERR_STORE_SLOT);
    return;
  }
  const uint4* ksrc = key + token * key_stride_vec;
  const uint4* vsrc = value + token * value_stride_vec;
  uint4* kdst = k_cache + static_cast<int64_t>(slot) * row_vecs;
  uint4* vdst = v_cache + static_cast<int64_t>(slot) * row_vecs;
  // Issue all loads of the row pair before the stores (up to 4+4 vectors per
  // lane at 8 kv heads) so the warp keeps 4 KiB in flight.
  constexpr int kMaxUnroll = 4;
  for (int base = 0; base < row_vecs; base += 32 * kMaxUnroll) {
    uint4 kv[kMaxUnroll], vv[kMaxUnroll];
#pragma unroll
    for (int u = 0; u < kMaxUnroll; ++u) {
      const int i = base + u * 32 + lane;
      if (i < row_vecs) {
        kv[u] = __ldg(ksrc + i);
        vv[u] = __ldg(vsrc + i);
      }
    }
#pragma unroll
    for (int u = 0; u < kMaxUnroll; ++u) {
      const int i = base + u * 32 + lane;
      if (i < row_vecs) {
        kdst[i] = kv[u];
        vdst[i] = vv[u];
      }
    }
  }
}

}  // namespace nkv
