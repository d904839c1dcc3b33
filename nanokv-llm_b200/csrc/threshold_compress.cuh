// KvChat threshold compression (S -> R with a W-query window) and the
// device-side query-window ring.
//
// query_window_append_kernel replaces QueryWindowManager.append
// (KvChat/engine/query_window_manager.py:46-58): one CTA per active sequence
// copies its Hq x 128 query rows into ring[slot, layer, pos]. The slot and
// position arrays are device tensors, so the copy can live in a captured
// decode graph (the reference's Python loop cannot, so graph replays never
// append; the reference then scores uninitialised rows).
//
// threshold_compress_kernel replaces MyCompressCompact
// (KvChat/layers/compress_utils.py:10-171) with TritonGetKVForComp (:218-252)
// and SnapKV(window=W, num_keep=R-W-1) (KvChat/layers/CompressMethod.py:4-58).
// Launch: grid (num_kv_heads, num_selected), one cluster per sequence.
//   * Keys are positions [0, S-W) of the sequence (TritonGetKVForComp gathers
//     the first S positions; the compaction window starts at
//     max(len - S, 0) -- the two coincide whenever compression triggers).
//   * The CTA stages its kv head's key rows in shared memory once (when they
//     fit) and, for each of the W window queries, scores all keys for its g
//     query heads (bf16(q.k), bf16(* scale), sink -> -inf), takes the per-row
//     softmax (bf16 output) and accumulates it over the window in fp32; the
//     window sum is rounded to bf16 per head, summed over the group in fp32,
//     and the cluster sum of those partials is rounded to bf16 -- the two
//     bf16 roundings of the reference's sum(dim=2).sum(dim=1).
//   * Top-k / ordering / in-place compaction as in the window kernel; kept
//     rows go to positions [0, R) of the block table; context_lens[b] = R.
#pragma once
#include "window_compress.cuh"

namespace nkv {

__global__ void __launch_bounds__(kCompressThreads)
query_window_append_kernel(const __nv_bfloat16* __restrict__ q, int64_t q_stride_token,
                           __nv_bfloat16* __restrict__ ring, int num_ring_slots, int num_layers,
                           int window_size, int layer_id, const int32_t* __restrict__ batch_index,
                           const int32_t* __restrict__ ring_slot,
                           const int32_t* __restrict__ ring_pos, int row_vecs) {
  const int j = blockIdx.x;
  const int b = __ldg(batch_index + j);
  const int slot = __ldg(ring_slot + j);
  const int pos = __ldg(ring_pos + j);
  if (b < 0 || slot < 0 || slot >= num_ring_slots || pos < 0 || pos >= window_size ||
      layer_id < 0 || layer_id >= num_layers) {
    if (threadIdx.x == 0) raise_error(NKV_DEVERR_RING_RANGE);
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(q + static_cast<int64_t>(b) * q_stride_token);
  uint4* dst = reinterpret_cast<uint4*>(
      ring + ((static_cast<int64_t>(slot) * num_layers + layer_id) * window_size + pos) *
                 static_cast<int64_t>(row_vecs) * 8);
  for (int i = threadIdx.x; i < row_vecs; i += blockDim.x) dst[i] = __ldg(src + i);
}

struct ThresholdCompressParams {
  const __nv_bfloat16* ring;  // [slots, layers, W, Hq, 128]
  const int32_t* ring_slot_of_selected;
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  int64_t num_blocks;
  const int32_t* block_tables;
  int32_t* context_lens;
  const int32_t* selected;
  int32_t* out_keep_idx;
  float scale;
  int num_ring_slots;
  int num_layers;
  int window;  // W
  int layer_id;
  int max_blocks;
  int S;
  int R;
  int num_q_heads;
  int num_kv_heads;
  int g;
  int block_size;
  int num_keys;      // S - W
  int keys_pad;      // rounded up to kCompressThreads
  int stage_keys;    // 1: key rows staged in shared memory
};

__device__ __forceinline__ float dot128_bf16_f32(const __nv_bfloat16* krow, const float* qrow) {
  const uint4* kv = reinterpret_cast<const uint4*>(krow);
  float acc0 = 0.f, acc1 = 0.f;
#pragma unroll 4
  for (int c = 0; c < kCompressHeadDim / 8; ++c) {
    const uint4 w = kv[c];
    const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int d = c * 8 + 2 * e;
      acc0 = fmaf(qrow[d], __uint_as_float(wv[e] << 16), acc0);
      acc1 = fmaf(qrow[d + 1], __uint_as_float(wv[e] & 0xffff0000u), acc1);
    }
  }
  return acc0 + acc1;
}

__global__ void __launch_bounds__(kCompressThreads, 1)
threshold_compress_kernel(const ThresholdCompressParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const int head = static_cast<int>(cluster.block_rank());
  const int sel_i = blockIdx.y;
  const int g = p.g;
  const int nk = p.num_keys;
  const int kp = p.keys_pad;
  const int bs = p.block_size;
  const int W = p.window;

  __nv_bfloat16* kst = reinterpret_cast<__nv_bfloat16*>(smem);  // [nk][128] if staged
  const size_t kst_bytes = p.stage_keys ? static_cast<size_t>(nk) * kCompressHeadDim * 2 : 0;
  float* qs = reinterpret_cast<float*>(smem + kst_bytes);       // [g][128]
  float* srow = qs + g * kCompressHeadDim;                       // [g][kp]
  float* kacc = srow + g * kp;                                   // [g][kp]
  float* partial = kacc + g * kp;                                // [kp] (cluster-visible)
  uint16_t* keys = reinterpret_cast<uint16_t*>(partial + kp);    // [kp]
  int* final_idx = reinterpret_cast<int*>(keys + kp + (kp & 1));  // [R]
  int* red = final_idx + p.R;                                    // [32]
  __shared__ int s_valid;
  __shared__ int s_start;

  const int b = __ldg(p.selected + sel_i);
  const int64_t bt_row = static_cast<int64_t>(b) * p.max_blocks;
  auto slot_of = [&](int pos) -> int64_t {
    const int bi = pos / bs;
    if (bi < 0 || bi >= p.max_blocks) return -1;
    const int id = __ldg(p.block_tables + bt_row + bi);
    if (id < 0 || id >= p.num_blocks) return -1;
    return static_cast<int64_t>(id) * bs + (pos % bs);
  };

  if (threadIdx.x == 0) {
    const int len = p.context_lens[b];
    s_start = max(len - p.S, 0);
    const int rs = __ldg(p.ring_slot_of_selected + sel_i);
    int valid = (rs >= 0 && rs < p.num_ring_slots && p.layer_id >= 0 && p.layer_id < p.num_layers);
    // every key / source / destination position must resolve to a cache slot
    if (valid && (slot_of(p.S - 1) < 0 || slot_of(s_start + p.S - 1) < 0 || slot_of(0) < 0))
      valid = 0;
    if (!valid && head == 0) raise_error(NKV_DEVERR_COMPRESS_RANGE);
    s_valid = valid;
  }
  __syncthreads();
  const bool valid = s_valid != 0;
  const int start = s_start;

  if (valid) {
    const int rslot = __ldg(p.ring_slot_of_selected + sel_i);
    // stage key rows (positions [0, S - W)) of this kv head
    if (p.stage_keys) {
      for (int i = threadIdx.x; i < nk * 16; i += kCompressThreads) {
        const int t = i >> 4, c = i & 15;
        const int64_t slot = slot_of(t);
        uint4 v = make_uint4(0, 0, 0, 0);
        if (slot >= 0)
          v = reinterpret_cast<const uint4*>(
              p.k_cache + (slot * p.num_kv_heads + head) * kCompressHeadDim)[c];
        reinterpret_cast<uint4*>(kst + static_cast<int64_t>(t) * kCompressHeadDim)[c] = v;
      }
    }
    for (int i = threadIdx.x; i < g * kp; i += kCompressThreads) kacc[i] = 0.f;
    __syncthreads();
    for (int w = 0; w < W; ++w) {
      const __nv_bfloat16* qbase =
          p.ring + ((static_cast<int64_t>(rslot) * p.num_layers + p.layer_id) * W + w) *
                       static_cast<int64_t>(p.num_q_heads) * kCompressHeadDim;
      for (int i = threadIdx.x; i < g * kCompressHeadDim; i += kCompressThreads) {
        const int r = i / kCompressHeadDim, d = i % kCompressHeadDim;
        qs[i] = __bfloat162float(qbase[static_cast<int64_t>(head * g + r) * kCompressHeadDim + d]);
      }
      __syncthreads();
      for (int t = threadIdx.x; t < nk; t += kCompressThreads) {
        const __nv_bfloat16* krow;
        if (p.stage_keys) {
          krow = kst + static_cast<int64_t>(t) * kCompressHeadDim;
        } else {
          const int64_t slot = slot_of(t);
          krow = p.k_cache + (max(slot, int64_t(0)) * p.num_kv_heads + head) * kCompressHeadDim;
        }
        for (int r = 0; r < g; ++r) {
          float v = -INFINITY;
          if (t != 0) v = round_bf16(round_bf16(dot128_bf16_f32(krow, qs + r * kCompressHeadDim)) * p.scale);
          srow[r * kp + t] = v;
        }
      }
      __syncthreads();
      for (int r = 0; r < g; ++r) {
        float* row = srow + r * kp;
        float mx = -INFINITY;
        for (int t = threadIdx.x; t < nk; t += kCompressThreads) mx = fmaxf(mx, row[t]);
        mx = block_max_float(mx, reinterpret_cast<float*>(red));
        float sum = 0.f;
        for (int t = threadIdx.x; t < nk; t += kCompressThreads) {
          const float e = expf(row[t] - mx);
          row[t] = e;
          sum += e;
        }
        sum = block_sum_float(sum, reinterpret_cast<float*>(red));
        for (int t = threadIdx.x; t < nk; t += kCompressThreads)
          kacc[r * kp + t] += round_bf16(row[t] / sum);
      }
      __syncthreads();
    }
    for (int t = threadIdx.x; t < kp; t += kCompressThreads) {
      float s = 0.f;
      if (t < nk)
        for (int r = 0; r < g; ++r) s += round_bf16(kacc[r * kp + t]);
      partial[t] = s;
    }
  }
  cluster.sync();
  if (valid) {
    const int nranks = static_cast<int>(cluster.num_blocks());
    for (int t = threadIdx.x; t < kp; t += kCompressThreads) {
      float s = 0.f;
      for (int c = 0; c < nranks; ++c) s += cluster.map_shared_rank(partial, c)[t];
      keys[t] = (t < nk) ? static_cast<uint16_t>(bf16_key(s)) : 0;
    }
  }
  cluster.sync();
  if (!valid) return;

  const int num_keep = p.R - W - 1;
  if (threadIdx.x == 0) final_idx[0] = 0;
  topk_ascending(keys, nk, num_keep, final_idx + 1, red);
  for (int i = threadIdx.x; i < W; i += kCompressThreads) final_idx[1 + num_keep + i] = p.S - W + i;
  __syncthreads();

  compact_rows_in_order(p.k_cache, p.v_cache, p.num_kv_heads, head, p.R,
                        [&](int i, int64_t& src, int64_t& dst) {
                          src = slot_of(start + final_idx[i]);
                          dst = slot_of(i);
                        });
  if (head == 0) {
    if (threadIdx.x == 0) p.context_lens[b] = p.R;
    if (p.out_keep_idx) {
      for (int i = threadIdx.x; i < p.R; i += kCompressThreads)
        p.out_keep_idx[static_cast<int64_t>(sel_i) * p.R + i] = final_idx[i];
    }
  }
}

}  // namespace nkv
