// Periodic window KV compression, fused into one kernel launch per layer:
// score -> importance -> top-k -> in-place compaction -> context_lens update.
// Replaces MyCompressCompact (nanokvllm/layers/compress_utils.py:100-263) with
// its helpers get_tail_window_and_tail_slots (:9-72), gather_kv_by_slots
// (:75-97) and SnapKV (nanokvllm/layers/CompressMethod.py:4-58).
//
// Launch: grid (num_kv_heads, num_selected), one thread-block CLUSTER of
// num_kv_heads CTAs per selected sequence, CTA rank = kv head.
//   1. Each CTA scores the window keys of its kv head against the g query heads
//      of its GQA group, reproducing the reference's bf16 rounding points:
//      score = bf16(q.k) (exact fp64 accumulation, then float, then bf16, as the
//      reference's CPU matmul rounds), bf16(score * scale), sink key 0 -> -inf,
//      p = bf16(exp(s - max) / sum) per head, and the CTA's fp32 partial sum of p
//      over its heads.
//   2. Cluster barrier; every CTA reads all partials through distributed shared
//      memory and forms importance = bf16(sum over all local heads), the single
//      rounding of the reference's head sum. One kept set per (sequence, rank).
//   3. Top-k over the bf16 importance keys: a 16-step bitwise search finds the
//      k-th largest key, ties at the cut are broken towards the lower index
//      (a deterministic refinement of torch.topk's unspecified tie order), and
//      a block scan emits the kept indices in ascending order.
//   4. Compaction of this CTA's kv-head slice of every kept row into the first
//      keep_tokens window slots, 64 rows at a time: a chunk's sources are all
//      read before any of its destinations is written, and since the i-th
//      kept index is >= i no later chunk can lose a source. The tail partial
//      block follows the kept rows (slot arithmetic as in the reference).
// No host round trip, no scratch memory, no V traffic for scoring.
#pragma once
#include <cooperative_groups.h>

#include "nkv_common.cuh"

namespace nkv {

namespace cg = cooperative_groups;

constexpr int kCompressThreads = 256;
constexpr int kCompressWarps = kCompressThreads / 32;
constexpr int kCompressHeadDim = 128;
constexpr int kCompactChunkRows = 64;
constexpr int kMaxWindowBlocks = 64;

struct WindowCompressParams {
  const __nv_bfloat16* q;
  int64_t q_stride_token;
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  int64_t num_blocks;
  const int32_t* block_tables;
  const int32_t* base_lens;
  int32_t* context_lens;
  const int32_t* selected;
  int32_t* out_keep_idx;
  int32_t* out_new_lens;
  float scale;
  int max_blocks;
  int window_blocks;
  int keep_tokens;
  int obs_window;
  int num_kv_heads;
  int g;
  int block_size;
  int num_keys;     // window_tokens - obs_window
  int keys_pad;     // num_keys rounded up to kCompressThreads
};

// ---------------------------------------------------------------- block helpers
__device__ __forceinline__ int block_sum_int(int v, int* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = __reduce_add_sync(0xffffffffu, v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  int tot = 0;
#pragma unroll
  for (int w = 0; w < kCompressWarps; ++w) tot += red[w];
  __syncthreads();
  return tot;
}

__device__ __forceinline__ float block_max_float(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float m = red[0];
#pragma unroll
  for (int w = 1; w < kCompressWarps; ++w) m = fmaxf(m, red[w]);
  __syncthreads();
  return m;
}

__device__ __forceinline__ float block_sum_float(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < kCompressWarps; ++w) s += red[w];
  __syncthreads();
  return s;
}

// Exclusive prefix sum over threads in index order.
__device__ __forceinline__ int block_excl_scan(int v, int* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) red[warp] = x;
  __syncthreads();
  int before = 0;
  for (int w = 0; w < warp; ++w) before += red[w];
  __syncthreads();
  return before + x - v;
}

// Bit pattern of a non-negative bf16 value: monotone in the value.
__device__ __forceinline__ uint32_t bf16_key(float v) {
  return static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v)));
}

// Selects the `k` largest of keys[0, n) (ties -> lower index) and writes their
// indices, ascending, to out[0, k). Keys live in shared memory. Each thread
// owns a contiguous index range so that scans follow index order.
__device__ void topk_ascending(const uint16_t* keys, int n, int k, int* out, int* red) {
  const int per = (n + kCompressThreads - 1) / kCompressThreads;
  const int lo = threadIdx.x * per;
  const int hi = min(lo + per, n);
  uint32_t prefix = 0;
  for (int bit = 15; bit >= 0; --bit) {
    const uint32_t cand = prefix | (1u << bit);
    int c = 0;
    for (int t = lo; t < hi; ++t) c += (keys[t] >= cand) ? 1 : 0;
    if (block_sum_int(c, red) >= k) prefix = cand;
  }
  // prefix is now the k-th largest key.
  int gt = 0, eq = 0;
  for (int t = lo; t < hi; ++t) {
    gt += (keys[t] > prefix) ? 1 : 0;
    eq += (keys[t] == prefix) ? 1 : 0;
  }
  const int total_gt = block_sum_int(gt, red);
  const int need_eq = k - total_gt;
  const int eq_before = block_excl_scan(eq, red);
  int kept = 0;
  {
    int e = eq_before;
    for (int t = lo; t < hi; ++t) {
      const bool is_eq = keys[t] == prefix;
      kept += (keys[t] > prefix || (is_eq && e < need_eq)) ? 1 : 0;
      e += is_eq ? 1 : 0;
    }
  }
  int pos = block_excl_scan(kept, red);
  {
    int e = eq_before;
    for (int t = lo; t < hi; ++t) {
      const bool is_eq = keys[t] == prefix;
      if (keys[t] > prefix || (is_eq && e < need_eq)) out[pos++] = t;
      e += is_eq ? 1 : 0;
    }
  }
  __syncthreads();
}

// Copies rows src_slot[i] -> dst_slot[i] (this CTA's kv-head slice, K and V)
// for i in [0, n), 64 rows per chunk, all reads of a chunk before its writes.
template <typename SlotFn>
__device__ void compact_rows_in_order(__nv_bfloat16* k_cache, __nv_bfloat16* v_cache,
                                      int num_kv_heads, int head, int n, SlotFn slots) {
  const int t = threadIdx.x;
  const int row_in_chunk = t >> 2;  // 64 rows x 4 threads
  const int quarter = t & 3;        // 4 x 64 bytes of a 256-byte head row
  for (int base = 0; base < n; base += kCompactChunkRows) {
    const int i = base + row_in_chunk;
    int64_t src = -1, dst = -1;
    if (i < n) slots(i, src, dst);
    const bool move = (i < n) && src >= 0 && dst >= 0 && src != dst;
    uint4 kr[4], vr[4];
    if (move) {
      const uint4* ks = reinterpret_cast<const uint4*>(
          k_cache + (src * num_kv_heads + head) * kCompressHeadDim) + quarter * 4;
      const uint4* vs = reinterpret_cast<const uint4*>(
          v_cache + (src * num_kv_heads + head) * kCompressHeadDim) + quarter * 4;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        kr[u] = ks[u];
        vr[u] = vs[u];
      }
    }
    __syncthreads();
    if (move) {
      uint4* kd = reinterpret_cast<uint4*>(k_cache + (dst * num_kv_heads + head) * kCompressHeadDim) +
                  quarter * 4;
      uint4* vd = reinterpret_cast<uint4*>(v_cache + (dst * num_kv_heads + head) * kCompressHeadDim) +
                  quarter * 4;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        kd[u] = kr[u];
        vd[u] = vr[u];
      }
    }
    __syncthreads();
  }
}

// Dot product of a bf16 key row (128 dims) with fp32-held bf16 query rows,
// accumulated exactly in fp64 and rounded like the reference's CPU bf16 matmul
// (double -> float -> bf16, round to nearest even at each step).
__device__ __forceinline__ void score_key_row(const __nv_bfloat16* krow, const float* qs, int g,
                                              float* out_scores /*[g]*/) {
  double acc[16];
#pragma unroll
  for (int r = 0; r < 16; ++r) acc[r] = 0.0;
  const uint4* kv = reinterpret_cast<const uint4*>(krow);
#pragma unroll 4
  for (int c = 0; c < kCompressHeadDim / 8; ++c) {
    const uint4 w = kv[c];
    const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const double k0 = static_cast<double>(__uint_as_float(wv[e] << 16));
      const double k1 = static_cast<double>(__uint_as_float(wv[e] & 0xffff0000u));
      const int d = c * 8 + 2 * e;
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        if (r < g) {
          acc[r] = fma(static_cast<double>(qs[r * kCompressHeadDim + d]), k0, acc[r]);
          acc[r] = fma(static_cast<double>(qs[r * kCompressHeadDim + d + 1]), k1, acc[r]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < 16; ++r) {
    if (r < g) out_scores[r] = round_bf16(static_cast<float>(acc[r]));
  }
}

__global__ void __launch_bounds__(kCompressThreads, 1)
window_compress_kernel(const WindowCompressParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const int head = static_cast<int>(cluster.block_rank());  // == blockIdx.x
  const int sel_i = blockIdx.y;
  const int g = p.g;
  const int nk = p.num_keys;
  const int kp = p.keys_pad;
  const int bs = p.block_size;
  const int window_tokens = p.window_blocks * bs;

  float* qs = reinterpret_cast<float*>(smem);                      // [g][128]
  float* scores = qs + g * kCompressHeadDim;                       // [g][kp]
  float* partial = scores + g * kp;                                // [kp]  (cluster-visible)
  uint16_t* keys = reinterpret_cast<uint16_t*>(partial + kp);      // [kp]
  int* final_idx = reinterpret_cast<int*>(keys + kp + (kp & 1));   // [keep_tokens]
  int* wblk = final_idx + p.keep_tokens;                           // [window_blocks]
  int* red = wblk + kMaxWindowBlocks;                              // [32]
  __shared__ int s_valid;
  __shared__ int s_tail_block;

  const int b = __ldg(p.selected + sel_i);
  const int L0 = __ldg(p.base_lens + b);
  const int full_blocks = L0 / bs;
  const int tail_len = L0 % bs;

  if (threadIdx.x == 0) {
    int valid = (full_blocks >= p.window_blocks) ? 1 : 0;
    for (int j = 0; j < p.window_blocks && valid; ++j) {
      const int bi = full_blocks - p.window_blocks + j;
      const int id = (bi < p.max_blocks)
                         ? __ldg(p.block_tables + static_cast<int64_t>(b) * p.max_blocks + bi)
                         : -1;
      if (id < 0 || id >= p.num_blocks) valid = 0;
      wblk[j] = id;
    }
    int tb = -1;
    if (valid && tail_len > 0) {
      const int ti = min(full_blocks, p.max_blocks - 1);
      tb = __ldg(p.block_tables + static_cast<int64_t>(b) * p.max_blocks + ti);
      if (tb < 0 || tb >= p.num_blocks) valid = 0;
    }
    if (!valid && head == 0) raise_error(NKV_DEVERR_COMPRESS_RANGE);
    s_valid = valid;
    s_tail_block = tb;
  }
  // q rows of this GQA group, as fp32 copies of the bf16 inputs.
  for (int i = threadIdx.x; i < g * kCompressHeadDim; i += kCompressThreads) {
    const int r = i / kCompressHeadDim, d = i % kCompressHeadDim;
    qs[i] = __bfloat162float(
        p.q[static_cast<int64_t>(b) * p.q_stride_token +
            static_cast<int64_t>(head * g + r) * kCompressHeadDim + d]);
  }
  __syncthreads();
  const bool valid = s_valid != 0;  // identical in every CTA of the cluster

  if (valid) {
    // 1. scores: one thread per key row.
    for (int t = threadIdx.x; t < kp; t += kCompressThreads) {
      float sc[16];
      if (t < nk) {
        const int64_t slot = static_cast<int64_t>(wblk[t / bs]) * bs + (t % bs);
        score_key_row(p.k_cache + (slot * p.num_kv_heads + head) * kCompressHeadDim, qs, g, sc);
      }
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        if (r < g) {
          float v = -INFINITY;
          if (t < nk && t != 0) v = round_bf16(sc[r] * p.scale);
          scores[r * kp + t] = v;
        }
      }
    }
    __syncthreads();
    // 2. per-head softmax over the keys (bf16 output), fp32 sum over the group.
    for (int t = threadIdx.x; t < kp; t += kCompressThreads) partial[t] = 0.f;
    __syncthreads();
    for (int r = 0; r < g; ++r) {
      float* row = scores + r * kp;
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
      for (int t = threadIdx.x; t < nk; t += kCompressThreads) {
        partial[t] += round_bf16(row[t] / sum);
      }
      __syncthreads();
    }
  }
  cluster.sync();
  if (valid) {
    // 3. importance = bf16(sum over all local heads), read across the cluster.
    const int nranks = static_cast<int>(cluster.num_blocks());
    for (int t = threadIdx.x; t < kp; t += kCompressThreads) {
      float s = 0.f;
      for (int c = 0; c < nranks; ++c) s += cluster.map_shared_rank(partial, c)[t];
      keys[t] = (t < nk) ? static_cast<uint16_t>(bf16_key(s)) : 0;
    }
  }
  cluster.sync();  // no CTA may leave while a peer still reads its partials
  if (!valid) return;

  // 4. top-k and the final index list [0] + kept + [last obs_window tokens].
  const int num_keep = p.keep_tokens - 1 - p.obs_window;
  if (threadIdx.x == 0) final_idx[0] = 0;
  topk_ascending(keys, nk, num_keep, final_idx + 1, red);
  for (int i = threadIdx.x; i < p.obs_window; i += kCompressThreads)
    final_idx[1 + num_keep + i] = window_tokens - p.obs_window + i;
  __syncthreads();

  // 5. compaction of this head's slice.
  const int* wb = wblk;
  const int keep_tokens = p.keep_tokens;
  compact_rows_in_order(p.k_cache, p.v_cache, p.num_kv_heads, head, keep_tokens,
                        [&](int i, int64_t& src, int64_t& dst) {
                          const int s = final_idx[i];
                          src = static_cast<int64_t>(wb[s / bs]) * bs + (s % bs);
                          dst = static_cast<int64_t>(wb[i / bs]) * bs + (i % bs);
                        });
  if (tail_len > 0) {
    const int64_t last_dst =
        static_cast<int64_t>(wb[(keep_tokens - 1) / bs]) * bs + ((keep_tokens - 1) % bs);
    const int64_t num_slots = p.num_blocks * bs;
    const int64_t tail_block = s_tail_block;
    compact_rows_in_order(p.k_cache, p.v_cache, p.num_kv_heads, head, tail_len,
                          [&](int j, int64_t& src, int64_t& dst) {
                            src = tail_block * bs + j;
                            dst = last_dst + 1 + j;
                            if (dst >= num_slots) {
                              raise_error(NKV_DEVERR_COMPRESS_RANGE);
                              dst = -1;
                            }
                          });
  }

  // 6. metadata: new length (every layer writes the same value) and outputs.
  const int new_len = L0 - window_tokens + keep_tokens;
  if (head == 0) {
    if (threadIdx.x == 0) {
      p.context_lens[b] = new_len;
      if (p.out_new_lens) p.out_new_lens[sel_i] = new_len;
    }
    if (p.out_keep_idx) {
      for (int i = threadIdx.x; i < keep_tokens; i += kCompressThreads)
        p.out_keep_idx[static_cast<int64_t>(sel_i) * keep_tokens + i] = final_idx[i];
    }
  }
}

}  // namespace nkv
