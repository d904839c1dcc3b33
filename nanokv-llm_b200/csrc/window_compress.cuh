// Periodic window KV compression, fused into one kernel launch per layer:
// score -> importance -> top-k -> in-place compaction -> context_lens update.
// Replaces MyCompressCompact (nanokvllm/layers/compress_utils.py:100-263) with
// its helpers get_tail_window_and_tail_slots (:9-72), gather_kv_by_slots
// (:75-97) and SnapKV (nanokvllm/layers/CompressMethod.py:4-58).
//
// Launch: grid (num_kv_heads, num_selected), one thread-block CLUSTER of
// num_kv_heads CTAs per selected sequence, CTA rank = kv head; two CTAs fit
// on an SM, so 20 sequences x 8 heads run in a single wave.
//   1. Each CTA scores the window keys of its kv head against the g query heads
//      of its GQA group, reproducing the reference's bf16 rounding points:
//      score = bf16(q.k) (exact fp64 accumulation of the exact bf16 products,
//      then float, then bf16, as the reference's CPU matmul rounds),
//      bf16(score * scale), sink key 0 -> -inf, p = bf16(exp(s - max) / sum)
//      per head, and the CTA's fp32 sum of p over its heads.
//   2. Cluster barrier; every CTA reads all partials through distributed shared
//      memory and forms importance = bf16(sum over all local heads), the single
//      rounding of the reference's head sum. One kept set per (sequence, rank).
//   3. Top-k over the bf16 importance keys: a two-pass radix select finds the
//      k-th largest key, ties at the cut are broken towards the lower index
//      (a deterministic refinement of torch.topk's unspecified tie order), and
//      a block scan emits the kept indices in ascending order.
//   4. Compaction of this CTA's kv-head slice of every kept row into the first
//      keep_tokens window slots (compact_rows_pipelined), then the partial
//      tail block after them (slot arithmetic as in the reference).
// No host round trip, no scratch memory, no V traffic for scoring.
#pragma once
#include "compress_common.cuh"

namespace nkv {

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
  uint16_t* out_importance;  // bf16 bits [num_selected][num_keys], or null
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

// Shared-memory bytes of window_compress_kernel<G> (host and device agree).
__host__ __device__ constexpr size_t window_smem_bytes(int G, int keys_pad, int keep_tokens) {
  return sizeof(double) * G * kCompressHeadDim          // q rows as doubles
         + sizeof(float) * static_cast<size_t>(G) * keys_pad  // scores / exp
         + sizeof(float) * keys_pad                       // partial (cluster-visible)
         + sizeof(uint16_t) * (keys_pad + 2)              // bf16 importance keys
         + sizeof(int) * keep_tokens                      // final index list
         + sizeof(int) * kMaxWindowBlocks                 // window block ids
         + sizeof(float) * kReduceSlots                   // reductions
         + sizeof(int) * 256;                             // top-k histogram
}

// Exact q.k over 128 dims for the G query heads of a group: bf16 products are
// exact in fp64 and 128 of them sum exactly for any realistic exponent spread.
template <int G>
__device__ __forceinline__ void dot_rows_fp64(const __nv_bfloat16* krow, const double* qd,
                                              double (&acc)[G]) {
#pragma unroll
  for (int r = 0; r < G; ++r) acc[r] = 0.0;
  const uint4* kv = reinterpret_cast<const uint4*>(krow);
#pragma unroll 2
  for (int c = 0; c < kCompressHeadDim / 8; ++c) {
    const uint4 w = __ldg(kv + c);
    const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
    double kd[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      kd[2 * e] = static_cast<double>(__uint_as_float(wv[e] << 16));
      kd[2 * e + 1] = static_cast<double>(__uint_as_float(wv[e] & 0xffff0000u));
    }
#pragma unroll
    for (int r = 0; r < G; ++r) {
      const double2* qp = reinterpret_cast<const double2*>(qd + r * kCompressHeadDim + c * 8);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const double2 qq = qp[e];
        acc[r] = fma(qq.x, kd[2 * e], acc[r]);
        acc[r] = fma(qq.y, kd[2 * e + 1], acc[r]);
      }
    }
  }
}

template <int G>
__global__ void __launch_bounds__(kCompressThreads, 2)
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

  double* qd = reinterpret_cast<double*>(smem);                    // [G][128]
  float* scores = reinterpret_cast<float*>(qd + G * kCompressHeadDim);  // [G][kp]
  float* partial = scores + G * kp;                                // [kp] (cluster-visible)
  uint16_t* keys = reinterpret_cast<uint16_t*>(partial + kp);      // [kp]
  int* final_idx = reinterpret_cast<int*>(keys + kp + 2);          // [keep_tokens]
  int* wblk = final_idx + p.keep_tokens;                           // [window_blocks]
  float* red = reinterpret_cast<float*>(wblk + kMaxWindowBlocks);  // [kReduceSlots]
  int* hist = reinterpret_cast<int*>(red + kReduceSlots);          // [256]
  __shared__ int s_valid;
  __shared__ int s_tail_block;

  // The kv heads of a sequence are the CTAs of one cluster (their partial
  // sums meet in distributed shared memory). A launch that lost its
  // clusters (%cluster_nctarank 1) cannot form them: flag it and write
  // nothing (the condition is uniform, so no CTA waits at a cluster barrier).
  if (static_cast<int>(cluster.num_blocks()) != p.num_kv_heads) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) raise_error(NKV_DEVERR_LAUNCH_SHAPE);
    return;
  }
  const int b = __ldg(p.selected + sel_i);
  // -1: an unused entry of a fixed-size selection list (device-side
  // selection, graph replay); uniform across the cluster, before any
  // cluster barrier
  if (b < 0) return;
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
  // q rows of this GQA group as doubles (rows >= g are zero).
  for (int i = threadIdx.x; i < G * kCompressHeadDim; i += kCompressThreads) {
    const int r = i / kCompressHeadDim, d = i % kCompressHeadDim;
    qd[i] = (r < g) ? static_cast<double>(__bfloat162float(
                          p.q[static_cast<int64_t>(b) * p.q_stride_token +
                              static_cast<int64_t>(head * g + r) * kCompressHeadDim + d]))
                    : 0.0;
  }
  __syncthreads();
  const bool valid = s_valid != 0;  // identical in every CTA of the cluster

  if (valid) {
    // 1. scores, one thread per key row
    for (int t = threadIdx.x; t < kp; t += kCompressThreads) {
      if (t < nk) {
        const int64_t slot = static_cast<int64_t>(wblk[t / bs]) * bs + (t % bs);
        double acc[G];
        dot_rows_fp64<G>(p.k_cache + (slot * p.num_kv_heads + head) * kCompressHeadDim, qd, acc);
#pragma unroll
        for (int r = 0; r < G; ++r) {
          const float s = round_bf16(static_cast<float>(acc[r]));
          scores[r * kp + t] = (t == 0) ? -INFINITY : round_bf16(s * p.scale);
        }
      } else {
#pragma unroll
        for (int r = 0; r < G; ++r) scores[r * kp + t] = -INFINITY;
      }
    }
    __syncthreads();
    // 2. softmax of every head over the keys (bf16 output), fp32 group sum
    float mx[G], sm[G];
#pragma unroll
    for (int r = 0; r < G; ++r) mx[r] = -INFINITY;
    for (int t = threadIdx.x; t < nk; t += kCompressThreads) {
#pragma unroll
      for (int r = 0; r < G; ++r) mx[r] = fmaxf(mx[r], scores[r * kp + t]);
    }
    block_reduce_vec<G, true>(mx, red);
#pragma unroll
    for (int r = 0; r < G; ++r) sm[r] = 0.f;
    for (int t = threadIdx.x; t < nk; t += kCompressThreads) {
#pragma unroll
      for (int r = 0; r < G; ++r) {
        const float e = expf(scores[r * kp + t] - mx[r]);
        scores[r * kp + t] = e;
        sm[r] += e;
      }
    }
    block_reduce_vec<G, false>(sm, red);
    for (int t = threadIdx.x; t < kp; t += kCompressThreads) {
      float s = 0.f;
      if (t < nk) {
#pragma unroll
        for (int r = 0; r < G; ++r)
          if (r < g) s += round_bf16(scores[r * kp + t] / sm[r]);
      }
      partial[t] = s;
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
      if (head == 0 && p.out_importance != nullptr && t < nk)
        p.out_importance[static_cast<int64_t>(sel_i) * nk + t] = keys[t];
    }
  }
  cluster.sync();  // no CTA may leave while a peer still reads its partials
  if (!valid) return;

  // 4. top-k and the final index list [0] + kept + [last obs_window tokens].
  const int num_keep = p.keep_tokens - 1 - p.obs_window;
  if (threadIdx.x == 0) final_idx[0] = 0;
  topk_ascending(keys, nk, num_keep, final_idx + 1, reinterpret_cast<int*>(red), hist);
  for (int i = threadIdx.x; i < p.obs_window; i += kCompressThreads)
    final_idx[1 + num_keep + i] = window_tokens - p.obs_window + i;
  __syncthreads();

  // 5. compaction of this head's slice, then the tail block.
  const int* wb = wblk;
  const int keep_tokens = p.keep_tokens;
  compact_rows_pipelined(p.k_cache, p.v_cache, p.num_kv_heads, head, keep_tokens,
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
    compact_rows_pipelined(p.k_cache, p.v_cache, p.num_kv_heads, head, tail_len,
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

// Periodic-compression selection on the device, so a compression step can
// be replayed from a CUDA graph: the rule of the reference's prepare_decode
// (nanokvllm/engine/model_runner.py:305-321) -- row b (physical length L =
// context_lens[b]) is skipped when L % block_size == block_size - 1 and is
// eligible when tail_uncompressed[b] >= window_blocks * block_size and
// L / block_size >= window_blocks; the FIRST topk eligible rows in batch
// order are selected. One CTA; writes selected[0, topk) (-1 padded), the
// count, and a copy of context_lens as the step's base lengths.
constexpr int kSelectThreads = kCompressThreads;  // block_* helpers assume this size

struct WindowSelectParams {
  const int32_t* context_lens;
  const int32_t* tail_uncompressed;
  int32_t* selected;    // [topk]
  int32_t* count;       // [1] or null
  int32_t* base_lens;   // [batch] or null
  int batch;
  int block_size;
  int window_blocks;
  int topk;
};

__global__ void __launch_bounds__(kSelectThreads)
window_select_kernel(const WindowSelectParams p) {
  __shared__ int red[kCompressWarps];
  const int window_tokens = p.window_blocks * p.block_size;
  for (int i = threadIdx.x; i < p.topk; i += kSelectThreads) p.selected[i] = -1;
  __syncthreads();
  int taken = 0;  // eligible rows in earlier chunks
  for (int base = 0; base < p.batch; base += kSelectThreads) {
    const int b = base + threadIdx.x;
    int elig = 0;
    if (b < p.batch) {
      const int L = __ldg(p.context_lens + b);
      if (p.base_lens != nullptr) p.base_lens[b] = L;
      if (L % p.block_size != p.block_size - 1 && __ldg(p.tail_uncompressed + b) >= window_tokens &&
          L / p.block_size >= p.window_blocks)
        elig = 1;
    }
    const int before = block_excl_scan(elig, red);
    const int pos = taken + before;
    if (elig && pos < p.topk) p.selected[pos] = b;
    taken += block_sum_int(elig, red);
  }
  if (threadIdx.x == 0 && p.count != nullptr) p.count[0] = min(taken, p.topk);
}

}  // namespace nkv
