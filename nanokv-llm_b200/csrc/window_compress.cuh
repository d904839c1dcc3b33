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
//      then float, then bf16: the exactly rounded score), bf16(score *
//      scale), sink key 0 -> -inf, p = bf16(exp(s - max) / sum) per head, and
//      the CTA's fp32 sum of p over its heads. The window's K rows of this
//      head stream through a ring of four 64-token tiles (TMA, 128-byte
//      swizzle, no multicast, kept in L2 for the compaction that re-reads the
//      kept rows); each pair of warps owns one ring stage -- its leader
//      refills each 64-dim half of it as soon as both warps are done with
//      that half, while they score the other -- and each thread
//      scores four keys over a quarter of the dims from shared memory
//      (conflict-free through the swizzle; each q load, a broadcast, feeds
//      eight fp64 FMAs), the quarters summed by a shuffle reduce-scatter.
//   2. Cluster barrier; every CTA reads all partials through distributed shared
//      memory and forms importance = bf16(sum over all local heads), the single
//      rounding of the reference's head sum. One kept set per (sequence, rank).
//   3. Top-k over the bf16 importance keys: a two-pass radix select finds the
//      k-th largest key, ties at the cut are broken towards the lower index
//      (a deterministic refinement of torch.topk's unspecified tie order), and
//      a block scan emits the kept indices in ascending order.
//   4. Compaction of this CTA's kv-head slice of every kept row into the first
//      keep_tokens window slots, then the partial tail block after them (slot
//      arithmetic as in the reference), by bulk asynchronous copies staged
//      in the K ring (compact_rows_bulk).
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

constexpr int kWinTileTokens = 64;                    // tokens per K tile
constexpr int kWinStages = 4;                         // ring stages = warp pairs
constexpr int kWinHalfBytes = kWinTileTokens * 128;   // 64 dims x 64 tokens, bf16
constexpr int kWinTileBytes = 2 * kWinHalfBytes;      // 16 KB
constexpr int kWinRingBytes = kWinStages * kWinTileBytes + 64;  // + 2 barriers per stage
static_assert(kWinStages * 64 == kCompressThreads, "one warp pair (64 keys) per stage");
// Compaction: rows per chunk of the bulk copies; two chunks of K and V rows
// fill the K ring, which scoring no longer uses by then.
constexpr int kWinBulkRows = 64;
static_assert(2 * 2 * kWinBulkRows * 256 <= kWinStages * kWinTileBytes, "chunks fit the ring");
// Keys per thread in the scoring loop (and dim ranges per key), as many as
// the kWinSplit x G fp64 sums leave registers for without spilling.
template <int G>
constexpr int kWinSplit = G <= 4 ? 4 : (G <= 8 ? 2 : 1);

// Shared-memory bytes of window_compress_kernel<G> (host and device agree):
// the K ring (1024-byte aligned, hence the slack) and the layout after it.
__host__ __device__ constexpr size_t window_smem_bytes(int G, int keys_pad, int keep_tokens) {
  return 1024 + kWinRingBytes
         + sizeof(double) * G * kCompressHeadDim          // q rows as doubles
         + sizeof(float) * static_cast<size_t>(G) * keys_pad  // scores / exp
         + sizeof(float) * keys_pad                       // partial (cluster-visible)
         + sizeof(uint16_t) * (keys_pad + 2)              // bf16 importance keys
         + sizeof(int) * keep_tokens                      // final index list
         + sizeof(int) * kMaxWindowBlocks                 // window block ids
         + sizeof(float) * kReduceSlots                   // reductions
         + sizeof(int) * 256;                             // top-k histogram
}

__device__ __forceinline__ void pair_barrier(int pair) {
  asm volatile("bar.sync %0, 64;" ::"r"(1 + pair) : "memory");
}

template <int G>
__global__ void __launch_bounds__(kCompressThreads, 2)
window_compress_kernel(const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const WindowCompressParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + kWinStages * kWinTileBytes);
  uint8_t* smem = ring + kWinRingBytes;
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
  __shared__ int s_abort;           // a K tile never landed (cluster-visible)
  __shared__ int s_pair_abort[kWinStages];
  __shared__ alignas(8) uint64_t s_cbar[2];  // compaction chunk barriers

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
    s_abort = 0;
    for (int st = 0; st < kWinStages; ++st) {
      mbar_init(smem_u32(&full[2 * st]), 1);
      mbar_init(smem_u32(&full[2 * st + 1]), 1);
      s_pair_abort[st] = 0;
    }
    fence_barrier_init();
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
    // 1. scores: tile j (tokens [64 j, 64 j + 64) of the window, two 64-dim
    // halves of 64 rows x 128 bytes) lands in ring stage j % 4, which warp
    // pair j % 4 consumes, half by half.
    const int ntiles = window_tokens / kWinTileTokens;
    const int tiles_per_block = bs / kWinTileTokens;
    const int pair = threadIdx.x >> 6;
    const int tp = threadIdx.x & 63;
    const bool pair_leader = tp == 0;
    uint8_t* stage = ring + pair * kWinTileBytes;
    // one barrier per 64-dim half of the stage: a half is refilled as soon
    // as both warps are done with it, while they score the other half
    const uint32_t fb0 = smem_u32(&full[2 * pair]);
    const uint32_t fb1 = smem_u32(&full[2 * pair + 1]);
    int issued[2] = {0, 0}, landed[2] = {0, 0};
    auto issue_half = [&](int j, int h) {
      const int slot0 = wblk[j / tiles_per_block] * bs + (j % tiles_per_block) * kWinTileTokens;
      const uint32_t fb = h ? fb1 : fb0;
      mbar_arrive_expect_tx(fb, kWinHalfBytes);
      tma_load_3d(smem_u32(stage) + h * kWinHalfBytes, &tm_k, fb, 64 * h, head, slot0,
                  l2_policy_evict_last());
    };
    if (pair_leader && pair < ntiles) {
      prefetch_tmap(&tm_k);
      issue_half(pair, 0);
      issue_half(pair, 1);
    }
    if (pair < ntiles) issued[0] = issued[1] = 1;  // every thread tracks the leader's loads
    if (threadIdx.x == 32) {
      // Every K tile of the window starts moving into L2 now, so the ring's
      // refills find it there instead of waiting on DRAM one tile at a time.
      prefetch_tmap(&tm_v);
      for (int jj = kWinStages; jj < ntiles; ++jj) {
        const int slot0 = wblk[jj / tiles_per_block] * bs + (jj % tiles_per_block) * kWinTileTokens;
        tma_prefetch_l2_3d(&tm_k, 0, head, slot0);
        tma_prefetch_l2_3d(&tm_k, 64, head, slot0);
      }
    }
    // Each thread scores kWinSplit keys of the tile over 128 / kWinSplit dims:
    // the lanes of a warp form kWinSplit parts of kLanes lanes, part p taking
    // the 8-dim chunks c = p + kWinSplit * jj (half of them in each 64-dim
    // half) of keys kg + kKeyStride * kk. A q load (one address per 8-lane
    // phase: a broadcast) then feeds 2 * kWinSplit fp64 FMAs, and the K reads
    // of a phase hit 8 distinct swizzled chunks. The parts' sums meet by a
    // shuffle reduce-scatter that leaves lane part p with key kk = p (the sum
    // of exact products does not depend on its order at the precision kept).
    constexpr int kSplit = kWinSplit<G>;
    constexpr int kLanes = 32 / kSplit;
    constexpr int kKeyStride = kWinTileTokens / kSplit;
    constexpr int kChunks = (kCompressHeadDim / 8) / kSplit;
    const int lane = tp & 31;
    const int part = lane / kLanes;
    const int kg = (tp >> 5) * kLanes + lane % kLanes;
    bool aborted = false;
    int j = pair;
    for (; j < ntiles; j += kWinStages) {
      double acc[kSplit][G];
#pragma unroll
      for (int kk = 0; kk < kSplit; ++kk)
#pragma unroll
        for (int r = 0; r < G; ++r) acc[kk][r] = 0.0;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (!mbar_wait_bounded(h ? fb1 : fb0, landed[h] & 1)) s_pair_abort[pair] = 1;
        pair_barrier(pair);
        if (s_pair_abort[pair]) {  // uniform across the pair
          aborted = true;
          break;
        }
        ++landed[h];
        const uint8_t* half = stage + h * kWinHalfBytes;
#pragma unroll 1
        for (int jj = h * (kChunks / 2); jj < (h + 1) * (kChunks / 2); ++jj) {
          const int c = part + kSplit * jj;  // c >> 3 == h
          uint4 w[kSplit];
#pragma unroll
          for (int kk = 0; kk < kSplit; ++kk) {
            const int row = kg + kKeyStride * kk;
            w[kk] = *reinterpret_cast<const uint4*>(half + row * 128 + (((c & 7) ^ (row & 7)) << 4));
          }
          const double2* qp = reinterpret_cast<const double2*>(qd + c * 8);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            double kd[kSplit][2];
#pragma unroll
            for (int kk = 0; kk < kSplit; ++kk) {
              const uint32_t wv = e == 0 ? w[kk].x : e == 1 ? w[kk].y : e == 2 ? w[kk].z : w[kk].w;
              kd[kk][0] = static_cast<double>(__uint_as_float(wv << 16));
              kd[kk][1] = static_cast<double>(__uint_as_float(wv & 0xffff0000u));
            }
#pragma unroll
            for (int r = 0; r < G; ++r) {
              const double2 qq = qp[r * (kCompressHeadDim / 2) + e];
#pragma unroll
              for (int kk = 0; kk < kSplit; ++kk) {
                acc[kk][r] = fma(qq.x, kd[kk][0], acc[kk][r]);
                acc[kk][r] = fma(qq.y, kd[kk][1], acc[kk][r]);
              }
            }
          }
        }
        pair_barrier(pair);  // both warps are done with this half of the stage
        if (j + kWinStages < ntiles) {
          if (pair_leader) issue_half(j + kWinStages, h);
          ++issued[h];
        }
      }
      if (aborted) break;
      // reduce-scatter: level l pairs slots (2s, 2s + 1) (key bit l 0 / 1);
      // a lane keeps the key whose bit l matches its part's bit l
#pragma unroll
      for (int l = 0; (1 << l) < kSplit; ++l) {
        const bool hi = ((part >> l) & 1) != 0;
        const int mask = kLanes << l;
#pragma unroll
        for (int s = 0; s < (kSplit >> (l + 1)); ++s) {
#pragma unroll
          for (int r = 0; r < G; ++r) {
            const double a = acc[2 * s][r], b = acc[2 * s + 1][r];
            const double other = __shfl_xor_sync(0xffffffffu, hi ? a : b, mask);
            acc[s][r] = (hi ? b : a) + other;
          }
        }
      }
      const int t = j * kWinTileTokens + kg + kKeyStride * part;
      if (t < kp) {
#pragma unroll
        for (int r = 0; r < G; ++r) {
          const double sum = acc[0][r];
          const float sc = round_bf16(static_cast<float>(sum));
          scores[r * kp + t] = (t == 0 || t >= nk) ? -INFINITY : round_bf16(sc * p.scale);
        }
      }
    }
    if (pair_leader && !aborted) {
      // This pair is done with its K tiles, and every K load of the window
      // is requested: the V rows and the tail block the compaction reads
      // start moving into L2 now (a quarter per pair; after K, which the
      // scoring waits on, had DRAM first) while the softmax, the importance
      // and the top-k run.
      for (int jj = pair; jj < ntiles; jj += kWinStages) {
        const int slot0 = wblk[jj / tiles_per_block] * bs + (jj % tiles_per_block) * kWinTileTokens;
        tma_prefetch_l2_3d(&tm_v, 0, head, slot0);
        tma_prefetch_l2_3d(&tm_v, 64, head, slot0);
      }
      for (int t0 = pair * kWinTileTokens; t0 < tail_len; t0 += kWinStages * kWinTileTokens) {
        const int slot0 = s_tail_block * bs + t0;
        tma_prefetch_l2_3d(&tm_k, 0, head, slot0);
        tma_prefetch_l2_3d(&tm_k, 64, head, slot0);
        tma_prefetch_l2_3d(&tm_v, 0, head, slot0);
        tma_prefetch_l2_3d(&tm_v, 64, head, slot0);
      }
    }
    if (aborted && pair_leader) {
      // a half never landed: wait (bounded) for the loads still in flight,
      // then the cluster skips this sequence
#pragma unroll
      for (int h = 0; h < 2; ++h)
        if (issued[h] > landed[h]) mbar_wait_bounded(h ? fb1 : fb0, landed[h] & 1);
      s_abort = 1;
    }
    // keys past the window (padding) never win
    for (int t = window_tokens + threadIdx.x; t < kp; t += kCompressThreads) {
#pragma unroll
      for (int r = 0; r < G; ++r) scores[r * kp + t] = -INFINITY;
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
  // a CTA whose K ring gave up makes the whole sequence skip (no kept set is
  // formed from an incomplete importance)
  bool run = valid;
  if (valid) {
    for (int c = 0; c < static_cast<int>(cluster.num_blocks()); ++c)
      run = run && *cluster.map_shared_rank(&s_abort, c) == 0;
  }
  if (run) {
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
  if (!run) return;

  // 4. top-k and the final index list [0] + kept + [last obs_window tokens].
  const int num_keep = p.keep_tokens - 1 - p.obs_window;
  if (threadIdx.x == 0) final_idx[0] = 0;
  topk_ascending(keys, nk, num_keep, final_idx + 1, reinterpret_cast<int*>(red), hist);
  for (int i = threadIdx.x; i < p.obs_window; i += kCompressThreads)
    final_idx[1 + num_keep + i] = window_tokens - p.obs_window + i;
  __syncthreads();

  // 5. compaction of this head's slice, then the tail block.
  // The kept rows, then the tail rows (to dst_keep[-1] + 1 + j in slot
  // arithmetic), as one list: a tail row is stored only after every kept
  // row's load has landed, and no tail destination is a later row's source.
  const int* wb = wblk;
  const int keep_tokens = p.keep_tokens;
  const int64_t last_dst =
      static_cast<int64_t>(wb[(keep_tokens - 1) / bs]) * bs + ((keep_tokens - 1) % bs);
  const int64_t num_slots = p.num_blocks * bs;
  const int64_t tail_block = s_tail_block;
  if (!compact_rows_bulk<kCompressThreads, kWinBulkRows>(
          p.k_cache, p.v_cache, p.num_kv_heads, head, keep_tokens + tail_len,
          [&](int i, int64_t& src, int64_t& dst) {
            if (i < keep_tokens) {
              const int s = final_idx[i];
              src = static_cast<int64_t>(wb[s / bs]) * bs + (s % bs);
              dst = static_cast<int64_t>(wb[i / bs]) * bs + (i % bs);
            } else {
              const int j = i - keep_tokens;
              src = tail_block * bs + j;
              dst = last_dst + 1 + j;
              if (dst >= num_slots) {
                raise_error(NKV_DEVERR_COMPRESS_RANGE);
                dst = -1;
              }
            }
          },
          ring, s_cbar))
    return;  // a row never landed (flagged): no metadata from this CTA

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
