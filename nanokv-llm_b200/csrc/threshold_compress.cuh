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
// threshold_compress_kernel<G> replaces MyCompressCompact
// (KvChat/layers/compress_utils.py:10-171) with TritonGetKVForComp (:218-252)
// and SnapKV(window=W, num_keep=R-W-1) (KvChat/layers/CompressMethod.py:4-58).
// Launch: grid (num_kv_heads, num_selected), one cluster per sequence, CTA
// rank = kv head. The g x W window queries of the group are the rows of a
// dense [g*W x 128] x [128 x keys] product, so scoring runs on tensor cores:
//   A. per row group (up to 8 m-tiles of 16 rows, sized to shared memory):
//      K tiles of 64 keys (positions [0, S-W), gathered through the block
//      table with cp.async, double-buffered) meet the rows' A fragments in
//      mma.sync m16n8k16; every score is rounded like the reference
//      (bf16(q.k), bf16(* scale), sink key 0 -> -inf) and kept as bf16 in
//      shared memory;
//   B. per row: max and sum of exp over the keys (fp32);
//   C. per key: for each head, the bf16 softmax probabilities of its W rows
//      are added in window order into an fp32 accumulator (deterministic).
//   Then the window sum is rounded to bf16 per head, summed over the group in
//   fp32, and the cluster sum of those partials is rounded to bf16 -- the two
//   bf16 roundings of the reference's sum(dim=2).sum(dim=1). Top-k, ordering
//   and in-place compaction follow the window kernel; kept rows go to
//   positions [0, R) of the block table and context_lens[b] = R.
// Keys are positions [0, S-W) (TritonGetKVForComp gathers the first S
// positions); the compaction window starts at max(len - S, 0). The two
// coincide whenever compression triggers (len == S).
#pragma once
#include "compress_common.cuh"

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
  uint16_t* out_importance;  // bf16 bits [num_selected][num_keys], or null
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
  int num_keys;   // S - W
  int keys_pad;   // num_keys rounded up to kThrKeyTile
  int rows;       // g * W
  int mtiles;     // ceil(rows / 16)
  int group_mtiles;  // m-tiles per row group (<= kThrWarps / 2)
  int halves;     // CTAs per kv head (1 or 2), each taking one range of the keys
  int keys_half;  // keys per CTA, a multiple of kThrKeyTile (keys_pad when halves = 1)
};

// 16 warps: two per 16-row m-tile in the scoring, and enough threads that
// the per-key window sums (one thread per key and head) and the row
// statistics hide their exp / divide latency.
constexpr int kThrThreads = 512;
constexpr int kThrWarps = kThrThreads / 32;
constexpr int kThrReduceSlots = 16 * kThrWarps;
constexpr int kThrKeyTile = 64;
constexpr int kThrKRowElems = kCompressHeadDim + 8;  // padded smem row: conflict-free ldmatrix

constexpr int kThrKStages = 3;  // key-tile ring: two tiles of look-ahead

__host__ __device__ constexpr int thr_score_stride(int keys_pad) { return keys_pad + 8; }

// Bytes of the score region: the rows of the largest row group (bf16), later
// reused for the compaction's source and destination slot tables (2R ints).
__host__ __device__ constexpr size_t thr_score_bytes(int group_mtiles, int rows, int keys_pad,
                                                     int R) {
  const size_t sc_rows = static_cast<size_t>(group_mtiles * 16 < rows ? group_mtiles * 16 : rows);
  const size_t sc = sizeof(__nv_bfloat16) * sc_rows * thr_score_stride(keys_pad);
  const size_t slots = sizeof(int) * 2 * static_cast<size_t>(R);
  return ((sc > slots ? sc : slots) + 15) / 16 * 16;
}

// Shared-memory bytes of threshold_compress_kernel (host and device agree).
// keys_half: the keys one CTA scores (its score rows, window sums, partial
// and slots); keys_pad: all keys (the gathered importance for the top-k).
__host__ __device__ constexpr size_t threshold_smem_bytes(int G, int keys_pad, int keys_half,
                                                          int group_mtiles, int rows, int R) {
  return sizeof(__nv_bfloat16) * kThrKStages * kThrKeyTile * kThrKRowElems       // K tiles
         + thr_score_bytes(group_mtiles, rows, keys_half, R)                     // scores
         + sizeof(float) * 2 * group_mtiles * 16                                 // row max, sum
         + sizeof(float) * 4 * group_mtiles * 16                                 // exchange (2 x max, sum)
         + sizeof(float) * static_cast<size_t>(G) * keys_half                    // window sums
         + sizeof(float) * keys_half                                             // partial
         + sizeof(uint16_t) * (keys_pad + 2)                                     // keys
         + sizeof(int) * R                                                       // final index
         + sizeof(float) * kThrReduceSlots                                       // reductions
         + sizeof(int) * 256                                                     // top-k histogram
         + sizeof(int) * keys_half;                                              // key slots
}

template <int G>
__global__ void __launch_bounds__(kThrThreads, 1)
threshold_compress_kernel(const ThresholdCompressParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  cg::cluster_group cluster = cg::this_cluster();
  // cluster rank = kv head * halves + half; half h scores keys
  // [h * keys_half, (h + 1) * keys_half)
  const int H = p.halves;
  const int rank = static_cast<int>(cluster.block_rank());
  const int head = rank / H;
  const int half = rank - head * H;
  const int sel_i = blockIdx.y;
  const int g = p.g;
  const int nk = p.num_keys;
  const int kp = p.keys_pad;
  const int kh = p.keys_half;
  const int k0 = half * kh;                  // this CTA's first key
  const int nkl = max(0, min(nk - k0, kh));  // its real keys
  const int bs = p.block_size;
  const int W = p.window;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int ss = thr_score_stride(kh);
  const int gm16 = p.group_mtiles * 16;

  __nv_bfloat16* ktile = reinterpret_cast<__nv_bfloat16*>(smem);           // [3][64][136]
  __nv_bfloat16* sc = ktile + kThrKStages * kThrKeyTile * kThrKRowElems;   // [group rows][ss]
  float* rmax = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(sc) +
                                         thr_score_bytes(p.group_mtiles, p.rows, kh, p.R));
  float* rsum = rmax + gm16;
  float* xchg = rsum + gm16;                                                // [2][max, sum][gm16] (cluster-visible)
  float* kacc = xchg + 4 * gm16;                                            // [G][kh]
  float* partial = kacc + G * kh;                                           // [kh] (cluster-visible)
  uint16_t* keys = reinterpret_cast<uint16_t*>(partial + kh);               // [kp] (cluster-visible)
  int* final_idx = reinterpret_cast<int*>(keys + kp + 2);                   // [R]
  float* red = reinterpret_cast<float*>(final_idx + p.R);                   // [kThrReduceSlots]
  int* hist = reinterpret_cast<int*>(red + kThrReduceSlots);                // [256]
  int* kslot = hist + 256;                                                  // [kh] cache slot of key k0 + t
  __shared__ int s_valid;
  __shared__ int s_start;

  // The kv heads (and key halves) of a sequence are the CTAs of one cluster
  // (row statistics, partial sums and importance meet in distributed shared
  // memory). A launch that lost its clusters (%cluster_nctarank 1) cannot
  // form them: flag it and write nothing (the condition is uniform, so no
  // CTA waits at a cluster barrier).
  if (static_cast<int>(cluster.num_blocks()) != p.num_kv_heads * H) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) raise_error(NKV_DEVERR_LAUNCH_SHAPE);
    return;
  }
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
    if (!valid && rank == 0) raise_error(NKV_DEVERR_COMPRESS_RANGE);
    s_valid = valid;
  }
  for (int i = threadIdx.x; i < G * kh; i += kThrThreads) kacc[i] = 0.f;
  // every key's cache slot, resolved once (-1: unresolved or padding)
  for (int t = threadIdx.x; t < kh; t += kThrThreads)
    kslot[t] = t < nkl ? static_cast<int>(slot_of(k0 + t)) : -1;
  __syncthreads();
  const bool valid = s_valid != 0;  // identical in every CTA of the cluster
  const int start = s_start;

  if (valid) {
    const int rslot = __ldg(p.ring_slot_of_selected + sel_i);
    const __nv_bfloat16* qbase =
        p.ring + (static_cast<int64_t>(rslot) * p.num_layers + p.layer_id) *
                     static_cast<int64_t>(W) * p.num_q_heads * kCompressHeadDim;
    const int ntiles = kh / kThrKeyTile;
    // query row rho = r * W + w of this group -> its 128 bf16 values (or null)
    auto qrow = [&](int rho) -> const __nv_bfloat16* {
      if (rho >= p.rows) return nullptr;
      const int r = rho / W, w = rho - r * W;
      return qbase + (static_cast<int64_t>(w) * p.num_q_heads + head * g + r) * kCompressHeadDim;
    };
    auto load_ktile = [&](int tile, int buf) {
      const uint32_t base = smem_u32(ktile + buf * kThrKeyTile * kThrKRowElems);
      for (int i = threadIdx.x; i < kThrKeyTile * 16; i += kThrThreads) {
        const int kr = i >> 4, c = i & 15;
        const int t = tile * kThrKeyTile + kr;
        const uint32_t dst = base + (kr * kThrKRowElems + c * 8) * 2;
        const int64_t slot = kslot[t];
        if (slot >= 0) {
          cp_async_16(dst, p.k_cache + (slot * p.num_kv_heads + head) * kCompressHeadDim + c * 8);
        } else {
          *reinterpret_cast<uint4*>(ktile + buf * kThrKeyTile * kThrKRowElems +
                                    kr * kThrKRowElems + c * 8) = make_uint4(0, 0, 0, 0);
        }
      }
      cp_async_commit();
    };

    int group_parity = 0;
    for (int group0 = 0; group0 < p.mtiles; group0 += p.group_mtiles) {
      const int gm = min(p.group_mtiles, p.mtiles - group0);
      const int row0 = group0 * 16;
      // ---- A: scores of this row group over this CTA's keys; warps 2m and
      // 2m + 1 take m-tile m, each half of every key tile's eight columns
      uint32_t qa[8][4];
      const int mt = warp >> 1;
      const int nt0 = (warp & 1) * (kThrKeyTile / 16);
      const bool mma_warp = mt < gm;
      if (mma_warp) {
        const __nv_bfloat16* q_lo = qrow(row0 + mt * 16 + gid);
        const __nv_bfloat16* q_hi = qrow(row0 + mt * 16 + gid + 8);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const int d = kk * 16 + 2 * tig;
          qa[kk][0] = q_lo ? *reinterpret_cast<const uint32_t*>(q_lo + d) : 0u;
          qa[kk][1] = q_hi ? *reinterpret_cast<const uint32_t*>(q_hi + d) : 0u;
          qa[kk][2] = q_lo ? *reinterpret_cast<const uint32_t*>(q_lo + d + 8) : 0u;
          qa[kk][3] = q_hi ? *reinterpret_cast<const uint32_t*>(q_hi + d + 8) : 0u;
        }
      }
      // key-tile ring: tiles t+1 and t+2 stream while tile t is scored;
      // every step commits one cp.async group (empty past the last tile)
#pragma unroll
      for (int t = 0; t < kThrKStages - 1; ++t) {
        if (t < ntiles) {
          load_ktile(t, t);
        } else {
          cp_async_commit();
        }
      }
      const int grows = min(gm * 16, p.rows - row0);
      for (int tile = 0; tile < ntiles; ++tile) {
        const int buf = tile % kThrKStages;
        cp_async_wait<kThrKStages - 2>();  // this thread's copies of `tile` landed
        // all threads' copies of `tile` landed, and tile - 1 is scored: its
        // buffer takes tile + 2
        __syncthreads();
        if (tile + kThrKStages - 1 < ntiles) {
          load_ktile(tile + kThrKStages - 1, (tile + kThrKStages - 1) % kThrKStages);
        } else {
          cp_async_commit();
        }
        if (mma_warp) {
          const uint32_t kb = smem_u32(ktile + buf * kThrKeyTile * kThrKRowElems);
          const int lrow = mt * 16 + gid;
#pragma unroll
          for (int nt = nt0; nt < nt0 + kThrKeyTile / 16; ++nt) {
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int kq = 0; kq < 4; ++kq) {
              const uint32_t addr =
                  kb + ((nt * 8 + (lane & 7)) * kThrKRowElems + (kq * 4 + (lane >> 3)) * 8) * 2;
              uint32_t b0, b1, b2, b3;
              ldsm_x4(addr, b0, b1, b2, b3);
              mma_bf16_16816(acc, qa[2 * kq][0], qa[2 * kq][1], qa[2 * kq][2], qa[2 * kq][3], b0, b1);
              mma_bf16_16816(acc, qa[2 * kq + 1][0], qa[2 * kq + 1][1], qa[2 * kq + 1][2],
                             qa[2 * kq + 1][3], b2, b3);
            }
            const int t0 = tile * kThrKeyTile + nt * 8 + 2 * tig;  // local key
            float v[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int t = k0 + t0 + (e & 1);  // global key
              v[e] = (t == 0 || t >= nk) ? -INFINITY : round_bf16(round_bf16(acc[e]) * p.scale);
            }
            // rows past the group's real rows (m-tile padding) have no storage
            if (lrow < grows)
              *reinterpret_cast<uint32_t*>(sc + static_cast<size_t>(lrow) * ss + t0) =
                  pack_bf16x2(v[0], v[1]);
            if (lrow + 8 < grows)
              *reinterpret_cast<uint32_t*>(sc + static_cast<size_t>(lrow + 8) * ss + t0) =
                  pack_bf16x2(v[2], v[3]);
          }
        }
      }
      __syncthreads();  // scores complete; the ring's buffers are free
      // ---- B: per-row max and sum of exp over all keys. With two halves
      // each CTA reduces its own keys and the pair exchanges through
      // distributed shared memory (buffers by group parity: rewritten two
      // groups later, after the partner has passed this group's barriers):
      // the max, then the sum, the sum added in half order so both agree.
      float* xmax = xchg + group_parity * 2 * gm16;
      float* xsum = xmax + gm16;
      const float* pmax = H > 1 ? cluster.map_shared_rank(xmax, rank ^ 1) : nullptr;
      const float* psum = H > 1 ? cluster.map_shared_rank(xsum, rank ^ 1) : nullptr;
      for (int lr = warp; lr < grows; lr += kThrWarps) {
        const __nv_bfloat16* row = sc + static_cast<size_t>(lr) * ss;
        float m = -INFINITY;
        for (int t = lane; t < nkl; t += 32) m = fmaxf(m, __bfloat162float(row[t]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) xmax[lr] = m;
      }
      if (H > 1) cluster.sync();
      else __syncthreads();
      for (int lr = warp; lr < grows; lr += kThrWarps) {
        const __nv_bfloat16* row = sc + static_cast<size_t>(lr) * ss;
        const float m = H > 1 ? fmaxf(xmax[lr], pmax[lr]) : xmax[lr];
        float z = 0.f;
        for (int t = lane; t < nkl; t += 32) z += expf(__bfloat162float(row[t]) - m);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
        if (lane == 0) {
          rmax[lr] = m;
          xsum[lr] = z;
        }
      }
      if (H > 1) cluster.sync();
      else __syncthreads();
      for (int lr = threadIdx.x; lr < grows; lr += kThrThreads)
        rsum[lr] = H > 1 ? (half == 0 ? xsum[lr] + psum[lr] : psum[lr] + xsum[lr]) : xsum[lr];
      __syncthreads();
      group_parity ^= 1;
      // ---- C: per (key, head), window-ordered sum of the head's bf16
      // probabilities. A head's rows in this group are summed in a register,
      // continuing the head's running sum from earlier groups (the same fp32
      // additions in the same order as one sequential sum); the exponentials
      // and divisions of successive rows do not depend on each other and
      // overlap.
      const int r_first = row0 / W;
      const int ntask = ((row0 + grows - 1) / W - r_first + 1) * nkl;
      for (int task = threadIdx.x; task < ntask; task += kThrThreads) {
        const int r = r_first + task / nkl;
        const int t = task - (r - r_first) * nkl;
        const int lr_end = min(grows, (r + 1) * W - row0);
        float acc = kacc[r * kh + t];
#pragma unroll 4
        for (int lr = max(r * W - row0, 0); lr < lr_end; ++lr) {
          const float e = expf(__bfloat162float(sc[static_cast<size_t>(lr) * ss + t]) - rmax[lr]);
          acc += round_bf16(e / rsum[lr]);
        }
        kacc[r * kh + t] = acc;
      }
      __syncthreads();
    }
    for (int t = threadIdx.x; t < kh; t += kThrThreads) {
      float s = 0.f;
      if (t < nkl) {
#pragma unroll
        for (int r = 0; r < G; ++r)
          if (r < g) s += round_bf16(kacc[r * kh + t]);
      }
      partial[t] = s;
    }
  }
  cluster.sync();
  if (valid) {
    // this CTA's keys: the sum over the heads (CTAs of the same half, in head
    // order), rounded to bf16 -- the reference's sum(dim=1)
    for (int t = threadIdx.x; t < nkl; t += kThrThreads) {
      float s = 0.f;
      for (int hd = 0; hd < p.num_kv_heads; ++hd)
        s += cluster.map_shared_rank(partial, hd * H + half)[t];
      keys[k0 + t] = static_cast<uint16_t>(bf16_key(s));
      if (head == 0 && p.out_importance != nullptr)
        p.out_importance[static_cast<int64_t>(sel_i) * nk + k0 + t] = keys[k0 + t];
    }
  }
  cluster.sync();  // no CTA may leave while a peer still reads its partials
  if (H > 1) {
    // the other half's keys, from the partner CTA of the same head
    if (valid) {
      const int pk0 = (half ^ 1) * kh;
      const int pn = max(0, min(nk - pk0, kh));
      const uint16_t* pkeys = cluster.map_shared_rank(keys, rank ^ 1);
      for (int t = threadIdx.x; t < pn; t += kThrThreads) keys[pk0 + t] = pkeys[pk0 + t];
    }
    cluster.sync();  // ... nor while its partner still reads its keys
  }
  if (!valid) return;

  const int num_keep = p.R - W - 1;
  if (threadIdx.x == 0) final_idx[0] = 0;
  topk_ascending<kThrThreads>(keys, nk, num_keep, final_idx + 1, reinterpret_cast<int*>(red), hist);
  for (int i = threadIdx.x; i < W; i += kThrThreads) final_idx[1 + num_keep + i] = p.S - W + i;
  __syncthreads();

  // every row's source and destination slot, resolved in one round into the
  // (now unused) score region, so the compaction's chunks wait on no
  // block-table lookup
  int* src_slot = reinterpret_cast<int*>(sc);
  int* dst_slot = src_slot + p.R;
  for (int i = threadIdx.x; i < p.R; i += kThrThreads) {
    src_slot[i] = static_cast<int>(slot_of(start + final_idx[i]));
    dst_slot[i] = static_cast<int>(slot_of(i));
  }
  __syncthreads();
  // with two CTAs per head, one moves the K rows and the other the V rows
  compact_rows_pipelined<kThrThreads>(p.k_cache, p.v_cache, p.num_kv_heads, head, p.R,
                                      [&](int i, int64_t& src, int64_t& dst) {
                                        src = src_slot[i];
                                        dst = dst_slot[i];
                                      },
                                      H > 1 ? 1 + half : 3);
  if (rank == 0) {
    if (threadIdx.x == 0) p.context_lens[b] = p.R;
    if (p.out_keep_idx) {
      for (int i = threadIdx.x; i < p.R; i += kThrThreads)
        p.out_keep_idx[static_cast<int64_t>(sel_i) * p.R + i] = final_idx[i];
    }
  }
}

}  // namespace nkv
