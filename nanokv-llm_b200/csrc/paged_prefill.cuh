// Prefill / mixed-batch attention over the paged KV cache for sm_100a: the
// B200 replacement for flash_attn_varlen_func(q, k, v, cu_seqlens_q,
// cu_seqlens_k, max_seqlen_q, max_seqlen_k, softmax_scale, causal=True,
// block_table=...) at nanokvllm/layers/attention.py:96-102.
//
// Semantics (flash-attn >= 2.1): sequence b has Lq = cu_q[b+1]-cu_q[b] query
// rows and Lk = cu_k[b+1]-cu_k[b] keys; with `causal`, query i attends keys
// j <= Lk - Lq + i (the mask is aligned to the bottom-right corner, so a
// chunked-prefill chunk sees the whole cached prefix). Keys live in the paged
// cache (block_tables) or, without a block table, in rows cu_k[b] + j of
// contiguous K/V tensors.
//
// One CTA per (q-tile, kv head, sequence), q-tiles innermost so that the
// CTAs resident at once share one sequence's K/V stream in L2, longest-first
// (grid x reversed) to shorten the causal tail. A q-tile is the 128-row M side of
// the tensor-core tiles: QT = floor(128/g) query positions x the g query
// heads of the kv head's GQA group (row = i*g + r), so every K/V tile is
// read once for the whole group.
//
// Fifth-generation tensor cores (tcgen05), all accumulators in TMEM:
//   * warps 9 and 10, producers: TMA-load the q-tile and the 128-key K
//     tiles (warp 9) and the V tiles (warp 10), 128-byte swizzle, no
//     multicast, into a 4-deep K ring (its last stage is the q-tile buffer,
//     reused once Q has moved to TMEM) and a 2-deep V ring; the two rings
//     refill independently (K as soon as its S MMA is done, V after its PV
//     MMA). A tile is cut at cache-block boundaries when blocks hold < 128.
//   * warp 8, MMA issuer (one thread): S_j = Q K_j^T into one of two TMEM
//     S buffers (8 x UMMA 128x128x16, A and B from shared memory), then
//     O += P_{j-1} V_{j-1} (A = P from TMEM, B = V MN-major from shared
//     memory) once the softmax warps have written P_{j-1}: the tensor core
//     computes S_j while the softmax of tile j-1 runs.
//   * warps 0-7, softmax: row t = TMEM lane t belongs to warps t/32 and
//     t/32 + 4, which take key columns [0,64) and [64,128) of S (and dims
//     [0,64) / [64,128) of O). Per tile: S half-row from TMEM, causal /
//     length masks on diagonal and tail tiles, the two partial row maxima
//     exchanged through shared memory (an mbarrier of the 8 warps), online
//     softmax in the exp2 domain with a lazily moved maximum (O in TMEM is
//     rescaled only when the row maximum grows by more than 2^8, so
//     stale-maximum probabilities stay <= 256), P packed to bf16 into TMEM;
//     row sums stay per half until the epilogue O / l -> bf16 -> the query
//     rows that exist.
//   The q-tile is moved once from shared memory into TMEM (bf16 pairs, as
//   P), so the S MMAs take A from TMEM and shared memory only feeds K and V
//   to the tensor core (with A and B both in shared memory the S MMA would
//   be bound by shared-memory bandwidth).
// TMEM columns: S0 [0,128), S1 [128,256), O [256,384), P [384,448),
// Q [448,512).
#pragma once
#include "nkv_common.cuh"
#include "tcgen05.cuh"

namespace nkv {

constexpr int kPrefillRows = 128;      // M: rows (query x head) per CTA
constexpr int kPrefillKeyTile = 128;   // N of S / K of PV: keys per tile
constexpr int kPrefillKStages = 4;     // K ring depth; its last stage reuses the q-tile buffer
constexpr int kPrefillKSmemStages = kPrefillKStages - 1;
constexpr int kPrefillVStages = 2;
constexpr int kPrefillThreads = 352;   // 8 softmax warps, MMA warp, K and V producer warps
constexpr int kPrefillMmaWarp = 8;
constexpr int kPrefillProducerWarp = 9;  // Q and K; warp 10 loads V
constexpr int kPrefillHalf = kPrefillKeyTile * 128;   // 64 dims x 128 keys x 2 B
constexpr int kPrefillTileBytes = 2 * kPrefillHalf;   // one K or V tile, 32 KB
constexpr int kPrefillQHalf = kPrefillRows * 128;
constexpr int kPrefillNumBars = 23;
constexpr int kPrefillRedBytes = 2 * 2 * kPrefillRows * 4;  // [parity][half][row] floats
constexpr int kPrefillSmemBytes = 2 * kPrefillQHalf +
                                  (kPrefillKSmemStages + kPrefillVStages) * kPrefillTileBytes + 256 +
                                  kPrefillRedBytes + 1024 /* alignment */;
constexpr uint32_t kPrefillTmemCols = 512;
constexpr uint32_t kTmemS0 = 0, kTmemO = 256, kTmemP = 384, kTmemQ = 448;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct PrefillParams {
  const int32_t* block_tables;  // null: contiguous K/V rows cu_k[b] + j
  const int32_t* cu_q;
  const int32_t* cu_k;
  __nv_bfloat16* out;
  int64_t out_stride_token;
  int64_t num_blocks;
  int64_t num_q_tokens;  // rows of q / out
  int64_t num_kv_rows;   // rows of the K/V tensors (contiguous case)
  float scale_log2;
  int max_blocks;
  int batch;
  int num_kv_heads;
  int g;              // query heads per kv head
  int qt;             // query positions per CTA, floor(128 / g)
  int block_size;
  int rows_per_load;  // keys per TMA box: min(block_size, 128) paged, 128 contiguous
  int causal;
  int qtiles;         // q-tiles per sequence slot of the grid
};

// 3-D tiled TMA load with the default L2 policy (K/V tiles are re-read by
// every q-tile of the sequence, so they should stay in L2).
__device__ __forceinline__ void tma_load_3d_nohint(uint32_t dst, const CUtensorMap* map,
                                                   uint32_t bar, int32_t c0, int32_t c1,
                                                   int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// Publishes `v` for (row, half) and returns the other half's value, through
// shared-memory slots and an mbarrier of 8 warp arrivals (bounded wait).
__device__ __forceinline__ float exchange_half(float* red, uint64_t* red_bar, int step, int half,
                                               int row, int lane, float v) {
  float* slot = red + ((step & 1) * 2) * kPrefillRows;
  slot[half * kPrefillRows + row] = v;
  __syncwarp();
  const uint32_t bar = smem_u32(&red_bar[step & 1]);
  if (lane == 0) mbar_arrive(bar);
  mbar_wait_bounded(bar, (step >> 1) & 1);
  return slot[(half ^ 1) * kPrefillRows + row];
}

// ------------------------------------------------------------- paired fp32
// sm_100 executes two fp32 lanes per instruction on .b64 register pairs.
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// Shared-memory address of K stage s (the last one is the q-tile buffer).
__device__ __forceinline__ uint8_t* k_stage(uint8_t* k_mem, uint8_t* q_mem, int s) {
  return s < kPrefillKSmemStages ? k_mem + s * kPrefillTileBytes : q_mem;
}

__global__ void __launch_bounds__(kPrefillThreads, 1)
paged_prefill_kernel(const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v,
                     const __grid_constant__ CUtensorMap tm_q, const PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* q_mem = smem;  // Q lo, Q hi
  uint8_t* k_mem = smem + 2 * kPrefillQHalf;
  uint8_t* v_mem = k_mem + kPrefillKSmemStages * kPrefillTileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(v_mem + kPrefillVStages * kPrefillTileBytes);
  uint64_t* q_full = bars;                       // 1
  uint64_t* k_full = bars + 1;                   // 4
  uint64_t* k_empty = k_full + kPrefillKStages;  // 4
  uint64_t* v_full = k_empty + kPrefillKStages;  // 2
  uint64_t* v_empty = v_full + kPrefillVStages;  // 2
  uint64_t* s_full = v_empty + kPrefillVStages;  // 2
  uint64_t* s_free = s_full + 2;                 // 2
  uint64_t* p_full = s_free + 2;                 // 1
  uint64_t* pv_done = p_full + 1;                // 1
  uint64_t* mma_done = pv_done + 1;              // 1
  uint64_t* red_bar = mma_done + 1;              // 2: half-row exchange, by tile parity
  uint64_t* q_tmem = red_bar + 2;                // 1: q-tile copied into TMEM
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kPrefillNumBars);
  float* red = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 256);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = p.g;
  const int QT = p.qt;
  const int qtile = p.qtiles - 1 - static_cast<int>(blockIdx.x);
  const int kvh = blockIdx.y;
  const int b = blockIdx.z;
  const int q0 = __ldg(p.cu_q + b);
  const int Lq = __ldg(p.cu_q + b + 1) - q0;
  const int k0 = __ldg(p.cu_k + b);
  const int Lk = __ldg(p.cu_k + b + 1) - k0;
  // Metadata the grid and the tensors cannot hold: flag and skip the row.
  if (Lq < 0 || Lk < 0 || q0 < 0 || static_cast<int64_t>(q0) + Lq > p.num_q_tokens ||
      Lq > p.qtiles * QT ||
      (p.block_tables == nullptr ? (k0 < 0 || static_cast<int64_t>(k0) + Lk > p.num_kv_rows)
                                 : (static_cast<int64_t>(Lk) >
                                    static_cast<int64_t>(p.max_blocks) * p.block_size))) {
    if (threadIdx.x == 0 && blockIdx.x == 0) raise_error(NKV_DEVERR_PREFILL_RANGE);
    return;
  }
  const int qs = qtile * QT;  // first query position of this CTA
  if (qs >= Lq) return;       // uniform across the CTA
  const int qn = min(QT, Lq - qs);
  const int shift = Lk - Lq;  // causal: query i sees keys j <= shift + i
  int kend = Lk;
  if (p.causal) kend = max(0, min(Lk, shift + qs + qn));
  const int ntiles = (kend + kPrefillKeyTile - 1) / kPrefillKeyTile;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(q_full), 1);
    for (int s = 0; s < kPrefillKStages; ++s) {
      mbar_init(smem_u32(&k_full[s]), 1);
      mbar_init(smem_u32(&k_empty[s]), 1);
    }
    for (int s = 0; s < kPrefillVStages; ++s) {
      mbar_init(smem_u32(&v_full[s]), 1);
      mbar_init(smem_u32(&v_empty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&s_full[s]), 1);
      mbar_init(smem_u32(&s_free[s]), 8);
    }
    mbar_init(smem_u32(p_full), 8);
    mbar_init(smem_u32(pv_done), 1);
    mbar_init(smem_u32(mma_done), 1);
    mbar_init(smem_u32(&red_bar[0]), 8);
    mbar_init(smem_u32(&red_bar[1]), 8);
    mbar_init(smem_u32(q_tmem), 8);
    fence_barrier_init();
  }
  if (warp == kPrefillMmaWarp) {
    tmem_alloc(smem_u32(tmem_slot), kPrefillTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dependency_wait();

  if (warp >= kPrefillProducerWarp) {
    // ------------------------------------------------------------ producers
    const int kv = warp - kPrefillProducerWarp;  // 0: Q + K, 1: V
    if (lane == 0) {
      const CUtensorMap* map = kv ? &tm_v : &tm_k;
      prefetch_tmap(map);
      if (kv == 0) {
        prefetch_tmap(&tm_q);
        const uint32_t qb = smem_u32(q_mem);
        mbar_arrive_expect_tx(smem_u32(q_full), 2u * QT * G * 128);
        const uint64_t pol_q = l2_policy_evict_first();
        tma_load_3d(qb, &tm_q, smem_u32(q_full), 0, kvh * G, q0 + qs, pol_q);
        tma_load_3d(qb + kPrefillQHalf, &tm_q, smem_u32(q_full), 64, kvh * G, q0 + qs, pol_q);
      }
      const int sub = p.rows_per_load;
      const int stages = kv ? kPrefillVStages : kPrefillKStages;
      uint64_t* emp = kv ? v_empty : k_empty;
      uint64_t* ful = kv ? v_full : k_full;
      // bit s set while stage s has a fill in flight, with that fill's
      // full-barrier parity
      uint32_t armed = 0u, parity = 0u;
      for (int t = 0; t < ntiles; ++t) {
        const int s = t % stages;
        const uint32_t ph = (t / stages) & 1;
        if (!mbar_wait_bounded(smem_u32(&emp[s]), ph ^ 1u)) break;
        // the last K stage is the q-tile buffer: free once Q is in TMEM
        if (kv == 0 && t == kPrefillKSmemStages && !mbar_wait_bounded(smem_u32(q_tmem), 0)) break;
        armed &= ~(1u << s);  // the stage's previous fill was consumed
        const uint32_t fb = smem_u32(&ful[s]);
        mbar_arrive_expect_tx(fb, kPrefillTileBytes);
        armed |= 1u << s;
        parity = (parity & ~(1u << s)) | (ph << s);
        const uint32_t base =
            smem_u32(kv ? v_mem + s * kPrefillTileBytes : k_stage(k_mem, q_mem, s));
        for (int part = 0; part < kPrefillKeyTile; part += sub) {
          const int tok = t * kPrefillKeyTile + part;
          int row;
          if (p.block_tables != nullptr) {
            if (tok >= Lk) {
              row = -2 * sub;  // wholly past the sequence: zero fill
            } else {
              const int blk = __ldg(p.block_tables + static_cast<int64_t>(b) * p.max_blocks +
                                    tok / p.block_size);
              if (blk < 0 || static_cast<int64_t>(blk) >= p.num_blocks) {
                raise_error(NKV_DEVERR_DECODE_BLOCK);
                row = -2 * sub;
              } else {
                row = blk * p.block_size + (tok % p.block_size);
              }
            }
          } else {
            row = k0 + tok;
          }
          tma_load_3d_nohint(base + part * 128, map, fb, 0, kvh, row);
          tma_load_3d_nohint(base + kPrefillHalf + part * 128, map, fb, 64, kvh, row);
        }
      }
      // Fills still in flight (only after an abort) complete before exit.
      for (int s = 0; s < stages; ++s)
        if (armed & (1u << s)) mbar_wait_bounded(smem_u32(&ful[s]), (parity >> s) & 1u);
      if (kv == 0) mbar_wait_bounded(smem_u32(q_full), 0);
    }
  } else if (warp == kPrefillMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc_s = umma_idesc_bf16(128, kPrefillKeyTile, 0);
    constexpr uint32_t idesc_o = umma_idesc_bf16(128, 128, 1);
    bool ok = mbar_wait_bounded(smem_u32(q_tmem), 0);
    for (int j = 0; j <= ntiles && ok; ++j) {
      if (j < ntiles) {
        const int ks = j % kPrefillKStages;
        if (!mbar_wait_bounded(smem_u32(&k_full[ks]), (j / kPrefillKStages) & 1) ||
            !mbar_wait_bounded(smem_u32(&s_free[j & 1]), ((j >> 1) & 1) ^ 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t kb = smem_u32(k_stage(k_mem, q_mem, ks));
          const uint32_t d = tmem + kTmemS0 + (j & 1) * kPrefillKeyTile;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            // A = Q from TMEM (16 dims = 8 columns per step); B = K, K-major:
            // 16 dims per step, 32 bytes into the 128-byte swizzled rows of
            // the half holding them, 8-row groups 1024 B apart (SBO).
            const uint32_t koff = (kk >> 2) * kPrefillHalf + (kk & 3) * 32;
            umma_ts(d, tmem + kTmemQ + kk * 8, umma_desc_sw128(kb + koff, 16, 1024), idesc_s,
                    kk > 0 ? 1u : 0u);
          }
          umma_commit(smem_u32(&s_full[j & 1]));
          umma_commit(smem_u32(&k_empty[ks]));
        }
        __syncwarp();
      }
      if (j >= 1) {
        const int t = j - 1;
        const int vs = t % kPrefillVStages;
        if (!mbar_wait_bounded(smem_u32(p_full), t & 1) ||
            !mbar_wait_bounded(smem_u32(&v_full[vs]), (t / kPrefillVStages) & 1)) {
          ok = false;
          break;
        }
        uint8_t* vt = v_mem + vs * kPrefillTileBytes;
        const int valid = Lk - t * kPrefillKeyTile;
        if (valid < kPrefillKeyTile) {
          // V rows past the sequence may hold any bits (NaN included); their
          // P is 0, so zero them rather than let 0 * NaN reach O.
          const int nz = (kPrefillKeyTile - valid) * 8;  // 16-byte chunks per half
          for (int c = lane; c < 2 * nz; c += 32) {
            const int half = c / nz;
            const int idx = c - half * nz;
            *reinterpret_cast<uint4*>(vt + half * kPrefillHalf + valid * 128 + idx * 16) =
                make_uint4(0u, 0u, 0u, 0u);
          }
          fence_proxy_async_shared();
          __syncwarp();
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t vb = smem_u32(vt);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            // B = V (K = keys, N = dims, MN-major): 16 keys per step, the
            // dims 64..127 atom one half-tile further (LBO), 8-key groups
            // 1024 B apart (SBO).
            umma_ts(tmem + kTmemO, tmem + kTmemP + kk * 8,
                    umma_desc_sw128(vb + kk * 2048, kPrefillHalf, 1024), idesc_o,
                    (t > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(smem_u32(&v_empty[vs]));
          umma_commit(smem_u32(pv_done));
        }
        __syncwarp();
      }
    }
    // Every MMA this thread issued completes before the TMEM is released.
    if (lane == 0) umma_commit(smem_u32(mma_done));
    __syncwarp();
    mbar_wait_bounded(smem_u32(mma_done), 0);
  } else {
    // ------------------------------------------------------------ softmax
    const int quarter = warp & 3;
    const int half = warp >> 2;                      // key / dim columns [64*half, +64)
    const int row = quarter * 32 + lane;             // TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int qi = row / G;
    const int r = row - qi * G;
    const int lim = shift + qs + qi;
    const float scale_log2 = p.scale_log2;
    float m_used = -INFINITY;
    float l_half = 0.f;  // row sum over this half's columns
    // q-tile -> TMEM: this thread's row, dims [64*half, +64) from the
    // swizzled shared-memory half, as 32 columns of bf16 pairs
    bool ok = mbar_wait_bounded(smem_u32(q_full), 0);
    {
      uint32_t qv[32];
      const uint8_t* qh = q_mem + half * kPrefillQHalf;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 v = *reinterpret_cast<const uint4*>(qh + swz128(row, c));
        qv[4 * c] = v.x;
        qv[4 * c + 1] = v.y;
        qv[4 * c + 2] = v.z;
        qv[4 * c + 3] = v.w;
      }
      tmem_st32(tmem + lane_base + kTmemQ + half * 32, qv);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(q_tmem));
    }
    for (int j = 0; j < ntiles && ok; ++j) {
      if (!mbar_wait_bounded(smem_u32(&s_full[j & 1]), (j >> 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[2][32];
      const uint32_t sbase = tmem + lane_base + kTmemS0 + (j & 1) * kPrefillKeyTile + half * 64;
      tmem_ld32(sbase, sv[0]);
      tmem_ld32(sbase + 32, sv[1]);
      tmem_ld_wait(sv[0]);
      tmem_ld_wait(sv[1]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&s_free[j & 1]));

      const int tok0 = j * kPrefillKeyTile + half * 64;
      const bool masked = (j * kPrefillKeyTile + kPrefillKeyTile > Lk) ||
                          (p.causal && j * kPrefillKeyTile + kPrefillKeyTile - 1 > shift + qs);
      // Row maximum of the raw scores (the scale is positive): only diagonal
      // and tail tiles take the masking path.
      float mx8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) mx8[e] = -INFINITY;
      if (masked) {
        const int kmax = p.causal ? min(Lk - 1, lim) : Lk - 1;  // last admissible key
#pragma unroll
        for (int c = 0; c < 2; ++c) {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            if (tok0 + 32 * c + e > kmax) sv[c][e] = __float_as_uint(-INFINITY);
            mx8[e & 7] = fmaxf(mx8[e & 7], __uint_as_float(sv[c][e]));
          }
        }
      } else {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
#pragma unroll
          for (int e = 0; e < 32; ++e) mx8[e & 7] = fmaxf(mx8[e & 7], __uint_as_float(sv[c][e]));
        }
      }
      float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                       fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      // exchange the half-row maxima (slots and barriers by tile parity; a
      // slot is rewritten two tiles later, after its reader has arrived on
      // the next tile's barrier)
      mx = fmaxf(mx, exchange_half(red, red_bar, j, half, row, lane, mx));
      const float m_new = fmaxf(m_used, mx * scale_log2);  // log2 units
      float alpha = 1.f;
      bool rescale = false;
      if (m_used == -INFINITY) {
        m_used = m_new;  // nothing accumulated yet (O and l are zero)
      } else if (m_new > m_used + kRescaleThreshold) {
        alpha = fast_exp2(m_used - m_new);
        m_used = m_new;
        rescale = true;
      }
      const float neg_m = (m_used == -INFINITY) ? 0.f : -m_used;
      const uint64_t sc2 = f2_pack(scale_log2, scale_log2);
      const uint64_t nm2 = f2_pack(neg_m, neg_m);
      uint32_t pk[32];
      uint64_t rs2[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) rs2[e] = 0ull;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          float x0, x1;
          f2_unpack(f2_fma(f2_pack(__uint_as_float(sv[c][2 * e]), __uint_as_float(sv[c][2 * e + 1])),
                           sc2, nm2), x0, x1);
          const float p0 = fast_exp2(x0);
          const float p1 = fast_exp2(x1);
          rs2[e & 3] = f2_add(rs2[e & 3], f2_pack(p0, p1));
          pk[c * 16 + e] = pack_bf16x2(p0, p1);
        }
      }
      float r0, r1, r2, r3, r4, r5, r6, r7;
      f2_unpack(rs2[0], r0, r1);
      f2_unpack(rs2[1], r2, r3);
      f2_unpack(rs2[2], r4, r5);
      f2_unpack(rs2[3], r6, r7);
      const float rsum = ((r0 + r1) + (r2 + r3)) + ((r4 + r5) + (r6 + r7));
      l_half = l_half * alpha + rsum;
      // P buffer free and O current once the previous PV has completed.
      if (j > 0 && !mbar_wait_bounded(smem_u32(pv_done), (j - 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t ov[32];
          const uint32_t oa = tmem + lane_base + kTmemO + half * 64 + 32 * c;
          tmem_ld32(oa, ov);
          tmem_ld_wait(ov);
#pragma unroll
          for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
          tmem_st32(oa, ov);
        }
      }
      tmem_st32(tmem + lane_base + kTmemP + half * 32, pk);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(p_full));
    }
    // ---------------------------------------------------------- epilogue
    // whole-row sum from the two halves (slot parity of tile ntiles is free:
    // its last readers passed the barrier of tile ntiles - 1)
    const float l_run = l_half + exchange_half(red, red_bar, ntiles, half, row, lane, l_half);
    const bool row_out = qi < qn;
    __nv_bfloat16* dst = p.out + static_cast<int64_t>(q0 + qs + qi) * p.out_stride_token +
                         static_cast<int64_t>(kvh * G + r) * 128 + half * 64;
    if (ntiles == 0) {
      if (row_out)
        for (int c = 0; c < 8; ++c) reinterpret_cast<uint4*>(dst)[c] = make_uint4(0u, 0u, 0u, 0u);
    } else if (ok && mbar_wait_bounded(smem_u32(pv_done), (ntiles - 1) & 1)) {
      tc_fence_after();
      const float inv = (l_run > 0.f) ? 1.f / l_run : 0.f;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t ov[32];
        tmem_ld32(tmem + lane_base + kTmemO + half * 64 + 32 * c, ov);
        tmem_ld_wait(ov);
        uint32_t pkd[16];
#pragma unroll
        for (int e = 0; e < 16; ++e)
          pkd[e] = pack_bf16x2(__uint_as_float(ov[2 * e]) * inv, __uint_as_float(ov[2 * e + 1]) * inv);
        if (row_out) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + 32 * c);
#pragma unroll
          for (int e = 0; e < 4; ++e)
            d4[e] = make_uint4(pkd[4 * e], pkd[4 * e + 1], pkd[4 * e + 2], pkd[4 * e + 3]);
        }
      }
    }
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == kPrefillMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kPrefillTmemCols);
  }
}

}  // namespace nkv
