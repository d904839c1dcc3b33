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
// One CTA per (kv head, sequence, q-tile). A q-tile is up to 128 rows:
// QT = floor(128/g) query positions x the g query heads of the kv head's GQA
// group (row = i*g + r), so every K/V tile is read once for the whole group.
// q-tiles run longest-first (grid z reversed) to shorten the causal tail.
//   * warp 8, the producer: TMA-loads the q-tile (one transaction) and then
//     streams 64-key K and V tiles (128B swizzle, no multicast) through a
//     4-stage full/empty mbarrier ring; a tile never crosses a cache block.
//   * warps 0-7, the consumers: 16 rows each; S = Q K^T and O += P V with
//     mma.sync m16n8k16 (bf16 in, fp32 accumulate), online softmax in the
//     exp2 domain, causal and length masks by select on the diagonal tiles;
//     P is re-packed from the S accumulators as the A operand.
//   * epilogue: O / l in bf16 to the query rows that exist (Lq may end inside
//     the tile). Rows with no admissible key (Lk = 0) get zeros.
#pragma once
#include "nkv_common.cuh"

namespace nkv {

constexpr int kPrefillRows = 128;          // rows (query x head) per CTA
constexpr int kPrefillKeyTile = 64;        // keys per pipeline stage
constexpr int kPrefillConsumerWarps = 8;
constexpr int kPrefillThreads = (kPrefillConsumerWarps + 1) * 32;
constexpr int kPrefillStages = 4;
constexpr int kPrefillHalfKV = kPrefillKeyTile * 128;     // 64 rows x 64 dims x 2 B
constexpr int kPrefillStageBytes = 4 * kPrefillHalfKV;    // K lo/hi, V lo/hi
constexpr int kPrefillQHalf = kPrefillRows * 128;         // 128 rows x 64 dims x 2 B
constexpr int kPrefillSmemBytes =
    2 * kPrefillQHalf + kPrefillStages * kPrefillStageBytes + (2 * kPrefillStages + 1) * 8 + 64 +
    1024 /* alignment */;

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
  int g;            // query heads per kv head
  int qt;           // query positions per CTA, floor(128 / g)
  int block_size;
  int causal;
  int qtiles;   // q-tiles per sequence slot of the grid
};

__global__ void __launch_bounds__(kPrefillThreads, 1)
paged_prefill_kernel(const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v,
                     const __grid_constant__ CUtensorMap tm_q, const PrefillParams p) {
  const int G = p.g;
  const int QT = p.qt;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* q_mem = smem;                                  // Q lo, Q hi
  uint8_t* stage_mem = smem + 2 * kPrefillQHalf;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(stage_mem + kPrefillStages * kPrefillStageBytes);
  uint64_t* empty_bar = full_bar + kPrefillStages;
  uint64_t* q_bar = empty_bar + kPrefillStages;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Longest q-tiles (most keys under the causal mask) first.
  const int qtile = p.qtiles - 1 - static_cast<int>(blockIdx.z);
  const int kvh = blockIdx.x;
  const int b = blockIdx.y;
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
    if (threadIdx.x == 0 && blockIdx.z == 0) raise_error(NKV_DEVERR_PREFILL_RANGE);
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
    for (int s = 0; s < kPrefillStages; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), kPrefillConsumerWarps);
    }
    mbar_init(smem_u32(q_bar), 1);
    fence_barrier_init();
  }
  __syncthreads();
  grid_dependency_wait();

  if (warp == kPrefillConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane != 0) return;
    const uint64_t pol_stream = l2_policy_evict_first();
    const uint64_t pol_q = l2_policy_evict_first();
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
    prefetch_tmap(&tm_q);
    {
      const uint32_t qb = smem_u32(q_mem);
      mbar_arrive_expect_tx(smem_u32(q_bar), 2u * QT * G * 128);
      tma_load_3d(qb, &tm_q, smem_u32(q_bar), 0, kvh * G, q0 + qs, pol_q);
      tma_load_3d(qb + kPrefillQHalf, &tm_q, smem_u32(q_bar), 64, kvh * G, q0 + qs, pol_q);
    }
    int stage = 0;
    uint32_t phase = 0;
    uint32_t armed[kPrefillStages];
#pragma unroll
    for (int s = 0; s < kPrefillStages; ++s) armed[s] = 0;
    for (int t = 0; t < ntiles; ++t) {
      if (!mbar_wait_bounded(smem_u32(&empty_bar[stage]), phase ^ 1u)) break;
      armed[stage] = 0;
      const int tok = t * kPrefillKeyTile;
      int row;
      if (p.block_tables != nullptr) {
        const int blk = __ldg(p.block_tables + static_cast<int64_t>(b) * p.max_blocks +
                              tok / p.block_size);
        if (blk < 0 || static_cast<int64_t>(blk) >= p.num_blocks) {
          raise_error(NKV_DEVERR_DECODE_BLOCK);
          row = -2 * kPrefillKeyTile;  // fully out of range: zeros
        } else {
          row = blk * p.block_size + (tok % p.block_size);
        }
      } else {
        row = k0 + tok;
      }
      const uint32_t fb = smem_u32(&full_bar[stage]);
      mbar_arrive_expect_tx(fb, 4u * kPrefillHalfKV);
      armed[stage] = phase + 1u;
      const uint32_t base = smem_u32(stage_mem + stage * kPrefillStageBytes);
      tma_load_3d(base + 0 * kPrefillHalfKV, &tm_k, fb, 0, kvh, row, pol_stream);
      tma_load_3d(base + 1 * kPrefillHalfKV, &tm_k, fb, 64, kvh, row, pol_stream);
      tma_load_3d(base + 2 * kPrefillHalfKV, &tm_v, fb, 0, kvh, row, pol_stream);
      tma_load_3d(base + 3 * kPrefillHalfKV, &tm_v, fb, 64, kvh, row, pol_stream);
      if (++stage == kPrefillStages) {
        stage = 0;
        phase ^= 1u;
      }
    }
    // Drain outstanding transactions before leaving (only after an abort).
#pragma unroll
    for (int s = 0; s < kPrefillStages; ++s)
      if (armed[s]) mbar_wait_bounded(smem_u32(&full_bar[s]), armed[s] - 1u);
    mbar_wait_bounded(smem_u32(q_bar), 0);
    return;
  }

  // -------------------------------------------------------------- consumers
  const int cw = warp;
  const int gid = lane >> 2;
  const int tig = lane & 3;
  const float NEG_INF = -INFINITY;
  const float scale_log2 = p.scale_log2;
  // This thread's two rows of the warp's m-tile: rho = 16*cw + gid (+8).
  const int rho0 = 16 * cw + gid;
  const int rho1 = rho0 + 8;
  const int qi0 = rho0 / G, qi1 = rho1 / G;  // query positions within the tile
  const int lim0 = shift + qs + qi0;         // last admissible key (causal)
  const int lim1 = shift + qs + qi1;

  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_run[2] = {NEG_INF, NEG_INF}, l_run[2] = {0.f, 0.f};

  // Q fragments (A operand) of the warp's 16 rows, from the swizzled q-tile.
  uint32_t qa[8][4];
  const bool q_ok = mbar_wait_bounded(smem_u32(q_bar), 0);
  {
    const uint8_t* qlo = q_mem;
    const uint8_t* qhi = q_mem + kPrefillQHalf;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const uint8_t* qh = (kk < 4) ? qlo : qhi;
      const uint32_t c = 2u * (kk & 3);
      qa[kk][0] = *reinterpret_cast<const uint32_t*>(qh + swz128(rho0, c) + 4 * tig);
      qa[kk][1] = *reinterpret_cast<const uint32_t*>(qh + swz128(rho1, c) + 4 * tig);
      qa[kk][2] = *reinterpret_cast<const uint32_t*>(qh + swz128(rho0, c + 1) + 4 * tig);
      qa[kk][3] = *reinterpret_cast<const uint32_t*>(qh + swz128(rho1, c + 1) + 4 * tig);
    }
  }

  int stage = 0;
  uint32_t phase = 0;
  for (int t = 0; t < ntiles && q_ok; ++t) {
    if (!mbar_wait_bounded(smem_u32(&full_bar[stage]), phase)) break;
    const uint32_t sK0 = smem_u32(stage_mem + stage * kPrefillStageBytes);
    const uint32_t sK1 = sK0 + kPrefillHalfKV;
    const uint32_t sV0 = sK0 + 2 * kPrefillHalfKV;
    const uint32_t sV1 = sK0 + 3 * kPrefillHalfKV;
    const int tok0 = t * kPrefillKeyTile;

    float sacc[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.f;
#pragma unroll
    for (int kp = 0; kp < 4; ++kp) {
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const uint32_t r = nt * 8 + (lane & 7);
        const uint32_t c16 = kp * 4 + (lane >> 3);
        const uint32_t addr = ((c16 < 8) ? sK0 : sK1) + swz128(r, c16 & 7u);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(addr, b0, b1, b2, b3);
        mma_bf16_16816(sacc[nt], qa[2 * kp][0], qa[2 * kp][1], qa[2 * kp][2], qa[2 * kp][3], b0,
                       b1);
        mma_bf16_16816(sacc[nt], qa[2 * kp + 1][0], qa[2 * kp + 1][1], qa[2 * kp + 1][2],
                       qa[2 * kp + 1][3], b2, b3);
      }
    }
    // masks: keys past Lk (last tile) and, with causal, past each row's limit
    const bool need_mask =
        (tok0 + kPrefillKeyTile > Lk) ||
        (p.causal && tok0 + kPrefillKeyTile - 1 > shift + qs);
    float pr[8][4];
#pragma unroll
    for (int rs = 0; rs < 2; ++rs) {
      const int lim = rs ? lim1 : lim0;
      float mx = NEG_INF;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float v = sacc[nt][2 * rs + e] * scale_log2;
          if (need_mask) {
            const int key = tok0 + nt * 8 + 2 * tig + e;
            if (key >= Lk || (p.causal && key > lim)) v = NEG_INF;
          }
          sacc[nt][2 * rs + e] = v;
          mx = fmaxf(mx, v);
        }
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_run[rs], mx);
      const float m_use = (m_new == NEG_INF) ? 0.f : m_new;
      const float alpha = fast_exp2(m_run[rs] - m_use);
      m_run[rs] = m_new;
      float rsum = 0.f;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float pv = fast_exp2(sacc[nt][2 * rs + e] - m_use);
          pr[nt][2 * rs + e] = pv;
          rsum += pv;
        }
      }
      l_run[rs] = l_run[rs] * alpha + rsum;
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        o[n][2 * rs] *= alpha;
        o[n][2 * rs + 1] *= alpha;
      }
    }
    // O += P V over the tile's four 16-key k-steps. V rows past Lk are zeroed
    // in registers so uninitialised cache bytes never meet a zero weight.
    const bool tail = tok0 + kPrefillKeyTile > Lk;
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const uint32_t a0 = pack_bf16x2(pr[2 * jj][0], pr[2 * jj][1]);
      const uint32_t a1 = pack_bf16x2(pr[2 * jj][2], pr[2 * jj][3]);
      const uint32_t a2 = pack_bf16x2(pr[2 * jj + 1][0], pr[2 * jj + 1][1]);
      const uint32_t a3 = pack_bf16x2(pr[2 * jj + 1][2], pr[2 * jj + 1][3]);
      uint32_t mask_lo = 0xffffffffu, mask_hi = 0xffffffffu;
      if (tail) {
        const int ta = tok0 + 16 * jj + 2 * tig;
        mask_lo = (ta < Lk ? 0x0000ffffu : 0u) | (ta + 1 < Lk ? 0xffff0000u : 0u);
        mask_hi = (ta + 8 < Lk ? 0x0000ffffu : 0u) | (ta + 9 < Lk ? 0xffff0000u : 0u);
      }
      const int mi = lane >> 3;
      const uint32_t r = 16 * jj + (mi & 1) * 8 + (lane & 7);
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        const uint32_t c16 = 2 * dp + (mi >> 1);
        const uint32_t addr = ((c16 < 8) ? sV0 : sV1) + swz128(r, c16 & 7u);
        uint32_t v0, v1, v2, v3;
        ldsm_x4_trans(addr, v0, v1, v2, v3);
        v0 &= mask_lo;
        v2 &= mask_lo;
        v1 &= mask_hi;
        v3 &= mask_hi;
        mma_bf16_16816(o[2 * dp], a0, a1, a2, a3, v0, v1);
        mma_bf16_16816(o[2 * dp + 1], a0, a1, a2, a3, v2, v3);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&empty_bar[stage]));
    if (++stage == kPrefillStages) {
      stage = 0;
      phase ^= 1u;
    }
  }

  // ---------------------------------------------------------------- epilogue
#pragma unroll
  for (int rs = 0; rs < 2; ++rs) {
    float l = l_run[rs];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    const int qi = rs ? qi1 : qi0;
    const int r = (rs ? rho1 : rho0) % G;
    if (qi < qn) {
      const float inv = (l > 0.f) ? 1.f / l : 0.f;
      __nv_bfloat16* dst = p.out + static_cast<int64_t>(q0 + qs + qi) * p.out_stride_token +
                           static_cast<int64_t>(kvh * G + r) * 128;
#pragma unroll
      for (int n = 0; n < 16; ++n)
        *reinterpret_cast<uint32_t*>(dst + 8 * n + 2 * tig) =
            pack_bf16x2(o[n][2 * rs] * inv, o[n][2 * rs + 1] * inv);
    }
  }
}

}  // namespace nkv
