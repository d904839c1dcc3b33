// o_proj GEMM fused with the tensor-parallel all-reduce that follows it:
// the B200 replacement for RowParallelLinear.forward,
//   y = F.linear(x, W_local); dist.all_reduce(y)     nanokvllm/layers/linear.py:151-155
// for decode-sized token counts (T <= 512), in ONE kernel per rank:
//   * tcgen05 GEMM: output tile t (columns [t*TN, (t+1)*TN) of the hidden
//     dim, all T rows in up to four 128-row M tiles accumulated in TMEM) is
//     computed by a cluster of S CTAs, CTA j taking the K range
//     [j*K/S, (j+1)*K/S) -- so each CTA streams only 1/S of x and of its W
//     slice (TMA, 128-byte swizzle, no multicast, a ring of up to 6
//     stages; one thread issues UMMA 128 x TN x 16);
//   * epilogue: S > 1: each CTA stores its fp32 partial tile to an
//     L2-resident workspace, the cluster synchronises, and CTA j sums rows
//     [j*Tp/S, (j+1)*Tp/S) over the S K ranges (in K order); the sum -- or,
//     with S = 1, the accumulator -- is rounded to bf16 (the reference's
//     F.linear output type) into a block in shared memory (the drained
//     ring), which one thread sends with a bulk copy (cp.async.bulk, the
//     TMA engine, no multicast) -- large transfers, so NVLink carries them
//     at full width. The bf16 [T, N] buffers below are tile-major,
//     [N / TN][T][TN], so a CTA's block is contiguous there:
//       two-shot mode: to this rank's copy of a symmetric bf16 [T, N]
//         partial buffer; barrier 1; each rank reduces its 1/world slice
//         with multimem.ld_reduce.add.acc::f32 (NVLink SHARP: the NVSwitch
//         reads every rank's bf16 partial, sums in fp32, returns bf16) and
//         broadcasts it into every rank's copy of a symmetric bf16 [T, N]
//         result buffer with multimem.st (four 16-byte reductions in flight
//         per thread); barrier 2; the tile's CTAs copy their share to y.
//         NVLink traffic per rank does not grow with the group.
//       one-shot mode: into this rank's slot of EVERY rank's receive buffer
//         (a bulk copy per rank, over NVLink for the others, issued while
//         other tiles still run their GEMM); one barrier; every rank sums
//         the world slots of its tile in rank order (fp32, so every rank
//         holds the same bf16 result) into y. Receive buffers alternate
//         between two parities per call, so no second barrier guards their
//         reuse: a rank can only be one call ahead of the slowest.
// A barrier: every CTA fences its stores (fence.acq_rel.sys) and adds one
// to every rank's arrival counter (one multimem.red through the switch, or
// a red per rank), then waits until its own rank's counter reaches this
// call's target (ld.acquire.sys, bounded by %globaltimer). Counters only
// grow; the targets and the call's epoch (its parity) live in device memory
// and are advanced by CTA 0 once every CTA has read them, so a CUDA graph can
// replay the launch. The launch is cooperative (all CTAs resident: each
// waits on all the others).
// A wait that gives up never yields a plausible wrong result: the CTA records
// which wait failed in the call's status word (flags[3], sticky, plus
// NKV_DEVERR_WAIT_TIMEOUT in the device error word) and its share of the
// data becomes NaN -- a failed GEMM sends NaN partials (so every rank's sum
// of that tile is NaN), a failed rank barrier writes NaN to the CTA's rows of
// y instead of summing slots that may be incomplete -- and CTA 0 does not
// advance the targets after a barrier it did not pass. CTA 0 also records
// the tiling that ran in flags[2] ((TN << 8) | S, plus bit 16 when the launch
// lacked its clusters and each tile ran unsplit).
#pragma once
#include "nkv_common.cuh"
#include "tcgen05.cuh"

namespace nkv {

constexpr int kOpK = 64;            // K elements per stage (one 128-byte row)
constexpr int kOpMaxStages = 6;     // ring depth (fewer when the M tiles are many)
constexpr int kOpThreads = 192;     // warp 0 TMA, warp 1 MMA + TMEM, warps 2-5 epilogue
constexpr int kOpMaxMTiles = 4;     // T <= 512
constexpr int kOpATile = 128 * 128;  // one 128-row x 64-K bf16 tile, bytes
constexpr int kOpMaxSplits = 4;     // cluster size along K
constexpr int kOpReduceUnroll = 4;  // two-shot: switch reductions in flight per thread
constexpr int kOpSumBatch = 8;      // one-shot: result groups per thread in flight
constexpr int kOpSplitBatch = 3;    // split-K sum: 8-column groups per thread in flight
constexpr int kOpSendRows = 32;     // rows per bulk send (the next chunk is summed meanwhile)

struct OprojParams {
  // two-shot (NVLS) mode
  // (the bf16 [T, N] buffers are tile-major: [N / TN][T][TN])
  __nv_bfloat16* part_mc;          // multicast address of the bf16 [T, N] partial buffer
  __nv_bfloat16* part_local;       // this rank's copy of it
  __nv_bfloat16* out_mc;           // multicast address of the bf16 [T, N] gathered result
  const __nv_bfloat16* out_local;  // this rank's copy of it
  uint32_t* sig_mc;                // multicast address of the [2] arrival counters
  // one-shot (peer-store) mode, device arrays indexed by rank
  __nv_bfloat16* const* recv_peers;  // each rank's [2 parities][world][slot_stride] bf16
  uint32_t* const* sig_peers;        // each rank's [2] arrival counters
  int64_t slot_stride;               // elements per (parity, source rank) slot, >= T * N
  uint32_t* sig_local;    // this rank's [2] arrival counters
  float* splitk_ws;       // S > 1: fp32 partial tiles, [S][N / TN][TN / 4][mtiles * 128][4]
  unsigned int* flags;    // this rank's [target 1, target 2, tiling, status, epoch]
  __nv_bfloat16* y;
  int64_t ldy;
  int T, K, N;
  int mtiles;             // ceil(T / 128)
  int tn;                 // output columns per tile: 32, 64 or 128
  int splits;             // S: CTAs (one cluster) per tile, each a K / S range
  int stages;             // <= kOpMaxStages
  int rank, world;
  int one_shot;           // 1: peer-store mode, 0: NVLS mode
  uint64_t timeout_ns;
};

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const unsigned int* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// 2-D tiled TMA load (x = K, y = rows), 128-byte swizzle, no multicast.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

// flags[2] bit: the launch lacked its clusters and ran unsplit (see below).
constexpr uint32_t kOpTilingUnclustered = 1u << 16;

__device__ __forceinline__ uint4 pack8_bf16(const float (&a)[8]) {
  return make_uint4(pack_bf16x2(a[0], a[1]), pack_bf16x2(a[2], a[3]), pack_bf16x2(a[4], a[5]),
                    pack_bf16x2(a[6], a[7]));
}

// Cross-rank barrier `which` (0 or 1) with this call's counter target:
// every CTA arrives at every rank's counter after fencing its own stores (a
// release pattern at system scope), then waits for its rank's counter to
// reach the target (an acquire). Bounded by p.timeout_ns; returns false, to
// every thread of the CTA, if the wait gave up (`passed` is a shared word).
__device__ __forceinline__ bool rank_barrier(const OprojParams& p, int which, uint32_t target,
                                             volatile uint32_t* passed) {
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t ok = 1u;
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    if (p.one_shot) {
      for (int r = 0; r < p.world; ++r)
        asm volatile("red.relaxed.sys.global.add.u32 [%0], 1;" ::"l"(p.sig_peers[r] + which)
                     : "memory");
    } else {
      asm volatile("multimem.red.relaxed.sys.global.add.u32 [%0], 1;" ::"l"(p.sig_mc + which)
                   : "memory");
    }
    const uint64_t t0 = global_ns();
    while (static_cast<int32_t>(ld_acquire_sys(p.sig_local + which) - target) < 0) {
      if (global_ns() - t0 > p.timeout_ns) {
        ok = 0u;
        break;
      }
      __nanosleep(32);
    }
    *passed = ok;
  }
  __syncthreads();
  return *passed != 0u;
}

// Status bits of one call (flags[3]): which bounded wait gave up.
constexpr uint32_t kOpStatusRing = 1u;     // producer: a ring slot never freed
constexpr uint32_t kOpStatusMma = 2u;      // MMA issuer: a stage's TMA never landed
constexpr uint32_t kOpStatusAcc = 4u;      // epilogue: the accumulator never completed
constexpr uint32_t kOpStatusBarrier = 8u;  // a cross-rank barrier's counter never reached its target

// Records a failed wait: the call's sticky status word and the device error word.
__device__ __forceinline__ void op_fail(const OprojParams& p, uint32_t bit) {
  atomicOr(p.flags + 3, bit);
  raise_error(NKV_DEVERR_WAIT_TIMEOUT);
}

constexpr uint32_t kBf16NanPair = 0x7FC07FC0u;  // two bf16 quiet NaNs

// Sends rows [row, row + nrows) of this CTA's bf16 block -- rows
// [r0, r0 + ...) of tile `tile`, row-major in shared memory at `block` -- to
// the NVLS partial buffer, or (one-shot) into this rank's slot of every
// rank's receive buffer of the call's parity (peers first). One thread,
// after the writing threads' proxy fences and a CTA barrier; asynchronous:
// send_wait() completes every send of the thread.
__device__ __forceinline__ void send_rows(const OprojParams& p, uint32_t block, int tile, int r0,
                                          int row, int nrows, uint32_t parity) {
  const int64_t off = (static_cast<int64_t>(tile) * p.T + r0 + row) * p.tn;
  const uint32_t src = block + static_cast<uint32_t>(row * p.tn * 2);
  const uint32_t bytes = static_cast<uint32_t>(nrows * p.tn * 2);
  if (!p.one_shot) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(
                     p.part_local + off),
                 "r"(src), "r"(bytes)
                 : "memory");
  } else {
    const int64_t slot = (static_cast<int64_t>(parity) * p.world + p.rank) * p.slot_stride + off;
    for (int i = 0; i < p.world; ++i) {
      const int q = (p.rank + 1 + i) % p.world;
      asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(
                       p.recv_peers[q] + slot),
                   "r"(src), "r"(bytes)
                   : "memory");
    }
  }
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// The thread's bulk sends have completed; ordered before its later accesses.
__device__ __forceinline__ void send_wait() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  asm volatile("fence.proxy.async;" ::: "memory");
}

__global__ void __launch_bounds__(kOpThreads, 1)
oproj_allreduce_kernel(const __grid_constant__ CUtensorMap tm_x,
                       const __grid_constant__ CUtensorMap tm_w, const OprojParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int b_bytes = p.tn * 128;                        // W slice of one stage
  const int stage_bytes = p.mtiles * kOpATile + b_bytes;  // multiple of 1024
  const int stages = p.stages;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + stages * stage_bytes);
  uint64_t* full = bars;                   // [stages]
  uint64_t* empty = bars + kOpMaxStages;   // [stages]
  uint64_t* acc_full = bars + 2 * kOpMaxStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kOpMaxStages + 1);
  // status bits of this CTA's GEMM waits, and the last barrier's outcome
  volatile uint32_t* cta_status = tmem_slot + 1;
  volatile uint32_t* barrier_passed = tmem_slot + 2;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // A tile's p.splits CTAs are consecutive in x (one cluster). If the launch
  // did not get its clusters (a tool that relaunches the kernel may drop the
  // attribute: %cluster_nctarank is then 1), the CTAs cannot synchronise to
  // sum K ranges, so every CTA computes its tile over the whole K (S = 1)
  // and only the tile's first CTA sends it: the result is the same, only
  // slower. `nct` CTAs share a tile; S is the number of K ranges.
  const int nct = p.splits;
  const bool clustered = nct == 1 || static_cast<int>(cluster_nctarank()) == nct;
  const int S = clustered ? nct : 1;
  const int split = static_cast<int>(blockIdx.x) % nct;
  const bool publisher = S > 1 || split == 0;  // sends (part of) the tile
  const int tile = blockIdx.x / nct;
  const int n0 = tile * p.tn;
  const int kper = p.K / S;
  const int k0 = S > 1 ? split * kper : 0;
  // The call's epoch and counter targets live on the device (so the launch
  // can be replayed from a CUDA graph): every CTA reads them here, before
  // its first arrival; CTA 0 advances them after the call's last barrier.
  const uint32_t epoch = ld_acquire_gpu(p.flags + 4) + 1u;
  const uint32_t parity = epoch & 1u;
  const uint32_t arrivals = gridDim.x * static_cast<uint32_t>(p.world);
  const uint32_t target0 = ld_acquire_gpu(p.flags + 0) + arrivals;
  const uint32_t target1 = ld_acquire_gpu(p.flags + 1) + arrivals;
  const int ksteps = kper / kOpK;
  uint32_t cols = 32;
  while (cols < static_cast<uint32_t>(p.mtiles * p.tn)) cols <<= 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    mbar_init(smem_u32(acc_full), 1);
    fence_barrier_init();
    *cta_status = 0u;
    if (blockIdx.x == 0)
      p.flags[2] = (static_cast<uint32_t>(p.tn) << 8) | static_cast<uint32_t>(S) |
                   (clustered ? 0u : kOpTilingUnclustered);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dependency_wait();

  bool acc_ok = false;
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&tm_x);
      prefetch_tmap(&tm_w);
      uint32_t armed = 0u, par = 0u;
      for (int ks = 0; ks < ksteps; ++ks) {
        const int s = ks % stages;
        const uint32_t ph = (ks / stages) & 1;
        if (!mbar_wait_bounded(smem_u32(&empty[s]), ph ^ 1u)) {
          atomicOr(const_cast<uint32_t*>(cta_status), kOpStatusRing);
          break;
        }
        armed &= ~(1u << s);
        const uint32_t fb = smem_u32(&full[s]);
        mbar_arrive_expect_tx(fb, stage_bytes);
        armed |= 1u << s;
        par = (par & ~(1u << s)) | (ph << s);
        const uint32_t base = smem_u32(smem + s * stage_bytes);
        for (int mt = 0; mt < p.mtiles; ++mt)
          tma_load_2d(base + mt * kOpATile, &tm_x, fb, k0 + ks * kOpK, mt * 128);
        tma_load_2d(base + p.mtiles * kOpATile, &tm_w, fb, k0 + ks * kOpK, n0);
      }
      for (int s = 0; s < stages; ++s)
        if (armed & (1u << s)) mbar_wait_bounded(smem_u32(&full[s]), (par >> s) & 1u);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc = umma_idesc_bf16(128, p.tn, 0);
    bool ok = true;
    for (int ks = 0; ks < ksteps && ok; ++ks) {
      const int s = ks % stages;
      if (!mbar_wait_bounded(smem_u32(&full[s]), (ks / stages) & 1)) {
        ok = false;
        if (lane == 0) atomicOr(const_cast<uint32_t*>(cta_status), kOpStatusMma);
        break;
      }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t base = smem_u32(smem + s * stage_bytes);
        const uint32_t bb = base + p.mtiles * kOpATile;
        for (int mt = 0; mt < p.mtiles; ++mt) {
#pragma unroll
          for (int kk = 0; kk < kOpK / 16; ++kk) {
            // A = x rows, B = W rows, both K-major: 16 K per step, 32 bytes
            // into the swizzled 128-byte rows, 8-row groups 1024 B apart
            umma_ss(tmem + mt * p.tn, umma_desc_sw128(base + mt * kOpATile + kk * 32, 16, 1024),
                    umma_desc_sw128(bb + kk * 32, 16, 1024), idesc, (ks > 0 || kk > 0) ? 1u : 0u);
          }
        }
        umma_commit(smem_u32(&empty[s]));
      }
      __syncwarp();
    }
    if (lane == 0) umma_commit(smem_u32(acc_full));
    __syncwarp();
  } else {
    // acc_full: every MMA has completed, so every TMA load has landed and
    // the ring is free for staging
    acc_ok = mbar_wait_bounded(smem_u32(acc_full), 0);
    if (!acc_ok && lane == 0) atomicOr(const_cast<uint32_t*>(cta_status), kOpStatusAcc);
  }

  // ---------------------------------------------------------------- epilogue
  // warps 2-5, thread = one accumulator row. S > 1: the fp32 row to this K
  // range's workspace tile, laid out [column / 4][row][4] so that a warp's
  // 16-byte stores (32 consecutive rows) cover 512 contiguous bytes. S = 1:
  // the bf16 row into the shared-memory block [T][TN].
  const int tp = p.mtiles * 128;
  const int rows = tp / S;  // rows summed per cluster CTA, a multiple of 32
  const int64_t ws_tiles = static_cast<int64_t>(p.N / p.tn) * tp * p.tn;  // one K range
  __nv_bfloat16* block = reinterpret_cast<__nv_bfloat16*>(smem);
  if (warp >= 2 && acc_ok) {
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, +32)
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    float4* ws4 = reinterpret_cast<float4*>(p.splitk_ws + split * ws_tiles +
                                            static_cast<int64_t>(tile) * tp * p.tn);
    tc_fence_after();
    for (int mt = 0; mt < p.mtiles; ++mt) {
      const int r = mt * 128 + quarter * 32 + lane;
      for (int c = 0; c < p.tn; c += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_base + mt * p.tn + c, v);
        tmem_ld_wait(v);
        if (r >= p.T) {
        } else if (S > 1) {
#pragma unroll
          for (int i = 0; i < 8; ++i)
            __stcg(ws4 + static_cast<int64_t>(c / 4 + i) * tp + r,
                   make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                               __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3])));
        } else {
          uint4* dst = reinterpret_cast<uint4*>(block + r * p.tn + c);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float a[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) a[e] = __uint_as_float(v[8 * i + e]);
            dst[i] = pack8_bf16(a);
          }
        }
      }
    }
    fence_proxy_async_shared();  // block rows written for the bulk send (S = 1)
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, cols);
  }
  // A GEMM wait gave up: the accumulator is incomplete, so this CTA's
  // partial becomes NaN (its workspace tile, or with S = 1 its bf16 block)
  // and every rank's sum of the tile is NaN rather than a plausible value.
  const uint32_t gemm_status = *cta_status;
  if (gemm_status != 0u) {
    if (threadIdx.x == 0) op_fail(p, gemm_status);
    if (S > 1) {
      float4* ws4 = reinterpret_cast<float4*>(p.splitk_ws + split * ws_tiles +
                                              static_cast<int64_t>(tile) * tp * p.tn);
      const float nan = __uint_as_float(0x7FC00000u);
      for (int i = threadIdx.x; i < tp * p.tn / 4; i += kOpThreads)
        __stcg(ws4 + i, make_float4(nan, nan, nan, nan));
    } else {
      uint4* b4 = reinterpret_cast<uint4*>(block);
      for (int i = threadIdx.x; i < p.T * p.tn / 8; i += kOpThreads)
        b4[i] = make_uint4(kBf16NanPair, kBf16NanPair, kBf16NanPair, kBf16NanPair);
      fence_proxy_async_shared();
    }
    __syncthreads();
  }

  int r0 = 0, nrows = p.T;
  if (S > 1) {
    // ------------------------------------ split-K sum of this CTA's rows
    // the cluster barrier (release / acquire at cluster scope) makes every
    // CTA's workspace tile visible. Rows go in chunks of kOpSendRows, each
    // sent as soon as it is summed, so NVLink carries one chunk while the
    // next is summed. Within a chunk a warp takes 8 rows x 4 eight-column
    // groups (its reads: 128 contiguous bytes per group and K range),
    // kOpSplitBatch such items per thread with all their loads issued
    // before the sums, which run in K-range order; bf16 into the block
    cluster_sync_all();
    r0 = split * rows;
    nrows = max(0, min(rows, p.T - r0));
    const int gblocks = p.tn / 32;  // 4-group column blocks: 1, 2 or 4
    const float4* ws4 = reinterpret_cast<const float4*>(p.splitk_ws +
                                                        static_cast<int64_t>(tile) * tp * p.tn);
    for (int row0 = 0; row0 < nrows; row0 += kOpSendRows) {
      const int crows = min(kOpSendRows, nrows - row0);
      const int rtiles = (crows + 7) / 8;
      const int items = rtiles * gblocks * 32;
      for (int i0 = threadIdx.x; i0 < items; i0 += kOpSplitBatch * kOpThreads) {
        float4 u[kOpSplitBatch][kOpMaxSplits][2];
        int lr[kOpSplitBatch], g[kOpSplitBatch];
#pragma unroll
        for (int b = 0; b < kOpSplitBatch; ++b) {
          const int i = i0 + b * kOpThreads;
          const int t = i >> 5, l = i & 31;
          lr[b] = row0 + (t % rtiles) * 8 + (l & 7);
          g[b] = (t / rtiles) * 4 + (l >> 3);
          if (i < items && lr[b] < row0 + crows) {
#pragma unroll
            for (int q = 0; q < kOpMaxSplits; ++q) {
              if (q < S) {
                const float4* src = ws4 + q * (ws_tiles / 4) +
                                    static_cast<int64_t>(2 * g[b]) * tp + r0 + lr[b];
                u[b][q][0] = __ldcg(src);
                u[b][q][1] = __ldcg(src + tp);
              }
            }
          }
        }
#pragma unroll
        for (int b = 0; b < kOpSplitBatch; ++b) {
          const int i = i0 + b * kOpThreads;
          if (i >= items || lr[b] >= row0 + crows) continue;
          float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int q = 0; q < kOpMaxSplits; ++q) {
            if (q < S) {
              a[0] += u[b][q][0].x; a[1] += u[b][q][0].y; a[2] += u[b][q][0].z;
              a[3] += u[b][q][0].w; a[4] += u[b][q][1].x; a[5] += u[b][q][1].y;
              a[6] += u[b][q][1].z; a[7] += u[b][q][1].w;
            }
          }
          *reinterpret_cast<uint4*>(block + lr[b] * p.tn + 8 * g[b]) = pack8_bf16(a);
        }
      }
      fence_proxy_async_shared();  // this chunk's rows, for the bulk send
      __syncthreads();
      if (threadIdx.x == 0) send_rows(p, smem_u32(block), tile, r0, row0, crows, parity);
    }
  } else if (publisher && threadIdx.x == 0 && nrows > 0) {
    send_rows(p, smem_u32(block), tile, 0, 0, nrows, parity);
  }
  if (threadIdx.x == 0) send_wait();

  const int per_row = p.tn / 8;
  if (p.one_shot) {
    // ------------------------------------------------------------ barrier
    const bool passed = rank_barrier(p, 0, target0, barrier_passed);
    if (!passed) {
      // a rank's partials may be missing: this CTA's rows of y become NaN
      if (threadIdx.x == 0) op_fail(p, kOpStatusBarrier);
      const uint4 nan8 = make_uint4(kBf16NanPair, kBf16NanPair, kBf16NanPair, kBf16NanPair);
      for (int i = split * kOpThreads + threadIdx.x; i < p.T * per_row; i += nct * kOpThreads) {
        const int r = i / per_row;
        *reinterpret_cast<uint4*>(p.y + static_cast<int64_t>(r) * p.ldy + n0 +
                                  (i - r * per_row) * 8) = nan8;
      }
      return;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {  // every CTA read them before arriving
      p.flags[0] = target0;
      p.flags[4] = epoch;
    }
    // every rank's partial of this tile is in this rank's receive buffer:
    // sum them in rank order (the same order on every rank, so every rank
    // holds the same result) and write y; the tile's S CTAs share the rows
    // (kOpSumBatch groups per thread at a time, two slots' loads issued
    // together)
    const __nv_bfloat16* recv = p.recv_peers[p.rank] +
                                static_cast<int64_t>(parity) * p.world * p.slot_stride +
                                static_cast<int64_t>(tile) * p.T * p.tn;
    const int items = p.T * per_row;
    const int step = nct * kOpThreads;
    for (int i0 = split * kOpThreads + threadIdx.x; i0 < items; i0 += kOpSumBatch * step) {
      int64_t off[kOpSumBatch];
#pragma unroll
      for (int b = 0; b < kOpSumBatch; ++b) {
        const int i = i0 + b * step;
        off[b] = i < items ? static_cast<int64_t>(i) * 8 : -1;  // tile block, row-major
      }
      float a[kOpSumBatch][8] = {};
      for (int q0 = 0; q0 < p.world; q0 += 2) {
        uint4 u[2][kOpSumBatch];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int b = 0; b < kOpSumBatch; ++b)
            if (off[b] >= 0 && q0 + h < p.world)
              u[h][b] = __ldcg(reinterpret_cast<const uint4*>(recv + (q0 + h) * p.slot_stride +
                                                              off[b]));
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // rank order
          if (q0 + h >= p.world) break;
#pragma unroll
          for (int b = 0; b < kOpSumBatch; ++b) {
            if (off[b] < 0) continue;
            const uint32_t w4[4] = {u[h][b].x, u[h][b].y, u[h][b].z, u[h][b].w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              a[b][2 * e] += __uint_as_float(w4[e] << 16);
              a[b][2 * e + 1] += __uint_as_float(w4[e] & 0xffff0000u);
            }
          }
        }
      }
#pragma unroll
      for (int b = 0; b < kOpSumBatch; ++b) {
        if (off[b] < 0) continue;
        const int i = i0 + b * step;
        const int r = i / per_row;
        *reinterpret_cast<uint4*>(p.y + static_cast<int64_t>(r) * p.ldy + n0 +
                                  (i - r * per_row) * 8) = pack8_bf16(a[b]);
      }
    }
    return;
  }

  // ---------------------------------------------------------------- barrier 1
  // (on a timeout this CTA's share of the switch reduction broadcasts NaN,
  // so no rank reads a sum of partials that may be incomplete)
  const bool passed1 = rank_barrier(p, 0, target0, barrier_passed);
  if (!passed1 && threadIdx.x == 0) op_fail(p, kOpStatusBarrier);

  // ------------------------------------------------- reduce this rank's slice
  // 16-byte groups [lo, hi) of the T x N result: fp32 sum of every rank's
  // bf16 partial through the switch, bf16 to every rank's result buffer;
  // kOpReduceUnroll reductions in flight per thread before their stores
  {
    const int64_t total8 = static_cast<int64_t>(p.T) * p.N / 8;
    const int64_t lo = total8 * p.rank / p.world, hi = total8 * (p.rank + 1) / p.world;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * kOpThreads;
    for (int64_t i0 = lo + static_cast<int64_t>(blockIdx.x) * kOpThreads + threadIdx.x; i0 < hi;
         i0 += kOpReduceUnroll * stride) {
      uint32_t v[kOpReduceUnroll][4];
#pragma unroll
      for (int u = 0; u < kOpReduceUnroll; ++u) {
        const int64_t i = i0 + u * stride;
        if (i < hi && passed1) {
          asm volatile(
              "multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
              : "=r"(v[u][0]), "=r"(v[u][1]), "=r"(v[u][2]), "=r"(v[u][3])
              : "l"(p.part_mc + 8 * i)
              : "memory");
        } else {
          v[u][0] = v[u][1] = v[u][2] = v[u][3] = kBf16NanPair;
        }
      }
#pragma unroll
      for (int u = 0; u < kOpReduceUnroll; ++u) {
        const int64_t i = i0 + u * stride;
        if (i < hi)
          asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(
                           p.out_mc + 8 * i),
                       "f"(__uint_as_float(v[u][0])), "f"(__uint_as_float(v[u][1])),
                       "f"(__uint_as_float(v[u][2])), "f"(__uint_as_float(v[u][3]))
                       : "memory");
      }
    }
  }

  // ---------------------------------------------------------------- barrier 2
  const bool passed2 = rank_barrier(p, 1, target1, barrier_passed);
  if (!passed2) {
    // the gathered result may be incomplete: this CTA's rows of y become NaN
    if (threadIdx.x == 0) op_fail(p, kOpStatusBarrier);
    const uint4 nan8 = make_uint4(kBf16NanPair, kBf16NanPair, kBf16NanPair, kBf16NanPair);
    for (int i = split * kOpThreads + threadIdx.x; i < p.T * per_row; i += nct * kOpThreads) {
      const int r = i / per_row;
      *reinterpret_cast<uint4*>(p.y + static_cast<int64_t>(r) * p.ldy + n0 +
                                (i - r * per_row) * 8) = nan8;
    }
    return;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && passed1) {  // every CTA read them before arriving
    p.flags[0] = target0;
    p.flags[1] = target1;
    p.flags[4] = epoch;
  }

  // ---------------------------------------------------------------- copy out
  // the tile's columns of the gathered bf16 result -> y, shared by its S CTAs
  for (int i = split * kOpThreads + threadIdx.x; i < p.T * per_row; i += nct * kOpThreads) {
    const int r = i / per_row;
    const int c = n0 + (i - r * per_row) * 8;
    const uint4 v = __ldcg(reinterpret_cast<const uint4*>(
        p.out_local + static_cast<int64_t>(tile) * p.T * p.tn + static_cast<int64_t>(i) * 8));
    *reinterpret_cast<uint4*>(p.y + static_cast<int64_t>(r) * p.ldy + c) = v;
  }
}

}  // namespace nkv
