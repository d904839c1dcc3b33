// o_proj GEMM fused with the tensor-parallel all-reduce that follows it:
// the B200 replacement for RowParallelLinear.forward,
//   y = F.linear(x, W_local); dist.all_reduce(y)     nanokvllm/layers/linear.py:151-155
// for decode-sized token counts (T <= 512), in ONE kernel per rank:
//   * tcgen05 GEMM: CTA c owns output columns [c*TN, (c+1)*TN) of the
//     hidden dim for all T rows (up to four 128-row M tiles, accumulated in
//     TMEM), x and the W slice streamed by TMA (128-byte swizzle, no
//     multicast) through a ring of up to 4 stages, one thread issuing UMMA
//     128 x TN x 16.
//   * epilogue: the fp32 partial tile goes from TMEM to this rank's copy of
//     a symmetric fp32 [T, N] partial buffer (local stores);
//   * barrier 1 (all ranks' partials written), then each rank reduces its
//     1/world slice of the T x N elements with multimem.ld_reduce (NVLink
//     SHARP: the NVSwitch reads every rank's partial and returns the fp32
//     sum), rounds it to bf16 and broadcasts it into every rank's copy of a
//     symmetric bf16 [T, N] buffer with multimem.st -- each element crosses
//     NVLink once per direction and partials are never rounded before the
//     sum;
//   * barrier 2 (all slices broadcast), then each CTA copies its share of
//     the gathered result to y.
// A barrier: after fence.acq_rel.sys and a device-scope arrival counter, the
// last CTA of the rank stores the call's epoch into every rank's slot with
// multimem.st.release and waits for all ranks' epochs (bounded by
// %globaltimer; on timeout it flags NKV_DEVERR_WAIT_TIMEOUT and goes on),
// then releases the rank's other CTAs. Two barriers per call also order the
// buffers' reuse: no rank writes call n+1's partials or broadcasts before
// every rank has finished call n. The epoch counter lives in device memory,
// so a CUDA graph can replay the launch.
// The launch is cooperative (all CTAs resident: non-last CTAs wait on the
// last one); every wait is bounded.
#pragma once
#include "nkv_common.cuh"
#include "tcgen05.cuh"

namespace nkv {

constexpr int kOpK = 64;            // K elements per stage (one 128-byte row)
constexpr int kOpMaxStages = 6;    // ring depth (fewer when the M tiles are many)
constexpr int kOpThreads = 192;     // warp 0 TMA, warp 1 MMA + TMEM, warps 2-5 epilogue
constexpr int kOpMaxMTiles = 4;     // T <= 512
constexpr int kOpATile = 128 * 128;  // one 128-row x 64-K bf16 tile, bytes

struct OprojParams {
  float* part_mc;         // multicast address of the fp32 [T, N] partial buffer
  float* part_local;      // this rank's copy of it
  __nv_bfloat16* out_mc;  // multicast address of the bf16 [T, N] gathered result
  const __nv_bfloat16* out_local;  // this rank's copy of it
  uint32_t* sig_mc;       // multicast address of the [2][world] epoch slots
  uint32_t* sig_local;    // this rank's copy of the slots
  unsigned int* flags;    // this rank's [ctr 1, go 1, ctr 2, go 2, epoch]
  __nv_bfloat16* y;
  int64_t ldy;
  int T, K, N;
  int mtiles;             // ceil(T / 128)
  int tn;                 // output columns per CTA: 32, 64 or 128
  int stages;             // <= kOpMaxStages
  int rank, world;
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

// Cross-rank barrier `which` (0 or 1) of the call with `epoch`: every CTA
// arrives once; the rank's last CTA signals all ranks and waits for theirs,
// then releases the rank's CTAs. Bounded by p.timeout_ns.
__device__ __forceinline__ void rank_barrier(const OprojParams& p, int which, uint32_t epoch) {
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned int* ctr = p.flags + 2 * which;
    unsigned int* go = p.flags + 2 * which + 1;
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    const unsigned int old = atomic_add_acq_rel_gpu(ctr, 1u);
    if (old == gridDim.x - 1) {
      asm volatile("fence.acq_rel.sys;" ::: "memory");
      asm volatile("multimem.st.release.sys.global.b32 [%0], %1;" ::"l"(
                       p.sig_mc + which * p.world + p.rank),
                   "r"(epoch)
                   : "memory");
      const uint64_t t0 = global_ns();
      for (int r = 0; r < p.world; ++r) {
        while (static_cast<int32_t>(ld_acquire_sys(p.sig_local + which * p.world + r) - epoch) < 0) {
          if (global_ns() - t0 > p.timeout_ns) {
            raise_error(NKV_DEVERR_WAIT_TIMEOUT);
            break;
          }
          __nanosleep(32);
        }
      }
      *ctr = 0u;
      if (which == 1) p.flags[4] = epoch;  // the next call's base (all CTAs have read it)
      asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(go), "r"(epoch) : "memory");
    } else {
      const uint64_t t0 = global_ns();
      while (static_cast<int32_t>(ld_acquire_gpu(go) - epoch) < 0) {
        if (global_ns() - t0 > p.timeout_ns) {
          raise_error(NKV_DEVERR_WAIT_TIMEOUT);
          break;
        }
        __nanosleep(32);
      }
    }
  }
  __syncthreads();
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

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * p.tn;
  // The call's epoch lives on the device (so the launch can be replayed from
  // a CUDA graph): every CTA reads it here, before it arrives at the
  // counter that lets the last CTA advance it.
  const uint32_t epoch = ld_acquire_gpu(p.flags + 4) + 1u;
  const int ksteps = p.K / kOpK;
  uint32_t cols = 32;
  while (cols < static_cast<uint32_t>(p.mtiles * p.tn)) cols <<= 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    mbar_init(smem_u32(acc_full), 1);
    fence_barrier_init();
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

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&tm_x);
      prefetch_tmap(&tm_w);
      uint32_t armed = 0u, parity = 0u;
      for (int ks = 0; ks < ksteps; ++ks) {
        const int s = ks % stages;
        const uint32_t ph = (ks / stages) & 1;
        if (!mbar_wait_bounded(smem_u32(&empty[s]), ph ^ 1u)) break;
        armed &= ~(1u << s);
        const uint32_t fb = smem_u32(&full[s]);
        mbar_arrive_expect_tx(fb, stage_bytes);
        armed |= 1u << s;
        parity = (parity & ~(1u << s)) | (ph << s);
        const uint32_t base = smem_u32(smem + s * stage_bytes);
        for (int mt = 0; mt < p.mtiles; ++mt)
          tma_load_2d(base + mt * kOpATile, &tm_x, fb, ks * kOpK, mt * 128);
        tma_load_2d(base + p.mtiles * kOpATile, &tm_w, fb, ks * kOpK, n0);
      }
      for (int s = 0; s < stages; ++s)
        if (armed & (1u << s)) mbar_wait_bounded(smem_u32(&full[s]), (parity >> s) & 1u);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc = umma_idesc_bf16(128, p.tn, 0);
    bool ok = true;
    for (int ks = 0; ks < ksteps && ok; ++ks) {
      const int s = ks % stages;
      if (!mbar_wait_bounded(smem_u32(&full[s]), (ks / stages) & 1)) {
        ok = false;
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
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, +32)
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    if (mbar_wait_bounded(smem_u32(acc_full), 0)) {
      tc_fence_after();
      for (int mt = 0; mt < p.mtiles; ++mt) {
        const int r = mt * 128 + quarter * 32 + lane;
        for (int c = 0; c < p.tn; c += 32) {
          uint32_t v[32];
          tmem_ld32(tmem + lane_base + mt * p.tn + c, v);
          tmem_ld_wait(v);
          if (r < p.T) {
            float4* dst = reinterpret_cast<float4*>(p.part_local + static_cast<int64_t>(r) * p.N +
                                                    n0 + c);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              dst[i] = make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                   __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, cols);
  }

  // ---------------------------------------------------------------- barrier 1
  rank_barrier(p, 0, epoch);

  // ------------------------------------------------- reduce this rank's slice
  // elements [lo, hi) of the T x N result, 4 per step: fp32 sum of every
  // rank's partial through the switch, bf16 to every rank's result buffer
  {
    const int64_t total4 = static_cast<int64_t>(p.T) * p.N / 4;
    const int64_t lo = total4 * p.rank / p.world, hi = total4 * (p.rank + 1) / p.world;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * kOpThreads;
    for (int64_t i = lo + static_cast<int64_t>(blockIdx.x) * kOpThreads + threadIdx.x; i < hi;
         i += stride) {
      float a, b, c, d;
      asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
                   : "=f"(a), "=f"(b), "=f"(c), "=f"(d)
                   : "l"(p.part_mc + 4 * i)
                   : "memory");
      const float lo2 = __uint_as_float(pack_bf16x2(a, b));
      const float hi2 = __uint_as_float(pack_bf16x2(c, d));
      asm volatile("multimem.st.relaxed.sys.global.v2.f32 [%0], {%1, %2};" ::"l"(p.out_mc + 4 * i),
                   "f"(lo2), "f"(hi2)
                   : "memory");
    }
  }

  // ---------------------------------------------------------------- barrier 2
  rank_barrier(p, 1, epoch);

  // ---------------------------------------------------------------- copy out
  // this CTA's columns of the gathered bf16 result -> y
  const int per_row = p.tn / 8;
  for (int i = threadIdx.x; i < p.T * per_row; i += kOpThreads) {
    const int r = i / per_row;
    const int c = n0 + (i - r * per_row) * 8;
    const uint4 v = __ldcg(reinterpret_cast<const uint4*>(p.out_local + static_cast<int64_t>(r) * p.N + c));
    *reinterpret_cast<uint4*>(p.y + static_cast<int64_t>(r) * p.ldy + c) = v;
  }
}

}  // namespace nkv
