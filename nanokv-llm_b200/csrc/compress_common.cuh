// Building blocks shared by the two compression kernels (periodic window and
// KvChat threshold): block-wide reductions and scans, the deterministic
// bf16 top-k, and the in-place row compaction.
#pragma once
#include <cooperative_groups.h>

#include "nkv_common.cuh"

namespace nkv {

namespace cg = cooperative_groups;

constexpr int kCompressThreads = 256;
constexpr int kCompressWarps = kCompressThreads / 32;
constexpr int kCompressHeadDim = 128;
constexpr int kMaxWindowBlocks = 64;
constexpr int kReduceSlots = 16 * kCompressWarps;  // floats/ints of scratch for reductions

// ---------------------------------------------------------------- block helpers
// kThreads: the block size (a multiple of 32); `red` holds >= kThreads / 32
// values (16 * kThreads / 32 for block_reduce_vec).
template <int kThreads = kCompressThreads>
__device__ __forceinline__ int block_sum_int(int v, int* red) {
  constexpr int kWarps = kThreads / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = __reduce_add_sync(0xffffffffu, v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  int tot = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) tot += red[w];
  __syncthreads();
  return tot;
}

// Exclusive prefix sum over threads in index order.
template <int kThreads = kCompressThreads>
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

// In-place block-wide max (kMax) or sum over each of N per-thread values.
template <int N, bool kMax, int kThreads = kCompressThreads>
__device__ __forceinline__ void block_reduce_vec_impl(float (&v)[N], float* red) {
  constexpr int kWarps = kThreads / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int r = 0; r < N; ++r) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float x = __shfl_xor_sync(0xffffffffu, v[r], o);
      v[r] = kMax ? fmaxf(v[r], x) : v[r] + x;
    }
    if (lane == 0) red[r * kWarps + warp] = v[r];
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < N; ++r) {
    float a = red[r * kWarps];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) {
      const float x = red[r * kWarps + w];
      a = kMax ? fmaxf(a, x) : a + x;
    }
    v[r] = a;
  }
  __syncthreads();
}

template <int N, bool kMax>
__device__ __forceinline__ void block_reduce_vec(float (&v)[N], float* red) {
  block_reduce_vec_impl<N, kMax>(v, red);
}

// Bit pattern of a non-negative bf16 value: monotone in the value.
__device__ __forceinline__ uint32_t bf16_key(float v) {
  return static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v)));
}

// One warp finds, from a 256-bin histogram of keys (bin = one byte of the
// key), the largest bin b whose suffix count (keys in bins >= b) reaches
// `need`; returns b and the count of keys in bins above b. Lane l holds bins
// [255 - 8l - 7, 255 - 8l] (lane 0 the highest), so an inclusive scan over
// lanes is a scan from the top bin down.
__device__ __forceinline__ void radix_pick_bin(const int* hist, int need, int* out_bin,
                                               int* out_above) {
  const int lane = threadIdx.x & 31;
  int c[8];
  int tot = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    c[i] = hist[255 - 8 * lane - i];
    tot += c[i];
  }
  int incl = tot;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  const int excl = incl - tot;
  if (excl < need && incl >= need) {  // exactly one lane holds the bin
    int acc = excl;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (acc + c[i] >= need) {
        *out_bin = 255 - 8 * lane - i;
        *out_above = acc;
        break;
      }
      acc += c[i];
    }
  }
}

// Selects the `k` largest of keys[0, n) (ties -> lower index) and writes their
// indices, ascending, to out[0, k). Keys live in shared memory; `hist` is 256
// ints of shared scratch, `red` kReduceSlots. The k-th largest key is found by
// a two-pass radix select (high byte, then low byte among keys sharing the
// high byte: two histogram passes instead of a 16-round bitwise search);
// then each thread, owning a contiguous index range, emits its keys above
// the cut and, in index order, the first (k - above) keys equal to it.
template <int kThreads = kCompressThreads>
__device__ void topk_ascending(const uint16_t* keys, int n, int k, int* out, int* red, int* hist) {
  __shared__ int s_bin, s_above;
  if (k <= 0) {
    __syncthreads();
    return;
  }
  uint32_t prefix = 0;
  int above = 0;
  for (int pass = 0; pass < 2; ++pass) {
    for (int i = threadIdx.x; i < 256; i += kThreads) hist[i] = 0;
    __syncthreads();
    for (int t = threadIdx.x; t < n; t += kThreads) {
      const uint32_t key = keys[t];
      if (pass == 0) {
        atomicAdd(&hist[key >> 8], 1);
      } else if ((key >> 8) == (prefix >> 8)) {
        atomicAdd(&hist[key & 0xFFu], 1);
      }
    }
    __syncthreads();
    if (threadIdx.x < 32) radix_pick_bin(hist, k - above, &s_bin, &s_above);
    __syncthreads();
    prefix |= static_cast<uint32_t>(s_bin) << (pass == 0 ? 8 : 0);
    above += s_above;
    __syncthreads();  // s_bin / s_above are rewritten by the next pass
  }
  // prefix is now the k-th largest key; `above` keys are larger.
  const int per = (n + kThreads - 1) / kThreads;
  const int lo = threadIdx.x * per;
  const int hi = min(lo + per, n);
  const int need_eq = k - above;
  int eq = 0;
  for (int t = lo; t < hi; ++t) eq += (keys[t] == prefix) ? 1 : 0;
  const int eq_before = block_excl_scan<kThreads>(eq, red);
  int kept = 0;
  {
    int e = eq_before;
    for (int t = lo; t < hi; ++t) {
      const bool is_eq = keys[t] == prefix;
      kept += (keys[t] > prefix || (is_eq && e < need_eq)) ? 1 : 0;
      e += is_eq ? 1 : 0;
    }
  }
  int pos = block_excl_scan<kThreads>(kept, red);
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

// Moves rows src(i) -> dst(i), i in [0, n), of this CTA's kv-head slice (256
// bytes of K and of V per row) by bulk asynchronous copies, global -> shared
// -> global, with no data in registers: kBulkRows rows per chunk, two chunks
// in flight through `buf` (2 buffers x kBulkRows rows x K and V, 16-byte
// aligned). Thread t < 2 * kBulkRows owns array t / kBulkRows (0 K, 1 V) of
// row t % kBulkRows of every chunk: it issues that row's load, its store once
// the chunk's mbarrier has completed, and the refill of its buffer slot once
// its own store has read it. Safe for in-place compaction when source index
// >= destination index (the contract of compact_rows_pipelined): a chunk's
// stores start after every load of that chunk and of each earlier chunk has
// landed, and no chunk reads a row an earlier chunk writes. Rows with src ==
// dst or an unresolved slot (< 0) are skipped. `bars`: two mbarriers, which
// this function initialises. Returns false, uniformly, when a load never
// landed (NKV_DEVERR_WAIT_TIMEOUT is raised; that chunk and later ones are not
// stored); every store issued has been performed when it returns.
template <int kThreads, int kBulkRows, typename SlotFn>
__device__ bool compact_rows_bulk(__nv_bfloat16* k_cache, __nv_bfloat16* v_cache, int num_kv_heads,
                                  int head, int n, SlotFn slots, uint8_t* buf, uint64_t* bars) {
  static_assert(2 * kBulkRows <= kThreads, "one thread per (row, array)");
  constexpr uint32_t kRowBytes = kCompressHeadDim * 2;
  constexpr uint32_t kBufBytes = 2 * kBulkRows * kRowBytes;
  const int t = threadIdx.x;
  if (t == 0) {
    mbar_init(smem_u32(&bars[0]), 2 * kBulkRows);
    mbar_init(smem_u32(&bars[1]), 2 * kBulkRows);
    fence_barrier_init();
  }
  // the buffers were last accessed through the generic proxy
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncthreads();
  bool ok = true;
  if (t < 2 * kBulkRows) {
    const int arr = t / kBulkRows;
    const int r = t % kBulkRows;
    __nv_bfloat16* const base = arr == 0 ? k_cache : v_cache;
    const uint32_t slot0 = smem_u32(buf) + static_cast<uint32_t>(t) * kRowBytes;
    const int nchunks = (n + kBulkRows - 1) / kBulkRows;
    int64_t dst0 = -1, dst1 = -1;  // this thread's destination in buffer 0 / 1
    auto load = [&](int c) {
      const int i = c * kBulkRows + r;
      int64_t src = -1, dst = -1;
      if (i < n) slots(i, src, dst);
      const uint32_t bar = smem_u32(&bars[c & 1]);
      if (i < n && src >= 0 && dst >= 0 && src != dst) {
        mbar_arrive_expect_tx(bar, kRowBytes);
        bulk_load_row(slot0 + (c & 1) * kBufBytes,
                      base + (src * num_kv_heads + head) * kCompressHeadDim, kRowBytes, bar);
      } else {
        dst = -1;
        mbar_arrive(bar);
      }
      if (c & 1) dst1 = dst; else dst0 = dst;
    };
    if (nchunks > 0) load(0);
    if (nchunks > 1) load(1);
    for (int c = 0; c < nchunks; ++c) {
      if (!mbar_wait_bounded(smem_u32(&bars[c & 1]), (c >> 1) & 1)) {
        ok = false;
        break;
      }
      const int64_t dst = (c & 1) ? dst1 : dst0;
      if (dst >= 0) {
        bulk_store_row(base + (dst * num_kv_heads + head) * kCompressHeadDim,
                       slot0 + (c & 1) * kBufBytes, kRowBytes);
        bulk_commit();
      }
      if (c + 2 < nchunks) {
        if (dst >= 0) bulk_wait_read_all();
        load(c + 2);
      }
    }
    bulk_wait_all();
  }
  return __syncthreads_and(ok ? 1 : 0) != 0;
}

// Moves rows src(i) -> dst(i), i in [0, n), of this CTA's kv-head slice (256
// bytes of K and of V per row), kThreads / 4 rows per chunk (4 threads per
// row), with the reads of chunk
// c+1 overlapping the writes of chunk c. Safe for in-place compaction when
// source index(i) >= i and destinations are the window's positions 0..n-1:
//   * every source of a chunk lies at or beyond its own first destination,
//     so no chunk's writes reach a source of a LATER chunk, and a later
//     chunk never reads a row an earlier chunk wrote;
//   * a chunk's sources may lie in the NEXT chunk's destination range, so a
//     barrier separates the reads of chunk c from the writes of chunk c+1.
// Rows with src == dst or an unresolved slot (< 0) are skipped. `parts`
// selects the arrays moved: 1 K, 2 V, 3 both (two CTAs may then share a
// head's compaction, one array each, with no ordering between them).
template <int kThreads = kCompressThreads, typename SlotFn>
__device__ void compact_rows_pipelined(__nv_bfloat16* k_cache, __nv_bfloat16* v_cache,
                                       int num_kv_heads, int head, int n, SlotFn slots,
                                       int parts = 3) {
  const bool do_k = (parts & 1) != 0, do_v = (parts & 2) != 0;
  constexpr int kChunkRows = kThreads / 4;
  const int t = threadIdx.x;
  const int row = t >> 2;      // kChunkRows rows x 4 threads
  const int quarter = t & 3;   // 4 x 64 bytes of a 256-byte head row
  auto kptr = [&](int64_t slot) {
    return reinterpret_cast<uint4*>(k_cache + (slot * num_kv_heads + head) * kCompressHeadDim) +
           quarter * 4;
  };
  auto vptr = [&](int64_t slot) {
    return reinterpret_cast<uint4*>(v_cache + (slot * num_kv_heads + head) * kCompressHeadDim) +
           quarter * 4;
  };
  uint4 kc[4], vc[4];
  int64_t dst_c = -1;
  {
    int64_t src = -1;
    if (row < n) slots(row, src, dst_c);
    if (row < n && src >= 0 && dst_c >= 0 && src != dst_c) {
      const uint4* ks = kptr(src);
      const uint4* vs = vptr(src);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (do_k) kc[u] = ks[u];
        if (do_v) vc[u] = vs[u];
      }
    } else {
      dst_c = -1;
    }
  }
  __syncthreads();
  for (int base = 0; base < n; base += kChunkRows) {
    const int i = base + kChunkRows + row;
    uint4 kn[4], vn[4];
    int64_t dst_n = -1;
    if (i < n) {
      int64_t src = -1;
      slots(i, src, dst_n);
      if (src >= 0 && dst_n >= 0 && src != dst_n) {
        const uint4* ks = kptr(src);
        const uint4* vs = vptr(src);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (do_k) kn[u] = ks[u];
          if (do_v) vn[u] = vs[u];
        }
      } else {
        dst_n = -1;
      }
    }
    if (dst_c >= 0) {
      uint4* kd = kptr(dst_c);
      uint4* vd = vptr(dst_c);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (do_k) kd[u] = kc[u];
        if (do_v) vd[u] = vc[u];
      }
    }
    __syncthreads();
    dst_c = dst_n;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      kc[u] = kn[u];
      vc[u] = vn[u];
    }
  }
}

}  // namespace nkv
