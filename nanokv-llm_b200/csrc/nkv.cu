// C-ABI entry points of libnkv.so (declared in include/nkv.h).
//
// Host side of every call: validate arguments (returning an nkv_status, never
// throwing), encode TMA tensor maps where a kernel needs them, pick the launch
// shape and launch on the caller's stream. No entry point allocates device
// memory or synchronises the host, so all of them can be captured in a CUDA
// graph (the reference's decode graphs, model_runner.py:401-441).
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>

#include "nkv_common.cuh"
#include "paged_decode.cuh"
#include "paged_prefill.cuh"
#include "qk_norm_rope.cuh"
#include "oproj_allreduce.cuh"
#include "store_kvcache.cuh"
#include "threshold_compress.cuh"
#include "window_compress.cuh"

namespace {

thread_local int t_last_cuda_error = 0;

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return NKV_OK;
  t_last_cuda_error = static_cast<int>(e);
  return NKV_ERR_CUDA;
}

int launch_status() { return cuda_status(cudaGetLastError()); }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------- devices
constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {0};
std::mutex g_dev_mutex;

int sm_count(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return 148;
  if (g_sm_count[dev] == 0) {
    std::lock_guard<std::mutex> lock(g_dev_mutex);
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

// ---------------------------------------------------------------- TMA encode
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  std::call_once(g_encode_once, []() {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode;
}

// 3-D bf16 map {dim0 (contiguous), dim1, dim2} with byte strides for dims 1, 2,
// box {64, box1, box2} and 128-byte swizzle (64 bf16 = one 128-byte row).
int encode_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
              uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box1, uint32_t box2,
              CUtensorMapL2promotion promo) {
  auto fn = encode_fn();
  if (!fn) return NKV_ERR_CUDA;
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  const cuuint32_t box[3] = {64, box1, box2};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, promo,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? NKV_OK : NKV_ERR_ALIGNMENT;
}

// 2-D bf16 map {d0 (contiguous), d1 rows} with row stride `stride1_bytes`,
// box {64, box1} and 128-byte swizzle.
int encode_2d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t stride1_bytes,
              uint32_t box1) {
  auto fn = encode_fn();
  if (!fn) return NKV_ERR_CUDA;
  const cuuint64_t dims[2] = {d0, d1};
  const cuuint64_t strides[1] = {stride1_bytes};
  const cuuint32_t box[2] = {64, box1};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? NKV_OK : NKV_ERR_ALIGNMENT;
}

// ---------------------------------------------------------------- decode plan
struct DecodePlan {
  int g;
  int cluster;  // > 1: splits of a pair form one cluster (its size)
  int chunk_tokens;
  int max_splits;
  int pairs;
  size_t off_split_counters, off_part_ml, off_part_o, total;
};

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// Upper bound on batch * num_kv_heads per decode call (size of the fixed
// split-counter region of the workspace).
constexpr int kMaxDecodePairs = 1 << 16;

// Longest split (tokens of one sequence and kv head per work item).
#ifndef NKV_DECODE_MAX_SPLIT_TOKENS
#define NKV_DECODE_MAX_SPLIT_TOKENS 4096
#endif
// Shortest split when the launch has enough work items without finer ones.
#ifndef NKV_DECODE_MIN_SPLIT_TOKENS
#define NKV_DECODE_MIN_SPLIT_TOKENS 2048
#endif
// Work items aimed for per SM (of a 148-SM part) when every row is full.
#ifndef NKV_DECODE_TARGET_ITEMS_PER_SM
#define NKV_DECODE_TARGET_ITEMS_PER_SM 7
#endif
// Rows up to this many tokens are not split when the launch has no more
// (row, kv head) pairs than a 148-SM part has SMs (latency-bound small
// batches: a split costs a cross-CTA merge). 0 disables.
#ifndef NKV_DECODE_SMALL_ROW_TOKENS
#define NKV_DECODE_SMALL_ROW_TOKENS 1024
#endif
// Small launches -- at most 74 (row, kv head) pairs, so that every pair can
// have at least two CTAs on a 148-SM part -- split each row over a cluster of
// up to 8 CTAs whose partials merge through distributed shared memory. One SM
// pulls only ~85 GB/s through TMA, so a B = 1 step over 8 kv heads would
// otherwise run on 8 SMs, and a merge through global memory costs several
// L2 round trips. Rows longer than this many 128-token tiles per CTA use the
// ordinary splits instead. 0 disables.
#ifndef NKV_DECODE_CLUSTER_MAX_TILES
#define NKV_DECODE_CLUSTER_MAX_TILES 64
#endif

// Opt-in shared memory per block on sm_100 (227 KB).
constexpr int kSmemOptinBytes = 232448;

// Largest cluster of splits whose receive rows fit next to the kernel's
// shared memory for padded group width G (0 or 1: no cluster mode).
template <int G>
constexpr int decode_cluster_cap() {
  using S = nkv::DecodeShape<G>;
  const int room = (kSmemOptinBytes - S::kSmemBytes) / S::kRecvBytesPerSplit;
  return room < nkv::kDecodeMaxClusterSplits ? room : nkv::kDecodeMaxClusterSplits;
}

int decode_cluster_cap_for(int g) {
  if (g <= 1) return decode_cluster_cap<1>();
  if (g <= 2) return decode_cluster_cap<2>();
  if (g <= 4) return decode_cluster_cap<4>();
  if (g <= 8) return decode_cluster_cap<8>();
  return 0;  // G = 16: the receive rows do not fit
}

// Split size depends only on the shapes (not on the device or the lengths), so
// the workspace query and the launch always agree.
DecodePlan make_decode_plan(int batch, int hq, int hk, int max_blocks, int block_size) {
  DecodePlan pl{};
  pl.g = hq / hk;
  pl.pairs = batch * hk;
  // Long splits amortise each item's fixed costs (grab, first-tile latency,
  // merge); short ones let the dynamic scheduler balance ragged lengths and
  // shrink the tail. Measured on B200: 4 K-token splits are best for a full
  // TP1 launch, ~2 K for the small launches of a TP8 shard; aiming at ~7
  // items per SM when every row is full gives both. 1 block .. the maximum.
  const int64_t block_units = static_cast<int64_t>(pl.pairs) * std::max(max_blocks, 1);
  const int64_t target_items = NKV_DECODE_TARGET_ITEMS_PER_SM * 148;
  int cb = static_cast<int>(block_units / target_items);
  // Few (row, kv head) pairs with long rows (e.g. 16 rows x 1 kv head of 32k
  // tokens on a TP8 shard) would otherwise be cut into 1-block splits whose
  // fixed costs (grab, first-tile latency, a 128-way merge) dominate: keep
  // splits >= 2,048 tokens whenever that still gives every SM an item
  // (measured on that shard: 1-block splits 184 us, 1,024 tokens 83 us,
  // 2,048 tokens 65 us per launch).
  // Latency-bound shapes with few items in total (one short row) keep the
  // fine splits.
  const int min_cb = std::max(1, NKV_DECODE_MIN_SPLIT_TOKENS / block_size);
  if (cb < min_cb &&
      static_cast<int64_t>(pl.pairs) * ((std::max(max_blocks, 1) + min_cb - 1) / min_cb) >= 148)
    cb = min_cb;
  if (pl.pairs <= 148 && static_cast<int64_t>(std::max(max_blocks, 1)) * block_size <=
                            NKV_DECODE_SMALL_ROW_TOKENS)
    cb = std::max(cb, max_blocks);
  const int max_cb = std::max(1, NKV_DECODE_MAX_SPLIT_TOKENS / block_size);
  pl.chunk_tokens = std::min(std::max(cb, 1), max_cb) * block_size;
  const int64_t row_tokens = static_cast<int64_t>(std::max(max_blocks, 1)) * block_size;
  const int64_t row_tiles = (row_tokens + nkv::kDecodeTileTokens - 1) / nkv::kDecodeTileTokens;
  pl.cluster = 0;
  const int cap = std::min(decode_cluster_cap_for(pl.g), 148 / std::max(pl.pairs, 1));
  if (NKV_DECODE_CLUSTER_MAX_TILES > 0 && cap >= 2 && row_tiles >= 2) {
    const int64_t c = std::min<int64_t>(cap, row_tiles);
    const int64_t tiles = (row_tiles + c - 1) / c;
    if (tiles <= NKV_DECODE_CLUSTER_MAX_TILES) {
      pl.chunk_tokens = static_cast<int>(tiles * nkv::kDecodeTileTokens);
      pl.cluster = static_cast<int>((row_tokens + pl.chunk_tokens - 1) / pl.chunk_tokens);
      if (pl.cluster < 2) pl.cluster = 0;
    }
  }
  pl.max_splits = static_cast<int>(std::max<int64_t>(1, (row_tokens + pl.chunk_tokens - 1) / pl.chunk_tokens));
  // Layout: [scheduler counters][split counters for kMaxDecodePairs pairs]
  // [partial (m, l)][partial O]. The counter region has a FIXED size so
  // that, whatever shapes share one workspace, a counter never lands on
  // bytes another shape used for partial results (only counters must be
  // zero between calls; partials may hold anything).
  size_t off = 256;
  pl.off_split_counters = off;
  off = align256(off + sizeof(unsigned int) * kMaxDecodePairs);
  pl.off_part_ml = off;
  off = align256(off + sizeof(float) * 2 * static_cast<size_t>(pl.pairs) * pl.max_splits * pl.g);
  pl.off_part_o = off;
  off = align256(off + sizeof(float) * 128 * static_cast<size_t>(pl.pairs) * pl.max_splits * pl.g);
  pl.total = off;
  return pl;
}

template <int G>
int launch_decode(const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tq,
                  const nkv::DecodeParams& p, cudaStream_t stream) {
  using S = nkv::DecodeShape<G>;
  constexpr int kCap = decode_cluster_cap<G>();
  constexpr int kMaxSmem = S::kSmemBytes + (kCap > 1 ? kCap : 0) * S::kRecvBytesPerSplit;
  static bool attr_set[kMaxDevices] = {false};
  // clusters of C splits that fit at once, per device and C (-1 = not asked)
  static int active_clusters[kMaxDevices][nkv::kDecodeMaxClusterSplits + 1];
  static std::once_flag init_once;
  std::call_once(init_once, [] {
    for (auto& row : active_clusters)
      for (int& v : row) v = -1;
  });
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) return NKV_ERR_CUDA;
  if (!attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(nkv::paged_decode_kernel<G>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
    if (e != cudaSuccess) return cuda_status(e);
    attr_set[dev] = true;
  }
  nkv::DecodeParams q = p;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(nkv::kDecodeThreads, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (q.cluster > 1 && q.cluster <= kCap) {
    // One cluster per pair, all resident at once (the leader waits for its
    // peers); otherwise the same splits merge through global memory.
    cfg.gridDim = dim3(q.total_items, 1, 1);
    cfg.dynamicSmemBytes = S::kSmemBytes + q.cluster * S::kRecvBytesPerSplit;
    attr[1].val.clusterDim.x = q.cluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
    int& fit = active_clusters[dev][q.cluster];
    if (fit < 0) {
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, nkv::paged_decode_kernel<G>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
      }
      fit = n;
    }
    if (fit * q.cluster < q.total_items) q.cluster = 0;
  } else {
    q.cluster = 0;
  }
  if (q.cluster == 0) {
    cfg.gridDim = dim3(std::max(1, std::min(sm_count(dev), q.total_items)), 1, 1);
    cfg.dynamicSmemBytes = S::kSmemBytes;
    cfg.numAttrs = 1;
  }
  return cuda_status(cudaLaunchKernelEx(&cfg, nkv::paged_decode_kernel<G>, tk, tv, tq, q));
}

int padded_group(int g) {
  if (g <= 1) return 1;
  if (g <= 2) return 2;
  if (g <= 4) return 4;
  if (g <= 8) return 8;
  if (g <= 16) return 16;
  return 0;
}

constexpr size_t kMaxSmem = 227 * 1024;

// launch_threshold: the requested cluster does not fit this GPU (not a
// public status; the caller falls back to smaller clusters).
constexpr int kThresholdNoFit = 0x7fff0000;

// Launches `kernel` (blocks of `threads`) with clusters of cluster_x CTAs
// along x. `smem_set` is
// the caller's per-kernel record of the dynamic shared-memory limit already
// granted on each device; the limit is raised only when a call needs more.
template <typename Kernel, typename Params>
int launch_cluster(Kernel kernel, int threads, size_t* smem_set, const Params& p, int cluster_x,
                   int grid_y, size_t smem, cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices || smem > smem_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_status(e);
    if (dev >= 0 && dev < kMaxDevices) smem_set[dev] = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cluster_x, grid_y, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster_x;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kernel, p));
}

template <int G>
int launch_threshold(const nkv::ThresholdCompressParams& p, int cluster_x, int grid_y,
                     size_t smem, cudaStream_t stream) {
  static size_t smem_set[kMaxDevices] = {0};
  auto kernel = nkv::threshold_compress_kernel<G>;
  if (cluster_x > 8) {
    // a non-portable cluster size: allowed explicitly, and used only when
    // such a cluster fits the GPU (else the caller plans 8-CTA clusters)
    static bool nonportable[kMaxDevices] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= kMaxDevices) return NKV_ERR_CUDA;
    if (!nonportable[dev]) {
      if (cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) !=
          cudaSuccess) {
        cudaGetLastError();
        return kThresholdNoFit;
      }
      nonportable[dev] = true;
    }
    if (smem > smem_set[dev]) {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
      if (e != cudaSuccess) return cuda_status(e);
      smem_set[dev] = smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cluster_x, 1, 1);
    cfg.blockDim = dim3(nkv::kThrThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cluster_x;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess || n < 1) {
      cudaGetLastError();
      return kThresholdNoFit;
    }
  }
  return launch_cluster(kernel, nkv::kThrThreads, smem_set, p, cluster_x, grid_y, smem, stream);
}

template <int G>
int launch_window(const CUtensorMap& tk, const CUtensorMap& tv, const nkv::WindowCompressParams& p,
                  int cluster_x, int grid_y, size_t smem, cudaStream_t stream) {
  static size_t smem_set[kMaxDevices] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices || smem > smem_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(nkv::window_compress_kernel<G>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_status(e);
    if (dev >= 0 && dev < kMaxDevices) smem_set[dev] = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cluster_x, grid_y, 1);
  cfg.blockDim = dim3(nkv::kCompressThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster_x;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, nkv::window_compress_kernel<G>, tk, tv, p));
}

}  // namespace

extern "C" {

const char* nkv_status_string(int status) {
  switch (status) {
    case NKV_OK: return "NKV_OK";
    case NKV_ERR_INVALID_ARGUMENT: return "NKV_ERR_INVALID_ARGUMENT";
    case NKV_ERR_UNSUPPORTED: return "NKV_ERR_UNSUPPORTED";
    case NKV_ERR_WORKSPACE: return "NKV_ERR_WORKSPACE";
    case NKV_ERR_ALIGNMENT: return "NKV_ERR_ALIGNMENT";
    case NKV_ERR_CUDA: return "NKV_ERR_CUDA";
    default: return "NKV_ERR_UNKNOWN";
  }
}

int nkv_abi_version(void) { return 102; }

int nkv_last_cuda_error(void) { return t_last_cuda_error; }

int nkv_read_device_error(uint32_t* out_bits, int clear) {
  if (!out_bits) return NKV_ERR_INVALID_ARGUMENT;
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, nkv::g_nkv_error, sizeof(v));
  if (e != cudaSuccess) return cuda_status(e);
  *out_bits = v;
  if (clear) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(nkv::g_nkv_error, &zero, sizeof(zero));
    if (e != cudaSuccess) return cuda_status(e);
  }
  return NKV_OK;
}

// ------------------------------------------------------------------ store
int nkv_store_kvcache(const void* key, int64_t key_stride, const void* value, int64_t value_stride,
                      void* k_cache, void* v_cache, int64_t num_slots,
                      const int32_t* slot_mapping, int32_t num_tokens, int32_t num_kv_heads,
                      int32_t head_dim, void* stream) {
  if (num_tokens < 0 || num_slots < 0 || num_kv_heads <= 0 || head_dim <= 0)
    return NKV_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0 || num_slots == 0) return NKV_OK;
  if (!key || !value || !k_cache || !v_cache || !slot_mapping) return NKV_ERR_INVALID_ARGUMENT;
  const int64_t row = static_cast<int64_t>(num_kv_heads) * head_dim;
  if ((row % 8) != 0 || (key_stride % 8) != 0 || (value_stride % 8) != 0 || !aligned16(key) ||
      !aligned16(value) || !aligned16(k_cache) || !aligned16(v_cache))
    return NKV_ERR_ALIGNMENT;
  if (key_stride < row || value_stride < row) return NKV_ERR_INVALID_ARGUMENT;
  const int blocks = (num_tokens + nkv::kStoreWarpsPerBlock - 1) / nkv::kStoreWarpsPerBlock;
  nkv::store_kvcache_kernel<<<blocks, nkv::kStoreWarpsPerBlock * 32, 0,
                              static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(key), key_stride / 8, static_cast<const uint4*>(value),
      value_stride / 8, static_cast<uint4*>(k_cache), static_cast<uint4*>(v_cache), num_slots,
      slot_mapping, num_tokens, static_cast<int32_t>(row / 8));
  return launch_status();
}

// ------------------------------------------------------------------ decode
size_t nkv_paged_decode_workspace_size(int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                                       int32_t head_dim, int32_t max_blocks, int32_t block_size) {
  if (batch <= 0 || num_kv_heads <= 0 || num_q_heads <= 0 || block_size <= 0 ||
      num_q_heads % num_kv_heads != 0 ||
      static_cast<int64_t>(batch) * num_kv_heads > kMaxDecodePairs)
    return 0;
  (void)head_dim;
  return make_decode_plan(batch, num_q_heads, num_kv_heads, max_blocks, block_size).total;
}

}  // extern "C"

namespace {

// The new-row and query-window inputs of a fused decode step.
struct FusedStep {
  const void* key = nullptr;
  int64_t key_stride = 0;
  const void* value = nullptr;
  int64_t value_stride = 0;
  const int32_t* slot_mapping = nullptr;
  void* ring = nullptr;
  int32_t num_ring_slots = 0, num_layers = 0, window_size = 0, layer_id = 0;
  const int32_t* ring_slot_of_row = nullptr;
  const int32_t* ring_pos_of_row = nullptr;
  int32_t metadata_ready = 0;
};

int paged_decode_impl(const void* q, int64_t q_stride_token, int64_t q_stride_head,
                      const void* k_cache, const void* v_cache, int64_t num_blocks,
                      const int32_t* block_tables, int32_t max_blocks, const int32_t* context_lens,
                      void* out, int64_t out_stride_token, int32_t batch, int32_t num_q_heads,
                      int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                      float softmax_scale, void* workspace, size_t workspace_bytes, void* stream,
                      const FusedStep* fused) {
  if (batch < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || max_blocks < 0 || num_blocks < 0)
    return NKV_ERR_INVALID_ARGUMENT;
  if (batch == 0) return NKV_OK;
  if (!q || !k_cache || !v_cache || !block_tables || !context_lens || !out)
    return NKV_ERR_INVALID_ARGUMENT;
  if (num_q_heads % num_kv_heads != 0) return NKV_ERR_INVALID_ARGUMENT;
  if (head_dim != nkv::kDecodeHeadDim || block_size <= 0 ||
      block_size % nkv::kDecodeTileTokens != 0)
    return NKV_ERR_UNSUPPORTED;
  const int g = num_q_heads / num_kv_heads;
  const int G = padded_group(g);
  if (G == 0) return NKV_ERR_UNSUPPORTED;
  if (static_cast<int64_t>(batch) * num_kv_heads > kMaxDecodePairs) return NKV_ERR_UNSUPPORTED;
  if (!std::isfinite(softmax_scale)) return NKV_ERR_INVALID_ARGUMENT;
  if (out_stride_token < static_cast<int64_t>(num_q_heads) * head_dim) return NKV_ERR_INVALID_ARGUMENT;
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || (q_stride_token % 8) ||
      (q_stride_head % 8) || (reinterpret_cast<uintptr_t>(out) & 7u) || (out_stride_token % 4))
    return NKV_ERR_ALIGNMENT;
  const DecodePlan pl = make_decode_plan(batch, num_q_heads, num_kv_heads, max_blocks, block_size);
  if (!workspace || workspace_bytes < pl.total) return NKV_ERR_WORKSPACE;
  if (num_blocks == 0 || max_blocks == 0) num_blocks = std::max<int64_t>(num_blocks, 0);

  const uint64_t num_slots = static_cast<uint64_t>(std::max<int64_t>(num_blocks, 1)) * block_size;
  const uint64_t row_bytes = static_cast<uint64_t>(num_kv_heads) * head_dim * 2;
  CUtensorMap tk, tv, tq;
  int st;
  if ((st = encode_3d(&tk, k_cache, head_dim, num_kv_heads, num_slots, head_dim * 2, row_bytes,
                      1, nkv::kDecodeTileTokens, CU_TENSOR_MAP_L2_PROMOTION_L2_256B)) != NKV_OK)
    return st;
  if ((st = encode_3d(&tv, v_cache, head_dim, num_kv_heads, num_slots, head_dim * 2, row_bytes,
                      1, nkv::kDecodeTileTokens, CU_TENSOR_MAP_L2_PROMOTION_L2_256B)) != NKV_OK)
    return st;
  if ((st = encode_3d(&tq, q, head_dim, num_q_heads, batch, q_stride_head * 2, q_stride_token * 2,
                      g, 1, CU_TENSOR_MAP_L2_PROMOTION_NONE)) != NKV_OK)
    return st;

  nkv::DecodeParams p{};
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.block_tables = block_tables;
  p.context_lens = context_lens;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride_token = out_stride_token;
  p.num_blocks = num_blocks;
  p.counters = reinterpret_cast<unsigned int*>(ws);
  p.split_counters = reinterpret_cast<unsigned int*>(ws + pl.off_split_counters);
  p.part_ml = reinterpret_cast<float*>(ws + pl.off_part_ml);
  p.part_o = reinterpret_cast<float*>(ws + pl.off_part_o);
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.max_blocks = max_blocks;
  p.batch = batch;
  p.num_kv_heads = num_kv_heads;
  p.g = g;
  p.block_size = block_size;
  p.chunk_tokens = pl.chunk_tokens;
  p.max_splits = pl.max_splits;
  p.cluster = pl.cluster;
  p.total_items = pl.pairs * pl.max_splits;
  if (fused != nullptr) {
    const int64_t row = static_cast<int64_t>(num_kv_heads) * head_dim;
    if (!fused->key || !fused->value || !fused->slot_mapping) return NKV_ERR_INVALID_ARGUMENT;
    if (!aligned16(fused->key) || !aligned16(fused->value) || (fused->key_stride % 8) ||
        (fused->value_stride % 8))
      return NKV_ERR_ALIGNMENT;
    if (fused->key_stride < row || fused->value_stride < row) return NKV_ERR_INVALID_ARGUMENT;
    p.new_k = static_cast<const uint4*>(fused->key);
    p.new_v = static_cast<const uint4*>(fused->value);
    p.new_k_stride_vec = fused->key_stride / 8;
    p.new_v_stride_vec = fused->value_stride / 8;
    p.slot_mapping = fused->slot_mapping;
    p.metadata_ready = fused->metadata_ready;
    p.k_cache_vec = static_cast<uint4*>(const_cast<void*>(k_cache));
    p.v_cache_vec = static_cast<uint4*>(const_cast<void*>(v_cache));
    if (fused->ring != nullptr) {
      if (!fused->ring_slot_of_row || !fused->ring_pos_of_row || fused->num_ring_slots <= 0 ||
          fused->num_layers <= 0 || fused->window_size <= 0 || fused->layer_id < 0 ||
          fused->layer_id >= fused->num_layers)
        return NKV_ERR_INVALID_ARGUMENT;
      if (q_stride_head != head_dim || !aligned16(fused->ring)) return NKV_ERR_ALIGNMENT;
      const int64_t per_pos = static_cast<int64_t>(num_q_heads) * head_dim / 8;
      p.q_vec = static_cast<const uint4*>(q);
      p.q_stride_token_vec = q_stride_token / 8;
      p.ring_vec = static_cast<uint4*>(fused->ring);
      p.ring_slot_of_row = fused->ring_slot_of_row;
      p.ring_pos_of_row = fused->ring_pos_of_row;
      p.ring_window = fused->window_size;
      p.ring_slots = fused->num_ring_slots;
      p.num_q_heads = num_q_heads;
      p.ring_layer_base_vec = static_cast<int64_t>(fused->layer_id) * fused->window_size * per_pos;
      p.ring_slot_stride_vec =
          static_cast<int64_t>(fused->num_layers) * fused->window_size * per_pos;
    }
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (G) {
    case 1: return launch_decode<1>(tk, tv, tq, p, s);
    case 2: return launch_decode<2>(tk, tv, tq, p, s);
    case 4: return launch_decode<4>(tk, tv, tq, p, s);
    case 8: return launch_decode<8>(tk, tv, tq, p, s);
    default: return launch_decode<16>(tk, tv, tq, p, s);
  }
}

}  // namespace

// ---------------------------------------------------------------- o_proj + all-reduce
namespace {

// Tiling choice and cooperative launch of oproj_allreduce_kernel; `p` comes
// with its buffers, rank and mode filled in.
int oproj_launch(nkv::OprojParams p, const void* x, int64_t ldx, const void* w, int64_t ldw,
                 int32_t tokens, int32_t k, int32_t n, void* workspace, int64_t workspace_bytes,
                 void* y, int64_t ldy, void* stream) {
  if (tokens > nkv::kOpMaxMTiles * 128 || k % nkv::kOpK != 0 || n % 32 != 0) return NKV_ERR_UNSUPPORTED;
  if (ldx < k || ldw < k || ldy < n) return NKV_ERR_INVALID_ARGUMENT;
  if (!aligned16(x) || !aligned16(w) || !aligned16(y) || (ldx % 8) || (ldw % 8) || (ldy % 8) ||
      !aligned16(workspace))
    return NKV_ERR_ALIGNMENT;
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = sm_count(dev);
  const int mtiles = (tokens + 127) / 128;
  constexpr int kSmemLimit = 227 * 1024;
  const int fixed = 1024 + 256;  // alignment slack, barriers, TMEM slot
  p.y = static_cast<__nv_bfloat16*>(y);
  p.ldy = ldy;
  p.T = tokens;
  p.K = k;
  p.N = n;
  p.mtiles = mtiles;
  p.splitk_ws = static_cast<float*>(workspace);

  // Tile width TN and split count S: fewest bytes streamed per CTA
  // ((rows + TN) * K/S bf16, plus the fp32 tile written and read back for
  // the cluster sum when S > 1) with at most one CTA per SM, TN * mtiles
  // TMEM columns, and S fp32 [mtiles * 128, n] slices fitting the workspace.
  auto stages_for = [&](int tn) {
    const int stage_bytes = mtiles * nkv::kOpATile + tn * 128;
    return std::make_pair(std::min(nkv::kOpMaxStages, (kSmemLimit - fixed) / stage_bytes),
                          stage_bytes);
  };
  auto fits = [&](int tn, int S) {
    if (n % tn != 0 || (n / tn) * S > sms || mtiles * tn > 512) return false;
    if (k % (S * nkv::kOpK) != 0) return false;
    const auto st = stages_for(tn);
    if (st.first < 2) return false;
    if (S > 1 && (workspace == nullptr ||
                  static_cast<int64_t>(S) * mtiles * 128 * n * 4 > workspace_bytes))
      return false;
    return true;
  };
  auto cost = [&](int tn, int S) {
    const int64_t bytes = static_cast<int64_t>(mtiles * 128 + tn) * (k / S) * 2;
    return bytes + (S > 1 ? static_cast<int64_t>(mtiles) * 128 * tn * 8 : 0);
  };
  auto launch = [&](int tn, int S) -> int {
    const auto st = stages_for(tn);
    const int smem = st.first * st.second + fixed;
    CUtensorMap tx, tw;
    int rc;
    if ((rc = encode_2d(&tx, x, k, tokens, ldx * 2, 128)) != NKV_OK) return rc;
    if ((rc = encode_2d(&tw, w, k, n, ldw * 2, tn)) != NKV_OK) return rc;
    p.tn = tn;
    p.splits = S;
    p.stages = st.first;
    static int attr_smem[kMaxDevices] = {0};
    if (dev >= 0 && dev < kMaxDevices && attr_smem[dev] < smem) {
      cudaError_t e = cudaFuncSetAttribute(nkv::oproj_allreduce_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return cuda_status(e);
      attr_smem[dev] = smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((n / tn) * S, 1, 1);
    cfg.blockDim = dim3(nkv::kOpThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: the barrier waits on peers
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = S;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = S > 1 ? 2 : 1;
    if (S > 1) {
      cudaLaunchConfig_t q = cfg;  // the cluster shape alone, for the residency query
      q.attrs = attr + 1;
      q.numAttrs = 1;
      int clusters = 0;
      if (cudaOccupancyMaxActiveClusters(&clusters, nkv::oproj_allreduce_kernel, &q) !=
              cudaSuccess ||
          clusters < n / tn) {
        cudaGetLastError();
        return NKV_ERR_UNSUPPORTED;
      }
    }
    return cuda_status(cudaLaunchKernelEx(&cfg, nkv::oproj_allreduce_kernel, tx, tw, p));
  };

  int best_tn = 0, best_s = 0;
  int64_t best = 0;
  for (int S = 1; S <= nkv::kOpMaxSplits; S *= 2)
    for (int tn = 32; tn <= 128; tn *= 2)
      if (fits(tn, S) && (best_tn == 0 || cost(tn, S) < best)) {
        best = cost(tn, S);
        best_tn = tn;
        best_s = S;
      }
  if (best_tn == 0) return NKV_ERR_UNSUPPORTED;
  int rc = launch(best_tn, best_s);
  if (rc == NKV_OK || best_s == 1) return rc;
  // the clusters do not all fit at once here, or a cooperative launch of
  // clusters was refused: the best single-CTA tiling
  cudaGetLastError();
  best_tn = 0;
  for (int tn = 32; tn <= 128; tn *= 2)
    if (fits(tn, 1) && (best_tn == 0 || cost(tn, 1) < best)) {
      best = cost(tn, 1);
      best_tn = tn;
    }
  if (best_tn == 0) return NKV_ERR_UNSUPPORTED;
  return launch(best_tn, 1);
}

}  // namespace

extern "C" {

int nkv_paged_decode(const void* q, int64_t q_stride_token, int64_t q_stride_head,
                     const void* k_cache, const void* v_cache, int64_t num_blocks,
                     const int32_t* block_tables, int32_t max_blocks, const int32_t* context_lens,
                     void* out, int64_t out_stride_token, int32_t batch, int32_t num_q_heads,
                     int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                     float softmax_scale, void* workspace, size_t workspace_bytes, void* stream) {
  return paged_decode_impl(q, q_stride_token, q_stride_head, k_cache, v_cache, num_blocks,
                           block_tables, max_blocks, context_lens, out, out_stride_token, batch,
                           num_q_heads, num_kv_heads, head_dim, block_size, softmax_scale,
                           workspace, workspace_bytes, stream, nullptr);
}

int nkv_decode_step(const void* q, int64_t q_stride_token, int64_t q_stride_head, const void* key,
                    int64_t key_stride, const void* value, int64_t value_stride,
                    const int32_t* slot_mapping, void* k_cache, void* v_cache, int64_t num_blocks,
                    const int32_t* block_tables, int32_t max_blocks, const int32_t* context_lens,
                    void* ring, int32_t num_ring_slots, int32_t num_layers, int32_t window_size,
                    int32_t layer_id, const int32_t* ring_slot_of_row,
                    const int32_t* ring_pos_of_row, void* out, int64_t out_stride_token,
                    int32_t batch, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                    int32_t block_size, float softmax_scale, int32_t metadata_ready,
                    void* workspace, size_t workspace_bytes, void* stream) {
  if (metadata_ready != 0 && metadata_ready != 1) return NKV_ERR_INVALID_ARGUMENT;
  FusedStep f;
  f.metadata_ready = metadata_ready;
  f.key = key;
  f.key_stride = key_stride;
  f.value = value;
  f.value_stride = value_stride;
  f.slot_mapping = slot_mapping;
  f.ring = ring;
  f.num_ring_slots = num_ring_slots;
  f.num_layers = num_layers;
  f.window_size = window_size;
  f.layer_id = layer_id;
  f.ring_slot_of_row = ring_slot_of_row;
  f.ring_pos_of_row = ring_pos_of_row;
  return paged_decode_impl(q, q_stride_token, q_stride_head, k_cache, v_cache, num_blocks,
                           block_tables, max_blocks, context_lens, out, out_stride_token, batch,
                           num_q_heads, num_kv_heads, head_dim, block_size, softmax_scale,
                           workspace, workspace_bytes, stream, &f);
}

// ---------------------------------------------------------------- q/k norm + RoPE + store
int nkv_qk_norm_rope_store(const void* qkv, int64_t qkv_stride_token, int32_t num_tokens,
                           const int64_t* positions, const float* cos_sin_cache,
                           int64_t max_positions, const void* q_norm_weight,
                           const void* k_norm_weight, float eps, void* q_out,
                           int64_t q_out_stride_token, void* k_out, int64_t k_out_stride_token,
                           void* k_cache, void* v_cache, int64_t num_slots,
                           const int32_t* slot_mapping, int32_t num_q_heads, int32_t num_kv_heads,
                           int32_t head_dim, void* stream) {
  if (num_tokens < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || max_positions <= 0 ||
      num_slots < 0)
    return NKV_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return NKV_OK;
  if (head_dim != 128) return NKV_ERR_UNSUPPORTED;
  if (!qkv || !positions || !cos_sin_cache || !q_norm_weight || !k_norm_weight || !q_out)
    return NKV_ERR_INVALID_ARGUMENT;
  if (k_cache && (!v_cache || !slot_mapping)) return NKV_ERR_INVALID_ARGUMENT;
  if (!(eps >= 0.f) || !std::isfinite(eps)) return NKV_ERR_INVALID_ARGUMENT;
  const int64_t heads = static_cast<int64_t>(num_q_heads) + 2 * num_kv_heads;
  if (qkv_stride_token < heads * head_dim || q_out_stride_token < int64_t(num_q_heads) * head_dim ||
      (k_out && k_out_stride_token < int64_t(num_kv_heads) * head_dim))
    return NKV_ERR_INVALID_ARGUMENT;
  if (!aligned16(qkv) || !aligned16(q_out) || !aligned16(q_norm_weight) ||
      !aligned16(k_norm_weight) || (k_out && !aligned16(k_out)) ||
      (k_cache && (!aligned16(k_cache) || !aligned16(v_cache))) || !aligned16(cos_sin_cache) ||
      (qkv_stride_token % 8) || (q_out_stride_token % 8) || (k_out && (k_out_stride_token % 8)))
    return NKV_ERR_ALIGNMENT;
  nkv::NormRopeParams p{};
  p.qkv = static_cast<const __nv_bfloat16*>(qkv);
  p.qkv_stride = qkv_stride_token;
  p.positions = positions;
  p.cos_sin = cos_sin_cache;
  p.max_positions = max_positions;
  p.q_weight = static_cast<const __nv_bfloat16*>(q_norm_weight);
  p.k_weight = static_cast<const __nv_bfloat16*>(k_norm_weight);
  p.eps = eps;
  p.q_out = static_cast<__nv_bfloat16*>(q_out);
  p.q_out_stride = q_out_stride_token;
  p.k_out = static_cast<__nv_bfloat16*>(k_out);
  p.k_out_stride = k_out_stride_token;
  p.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  p.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  p.num_slots = num_slots;
  p.slot_mapping = slot_mapping;
  p.num_tokens = num_tokens;
  p.num_q_heads = num_q_heads;
  p.num_kv_heads = num_kv_heads;
  // 4-head groups; one warp per token when tokens are plenty, one group per
  // warp for small (decode) batches
  const int64_t groups = (heads + 3) / 4;
  const int64_t gpw = std::min<int64_t>(
      groups, std::max<int64_t>(1, (int64_t(num_tokens) * groups + 32767) / 32768));
  p.groups_per_warp = static_cast<int>(gpw);
  p.warps_per_token = static_cast<int>((groups + gpw - 1) / gpw);
  const int64_t warps = static_cast<int64_t>(num_tokens) * p.warps_per_token;
  const int64_t blocks = (warps + nkv::kNormRopeWarps - 1) / nkv::kNormRopeWarps;
  if (blocks > 0x7fffffff) return NKV_ERR_UNSUPPORTED;
  nkv::qk_norm_rope_kernel<<<static_cast<unsigned>(blocks), nkv::kNormRopeWarps * 32, 0,
                             static_cast<cudaStream_t>(stream)>>>(p);
  return launch_status();
}

// ---------------------------------------------------------------- o_proj + all-reduce
int nkv_oproj_allreduce(const void* x, int64_t ldx, const void* w, int64_t ldw, int32_t tokens,
                        int32_t k, int32_t n, void* part_mc, void* part_local, void* out_mc,
                        const void* out_local, void* sig_mc, void* sig_local, uint32_t* flags,
                        int32_t rank, int32_t world, uint64_t timeout_ns, void* workspace,
                        int64_t workspace_bytes, void* y, int64_t ldy, void* stream) {
  if (tokens < 0 || k <= 0 || n <= 0 || world < 1 || rank < 0 || rank >= world)
    return NKV_ERR_INVALID_ARGUMENT;
  if (tokens == 0) return NKV_OK;
  if (!x || !w || !part_mc || !part_local || !out_mc || !out_local || !sig_mc || !sig_local ||
      !flags || !y)
    return NKV_ERR_INVALID_ARGUMENT;
  if (!aligned16(part_mc) || !aligned16(part_local) || !aligned16(out_mc) ||
      !aligned16(out_local) || (reinterpret_cast<uintptr_t>(sig_mc) & 3u) ||
      (reinterpret_cast<uintptr_t>(sig_local) & 3u))
    return NKV_ERR_ALIGNMENT;
  nkv::OprojParams p{};
  p.part_mc = static_cast<__nv_bfloat16*>(part_mc);
  p.part_local = static_cast<__nv_bfloat16*>(part_local);
  p.out_mc = static_cast<__nv_bfloat16*>(out_mc);
  p.out_local = static_cast<const __nv_bfloat16*>(out_local);
  p.sig_mc = static_cast<uint32_t*>(sig_mc);
  p.sig_local = static_cast<uint32_t*>(sig_local);
  p.flags = reinterpret_cast<unsigned int*>(flags);
  p.rank = rank;
  p.world = world;
  p.one_shot = 0;
  p.timeout_ns = timeout_ns;
  return oproj_launch(p, x, ldx, w, ldw, tokens, k, n, workspace, workspace_bytes, y, ldy, stream);
}

int nkv_oproj_allreduce_p2p(const void* x, int64_t ldx, const void* w, int64_t ldw,
                            int32_t tokens, int32_t k, int32_t n, void* const* recv_peers,
                            int64_t slot_stride, uint32_t* const* sig_peers, void* sig_local,
                            uint32_t* flags, int32_t rank, int32_t world, uint64_t timeout_ns,
                            void* workspace, int64_t workspace_bytes, void* y, int64_t ldy,
                            void* stream) {
  if (tokens < 0 || k <= 0 || n <= 0 || world < 1 || rank < 0 || rank >= world)
    return NKV_ERR_INVALID_ARGUMENT;
  if (tokens == 0) return NKV_OK;
  if (!x || !w || !recv_peers || !sig_peers || !sig_local || !flags || !y)
    return NKV_ERR_INVALID_ARGUMENT;
  if (slot_stride < static_cast<int64_t>(tokens) * n) return NKV_ERR_INVALID_ARGUMENT;
  if ((slot_stride % 8) || (reinterpret_cast<uintptr_t>(recv_peers) & 7u) ||
      (reinterpret_cast<uintptr_t>(sig_peers) & 7u) ||
      (reinterpret_cast<uintptr_t>(sig_local) & 3u))
    return NKV_ERR_ALIGNMENT;
  nkv::OprojParams p{};
  p.recv_peers = reinterpret_cast<__nv_bfloat16* const*>(recv_peers);
  p.sig_peers = reinterpret_cast<uint32_t* const*>(sig_peers);
  p.slot_stride = slot_stride;
  p.sig_local = static_cast<uint32_t*>(sig_local);
  p.flags = reinterpret_cast<unsigned int*>(flags);
  p.rank = rank;
  p.world = world;
  p.one_shot = 1;
  p.timeout_ns = timeout_ns;
  return oproj_launch(p, x, ldx, w, ldw, tokens, k, n, workspace, workspace_bytes, y, ldy, stream);
}

// ---------------------------------------------------------------- prefill
int nkv_paged_prefill(const void* q, int64_t q_stride_token, int64_t q_stride_head,
                      int64_t num_q_tokens, const void* k, int64_t k_stride_token, const void* v,
                      int64_t v_stride_token, int64_t num_kv_rows, const int32_t* block_tables,
                      int32_t max_blocks, int32_t block_size, const int32_t* cu_seqlens_q,
                      const int32_t* cu_seqlens_k, int32_t batch, int32_t max_seqlen_q,
                      int32_t causal, void* out, int64_t out_stride_token, int32_t num_q_heads,
                      int32_t num_kv_heads, int32_t head_dim, float softmax_scale, void* stream) {
  if (batch < 0 || max_seqlen_q < 0 || num_q_tokens < 0 || num_kv_rows < 0 || num_q_heads <= 0 ||
      num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0)
    return NKV_ERR_INVALID_ARGUMENT;
  if (batch == 0 || max_seqlen_q == 0 || num_q_tokens == 0) return NKV_OK;
  if (!q || !k || !v || !cu_seqlens_q || !cu_seqlens_k || !out) return NKV_ERR_INVALID_ARGUMENT;
  if (!std::isfinite(softmax_scale) || !(softmax_scale > 0.f)) return NKV_ERR_INVALID_ARGUMENT;
  const int g = num_q_heads / num_kv_heads;
  if (head_dim != 128 || g > nkv::kPrefillRows || batch > 65535 || num_kv_heads > 65535)
    return NKV_ERR_UNSUPPORTED;
  // A 128-key tile spans whole cache blocks (64-token blocks: two per tile)
  // or lies inside one (multiples of 128).
  if (block_tables != nullptr &&
      (max_blocks <= 0 || !(block_size == 64 || (block_size > 0 && block_size % 128 == 0))))
    return NKV_ERR_UNSUPPORTED;
  const int qt = nkv::kPrefillRows / g;
  const int64_t qtiles = (static_cast<int64_t>(max_seqlen_q) + qt - 1) / qt;
  if (qtiles > (1ll << 31) - 1) return NKV_ERR_UNSUPPORTED;
  const int64_t row = static_cast<int64_t>(num_kv_heads) * head_dim;
  if (k_stride_token < row || v_stride_token < row ||
      out_stride_token < static_cast<int64_t>(num_q_heads) * head_dim ||
      q_stride_head < head_dim || q_stride_token < q_stride_head * (num_q_heads - 1) + head_dim)
    return NKV_ERR_INVALID_ARGUMENT;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || (q_stride_token % 8) ||
      (q_stride_head % 8) || (k_stride_token % 8) || (v_stride_token % 8) ||
      !aligned16(out) || (out_stride_token % 8))
    return NKV_ERR_ALIGNMENT;
  const uint64_t kv_rows = static_cast<uint64_t>(std::max<int64_t>(num_kv_rows, 1));
  const int rows_per_load = block_tables ? std::min(block_size, nkv::kPrefillKeyTile)
                                         : nkv::kPrefillKeyTile;
  CUtensorMap tk, tv, tq;
  int st;
  if ((st = encode_3d(&tk, k, head_dim, num_kv_heads, kv_rows, head_dim * 2, k_stride_token * 2, 1,
                      rows_per_load, CU_TENSOR_MAP_L2_PROMOTION_L2_256B)) != NKV_OK)
    return st;
  if ((st = encode_3d(&tv, v, head_dim, num_kv_heads, kv_rows, head_dim * 2, v_stride_token * 2, 1,
                      rows_per_load, CU_TENSOR_MAP_L2_PROMOTION_L2_256B)) != NKV_OK)
    return st;
  if ((st = encode_3d(&tq, q, head_dim, num_q_heads, num_q_tokens, q_stride_head * 2,
                      q_stride_token * 2, g, qt, CU_TENSOR_MAP_L2_PROMOTION_NONE)) != NKV_OK)
    return st;

  nkv::PrefillParams p{};
  p.block_tables = block_tables;
  p.cu_q = cu_seqlens_q;
  p.cu_k = cu_seqlens_k;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride_token = out_stride_token;
  p.num_blocks = block_tables ? num_kv_rows / block_size : 0;
  p.num_q_tokens = num_q_tokens;
  p.num_kv_rows = num_kv_rows;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.max_blocks = max_blocks;
  p.batch = batch;
  p.num_kv_heads = num_kv_heads;
  p.g = g;
  p.qt = qt;
  p.block_size = block_size;
  p.rows_per_load = rows_per_load;
  p.causal = causal ? 1 : 0;
  p.qtiles = static_cast<int>(qtiles);

  static bool attr_set[kMaxDevices] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < kMaxDevices && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(nkv::paged_prefill_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         nkv::kPrefillSmemBytes);
    if (e != cudaSuccess) return cuda_status(e);
    attr_set[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(qtiles), num_kv_heads, batch);
  cfg.blockDim = dim3(nkv::kPrefillThreads, 1, 1);
  cfg.dynamicSmemBytes = nkv::kPrefillSmemBytes;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, nkv::paged_prefill_kernel, tk, tv, tq, p));
}

// ------------------------------------------------------------------ window compress
int nkv_window_compress(const void* q, int64_t q_stride_token, void* k_cache, void* v_cache,
                        int64_t num_blocks, const int32_t* block_tables, int32_t max_blocks,
                        const int32_t* base_context_lens, int32_t* context_lens,
                        const int32_t* selected_batch_indices, int32_t num_selected,
                        int32_t window_blocks, int32_t keep_tokens, int32_t obs_window,
                        int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                        int32_t block_size, float softmax_scale, int32_t* out_keep_idx,
                        int32_t* out_new_lens, void* out_importance, void* stream) {
  if (num_selected < 0) return NKV_ERR_INVALID_ARGUMENT;
  if (num_selected == 0) return NKV_OK;
  if (!q || !k_cache || !v_cache || !block_tables || !base_context_lens || !context_lens ||
      !selected_batch_indices)
    return NKV_ERR_INVALID_ARGUMENT;
  if (num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads) return NKV_ERR_INVALID_ARGUMENT;
  if (head_dim != nkv::kCompressHeadDim || num_kv_heads > 8 || obs_window != 1 || block_size <= 0 ||
      block_size % nkv::kWinTileTokens != 0)
    return NKV_ERR_UNSUPPORTED;
  const int g = num_q_heads / num_kv_heads;
  if (g > 16) return NKV_ERR_UNSUPPORTED;
  if (window_blocks <= 0 || window_blocks > nkv::kMaxWindowBlocks) return NKV_ERR_UNSUPPORTED;
  if (num_blocks <= 0) return NKV_ERR_INVALID_ARGUMENT;
  const int window_tokens = window_blocks * block_size;
  // SnapKV's own guard (CompressMethod.py:17-18) is the caller's job: the
  // Python layer skips the call, as the reference returns False.
  const int num_keep = keep_tokens - 1 - obs_window;
  if (window_tokens - obs_window <= 0 || window_tokens <= num_keep + obs_window || num_keep < 0)
    return NKV_ERR_INVALID_ARGUMENT;
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || (q_stride_token % 8))
    return NKV_ERR_ALIGNMENT;
  nkv::WindowCompressParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_stride_token = q_stride_token;
  p.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  p.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  p.num_blocks = num_blocks;
  p.block_tables = block_tables;
  p.base_lens = base_context_lens;
  p.context_lens = context_lens;
  p.selected = selected_batch_indices;
  p.out_keep_idx = out_keep_idx;
  p.out_new_lens = out_new_lens;
  p.out_importance = static_cast<uint16_t*>(out_importance);
  p.scale = softmax_scale;
  p.max_blocks = max_blocks;
  p.window_blocks = window_blocks;
  p.keep_tokens = keep_tokens;
  p.obs_window = obs_window;
  p.num_kv_heads = num_kv_heads;
  p.g = g;
  p.block_size = block_size;
  p.num_keys = window_tokens - obs_window;
  p.keys_pad = ((p.num_keys + nkv::kCompressThreads - 1) / nkv::kCompressThreads) * nkv::kCompressThreads;
  const int G = padded_group(g);
  const size_t smem = nkv::window_smem_bytes(G, p.keys_pad, keep_tokens);
  if (smem > kMaxSmem) return NKV_ERR_UNSUPPORTED;
  // K (and, for L2 prefetches, V) rows of one head in 64-token tiles (two
  // 64-dim halves, 128-byte swizzle)
  CUtensorMap tk, tv;
  const uint64_t num_slots = static_cast<uint64_t>(num_blocks) * block_size;
  const uint64_t row_bytes = static_cast<uint64_t>(num_kv_heads) * head_dim * 2;
  int st = encode_3d(&tk, k_cache, head_dim, num_kv_heads, num_slots, head_dim * 2, row_bytes, 1,
                     nkv::kWinTileTokens, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (st != NKV_OK) return st;
  st = encode_3d(&tv, v_cache, head_dim, num_kv_heads, num_slots, head_dim * 2, row_bytes, 1,
                 nkv::kWinTileTokens, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (st != NKV_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (G) {
    case 1: return launch_window<1>(tk, tv, p, num_kv_heads, num_selected, smem, s);
    case 2: return launch_window<2>(tk, tv, p, num_kv_heads, num_selected, smem, s);
    case 4: return launch_window<4>(tk, tv, p, num_kv_heads, num_selected, smem, s);
    case 8: return launch_window<8>(tk, tv, p, num_kv_heads, num_selected, smem, s);
    default: return launch_window<16>(tk, tv, p, num_kv_heads, num_selected, smem, s);
  }
}

int nkv_window_select(const int32_t* context_lens, const int32_t* tail_uncompressed,
                      int32_t batch, int32_t block_size, int32_t window_blocks, int32_t topk,
                      int32_t* out_selected, int32_t* out_count, int32_t* out_base_lens,
                      void* stream) {
  if (batch < 0 || topk < 0 || block_size <= 0 || window_blocks <= 0) return NKV_ERR_INVALID_ARGUMENT;
  if (topk == 0 && batch == 0) return NKV_OK;
  if ((batch > 0 && (!context_lens || !tail_uncompressed)) || (topk > 0 && !out_selected))
    return NKV_ERR_INVALID_ARGUMENT;
  nkv::WindowSelectParams p{};
  p.context_lens = context_lens;
  p.tail_uncompressed = tail_uncompressed;
  p.selected = out_selected;
  p.count = out_count;
  p.base_lens = out_base_lens;
  p.batch = batch;
  p.block_size = block_size;
  p.window_blocks = window_blocks;
  p.topk = topk;
  nkv::window_select_kernel<<<1, nkv::kSelectThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return launch_status();
}

// ------------------------------------------------------------------ KvChat
int nkv_query_window_append(const void* q, int64_t q_stride_token, void* ring,
                            int32_t num_ring_slots, int32_t num_layers, int32_t window_size,
                            int32_t layer_id, const int32_t* batch_index, const int32_t* ring_slot,
                            const int32_t* ring_pos, int32_t num_active, int32_t num_q_heads,
                            int32_t head_dim, void* stream) {
  if (num_active < 0) return NKV_ERR_INVALID_ARGUMENT;
  if (num_active == 0) return NKV_OK;
  if (!q || !ring || !batch_index || !ring_slot || !ring_pos) return NKV_ERR_INVALID_ARGUMENT;
  if (num_ring_slots <= 0 || num_layers <= 0 || window_size <= 0 || layer_id < 0 ||
      layer_id >= num_layers || num_q_heads <= 0 || head_dim <= 0)
    return NKV_ERR_INVALID_ARGUMENT;
  const int64_t row = static_cast<int64_t>(num_q_heads) * head_dim;
  if ((row % 8) || (q_stride_token % 8) || !aligned16(q) || !aligned16(ring)) return NKV_ERR_ALIGNMENT;
  nkv::query_window_append_kernel<<<num_active, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(q), q_stride_token, static_cast<__nv_bfloat16*>(ring),
      num_ring_slots, num_layers, window_size, layer_id, batch_index, ring_slot, ring_pos,
      static_cast<int>(row / 8));
  return launch_status();
}

int nkv_threshold_compress(const void* ring, int32_t num_ring_slots, int32_t num_layers,
                           int32_t window_size, int32_t layer_id,
                           const int32_t* ring_slot_of_selected, void* k_cache, void* v_cache,
                           int64_t num_blocks, const int32_t* block_tables, int32_t max_blocks,
                           int32_t* context_lens, const int32_t* selected_batch_indices,
                           int32_t num_selected, int32_t compress_S, int32_t compress_R,
                           int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                           int32_t block_size, float softmax_scale, int32_t* out_keep_idx,
                           void* out_importance, void* stream) {
  if (num_selected < 0) return NKV_ERR_INVALID_ARGUMENT;
  if (num_selected == 0) return NKV_OK;
  if (!ring || !ring_slot_of_selected || !k_cache || !v_cache || !block_tables || !context_lens ||
      !selected_batch_indices)
    return NKV_ERR_INVALID_ARGUMENT;
  if (num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads) return NKV_ERR_INVALID_ARGUMENT;
  if (head_dim != nkv::kCompressHeadDim || num_kv_heads > 8 || block_size <= 0) return NKV_ERR_UNSUPPORTED;
  // key slots are held as 32-bit ints
  if (num_blocks < 0 || num_blocks * static_cast<int64_t>(block_size) > INT32_MAX) return NKV_ERR_UNSUPPORTED;
  const int g = num_q_heads / num_kv_heads;
  const int W = window_size;
  const int num_keep = compress_R - W - 1;
  if (W <= 0 || compress_S - W <= 0 || compress_S <= num_keep + W || num_keep < 0)
    return NKV_ERR_INVALID_ARGUMENT;
  if (!aligned16(ring) || !aligned16(k_cache) || !aligned16(v_cache)) return NKV_ERR_ALIGNMENT;
  nkv::ThresholdCompressParams p{};
  p.ring = static_cast<const __nv_bfloat16*>(ring);
  p.ring_slot_of_selected = ring_slot_of_selected;
  p.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  p.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  p.num_blocks = num_blocks;
  p.block_tables = block_tables;
  p.context_lens = context_lens;
  p.selected = selected_batch_indices;
  p.out_keep_idx = out_keep_idx;
  p.out_importance = static_cast<uint16_t*>(out_importance);
  p.scale = softmax_scale;
  p.num_ring_slots = num_ring_slots;
  p.num_layers = num_layers;
  p.window = W;
  p.layer_id = layer_id;
  p.max_blocks = max_blocks;
  p.S = compress_S;
  p.R = compress_R;
  p.num_q_heads = num_q_heads;
  p.num_kv_heads = num_kv_heads;
  p.g = g;
  p.block_size = block_size;
  p.num_keys = compress_S - W;
  p.keys_pad = ((p.num_keys + nkv::kThrKeyTile - 1) / nkv::kThrKeyTile) * nkv::kThrKeyTile;
  p.rows = g * W;
  p.mtiles = (p.rows + 15) / 16;
  const int G = padded_group(g);
  if (G == 0) return NKV_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // halves CTAs per kv head, each scoring one range of the keys
  auto run = [&](int halves) -> int {
    p.halves = halves;
    const int per = (p.num_keys + halves - 1) / halves;
    p.keys_half = ((per + nkv::kThrKeyTile - 1) / nkv::kThrKeyTile) * nkv::kThrKeyTile;
    // As many 16-row m-tiles per row group as shared memory (and two warps
    // per m-tile) allow; more groups re-stream the keys from L2.
    int gm = std::min(p.mtiles, nkv::kThrWarps / 2);
    while (gm > 0 && nkv::threshold_smem_bytes(G, p.keys_pad, p.keys_half, gm, p.rows,
                                                compress_R) > kMaxSmem)
      --gm;
    if (gm == 0) return NKV_ERR_UNSUPPORTED;
    p.group_mtiles = gm;
    const size_t smem =
        nkv::threshold_smem_bytes(G, p.keys_pad, p.keys_half, gm, p.rows, compress_R);
    const int cx = num_kv_heads * halves;
    switch (G) {
      case 1: return launch_threshold<1>(p, cx, num_selected, smem, s);
      case 2: return launch_threshold<2>(p, cx, num_selected, smem, s);
      case 4: return launch_threshold<4>(p, cx, num_selected, smem, s);
      case 8: return launch_threshold<8>(p, cx, num_selected, smem, s);
      default: return launch_threshold<16>(p, cx, num_selected, smem, s);
    }
  };
  // Two CTAs per kv head (a 16-CTA cluster at 8 kv heads) halve each CTA's
  // scoring, row statistics, window sums and compaction; where that cluster
  // does not fit, one CTA per kv head.
  int st = kThresholdNoFit;
  if (num_kv_heads * 2 <= 16 && p.num_keys >= 2 * nkv::kThrKeyTile) st = run(2);
  if (st == kThresholdNoFit || st == NKV_ERR_UNSUPPORTED) st = run(1);
  return st == kThresholdNoFit ? NKV_ERR_UNSUPPORTED : st;
}

}  // extern "C"

// ------------------------------------------------------------------ static scratch
// Paged decode for callers that cannot allocate device memory (nkv.h,
// section 4). Its scratch is this fixed array in the library's device image:
// every GPU that loads the library holds NKV_STATIC_SCRATCH_BYTES of it until
// the process exits. In host code the name below is only a stand-in symbol,
// not a device address; the address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_static_decode_scratch[NKV_STATIC_SCRATCH_BYTES];

namespace {

void* g_static_scratch_addr[kMaxDevices] = {nullptr};
std::mutex g_static_scratch_mutex;

// Device address of g_static_decode_scratch on the current device, looked up
// once per device with that device current (the first call may load the
// module, so it belongs outside stream capture).
int static_scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev < 0 || dev >= kMaxDevices) return NKV_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_static_scratch_mutex);
  if (g_static_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_decode_scratch);
    if (e != cudaSuccess) return cuda_status(e);
    g_static_scratch_addr[dev] = p;
  }
  *out = g_static_scratch_addr[dev];
  return NKV_OK;
}

}  // namespace

extern "C" int nkv_paged_decode_static_scratch(
    const void* q, int64_t q_stride_token, int64_t q_stride_head, const void* k_cache,
    const void* v_cache, int64_t num_blocks, const int32_t* block_tables, int32_t max_blocks,
    const int32_t* context_lens, void* out, int64_t out_stride_token, int32_t batch,
    int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
    float softmax_scale, void* stream) {
  // Argument validation of nkv_paged_decode: without a workspace it stops at
  // NKV_ERR_WORKSPACE exactly when every other check passed (nothing launched).
  const int pre = nkv_paged_decode(q, q_stride_token, q_stride_head, k_cache, v_cache, num_blocks,
                                   block_tables, max_blocks, context_lens, out, out_stride_token,
                                   batch, num_q_heads, num_kv_heads, head_dim, block_size,
                                   softmax_scale, nullptr, 0, stream);
  if (pre != NKV_ERR_WORKSPACE) return pre;  // an argument error, or batch == 0 (no-op)
  const DecodePlan pl = make_decode_plan(batch, num_q_heads, num_kv_heads, max_blocks, block_size);
  if (pl.total > NKV_STATIC_SCRATCH_BYTES) return NKV_ERR_WORKSPACE;
  void* scratch = nullptr;
  const int st = static_scratch_address(&scratch);
  if (st != NKV_OK) return st;
  // The array keeps the previous call's bytes: zero the scheduler and split
  // counters this call uses (partial results need no clearing).
  const size_t counter_bytes = pl.off_split_counters + sizeof(unsigned int) * pl.pairs;
  cudaError_t e = cudaMemsetAsync(scratch, 0, counter_bytes, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_status(e);
  return nkv_paged_decode(q, q_stride_token, q_stride_head, k_cache, v_cache, num_blocks,
                          block_tables, max_blocks, context_lens, out, out_stride_token, batch,
                          num_q_heads, num_kv_heads, head_dim, block_size, softmax_scale, scratch,
                          NKV_STATIC_SCRATCH_BYTES, stream);
}
