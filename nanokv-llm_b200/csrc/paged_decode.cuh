// Paged split-KV decode attention for sm_100a: the B200 replacement for
// flash_attn_with_kvcache(q.unsqueeze(1), k_cache, v_cache, cache_seqlens,
// block_table, softmax_scale, causal=True) at nanokvllm/layers/attention.py:104-107.
//
// Design (HBM-bound: every K/V byte is read exactly once per step):
//   * Work item = (split s, batch row b, kv head h): up to `chunk` tokens of
//     one sequence for one kv head and ALL g = Hq/Hk query heads of that group
//     (GQA grouping: a K/V tile is read once for the whole group).
//   * Persistent CTAs (one per SM), three warp roles:
//       - warp 4, the producer: a CTA's first item is fixed by its block
//         index, later ones come from a global atomic counter (dynamic load
//         balance over the ragged context lengths). Per item one round of
//         loads spread over the lanes (length, slot, ring indices, 32
//         block-table entries, the fused step's new rows); then 128-token K
//         and V tiles stream with cp.async.bulk.tensor (TMA, 128B swizzle, L2
//         evict_first, no multicast) into a 3-stage shared-memory ring
//         guarded by full/empty mbarriers; the item's query rows ride in its
//         first tile's transaction. The fused step's new K/V row goes to the
//         cache and into the shared-memory copy of the tile that holds it
//         once that tile has landed;
//       - warps 0-3, the consumers: each owns 32 tokens of every tile and
//         keeps a warp-private online softmax (exp2 domain). For group widths
//         up to 8 they compute S^T = K Q^T and O^T = V^T P^T with mma.sync
//         m16n8k16 (tokens / dims on M, the heads on N), width 16 keeps Q on
//         M. At the end of an item they only dump their raw (m, l, O) into a
//         hand-off slot and go on with the next item;
//       - warp 5, the merger: takes a slot, merges the four warp states in a
//         fixed order (deterministic), and writes the bf16 output -- or, for
//         a split row, the fp32 partial plus an acq_rel arrival on the row's
//         counter; the last split to arrive merges all partials and writes
//         the output, then resets the counter.
//     The merge, the global writes and the cross-CTA hand-off therefore never
//     stall the tensor-core warps or the TMA ring.
//   * Small launches (few (row, kv head) pairs) are launched as thread-block
//     clusters, one per pair, CTA r taking split r; the splits' partials go
//     to the cluster leader's shared memory with st.async and merge there.
//   * Programmatic dependent launch: the next kernel may start while this one
//     drains; each role waits (griddepcontrol.wait) before its first access
//     to data the previous kernel may write. With metadata_ready the producer
//     reads its first item's metadata and requests its first K/V tile before
//     that wait, and only the tile's q rows after it.
//   * The work counter is reset by the last CTA to finish, so the workspace
//     counters are back at zero after every call (graph-replay safe).
//   * Tokens past context_lens in the last tile are masked in S (select, not
//     arithmetic) and their V rows are zeroed in registers, so uninitialised
//     cache memory (NaN patterns) never reaches the output.
//
// Tensor cores: the group width g (2..8 for Qwen3) is too narrow for tcgen05's
// M >= 64 tiles without wasting >= 87% of each instruction, and the kernel is
// bandwidth-bound by ~60x, so the warp-level mma.sync path keeps ALU work off
// the critical path while TMA does the address generation for the gathers.
#pragma once
#include "nkv_common.cuh"

namespace nkv {

constexpr int kDecodeHeadDim = 128;
constexpr int kDecodeTileTokens = 128;       // tokens per pipeline stage
constexpr int kDecodeConsumerWarps = 4;
constexpr int kDecodeProducerWarp = kDecodeConsumerWarps;
constexpr int kDecodeMergerWarp = kDecodeConsumerWarps + 1;
constexpr int kDecodeThreads = (kDecodeConsumerWarps + 2) * 32;
constexpr int kHalfTileBytes = kDecodeTileTokens * 128;  // 128 rows x 64 dims x 2 B
constexpr int kDecodeMetaInts = 8;
// A split's (O, m, l) of one q row as the cluster leader receives it:
// O[128], m, l, 2 floats of padding (16-byte aligned rows).
constexpr int kRecvRowFloats = kDecodeHeadDim + 4;
// Largest cluster of splits (portable cluster size).
constexpr int kDecodeMaxClusterSplits = 8;

template <int G>
struct DecodeShape {
  static_assert(G == 1 || G == 2 || G == 4 || G == 8 || G == 16, "padded group width");
  static constexpr int kStages = (G <= 8) ? 3 : 2;
  static constexpr int kQRows = (G < 8) ? 8 : G;
  static constexpr int kQHalfBytes = ((kQRows * 128 + 1023) / 1024) * 1024;
  static constexpr int kStageBytes = 4 * kHalfTileBytes + 2 * kQHalfBytes;
  // hand-off slots between consumers and merger
  static constexpr int kSlots = (G <= 4) ? 2 : 1;
  static constexpr int kORowStride = kDecodeHeadDim + 4;  // floats; 16-byte aligned rows
  static constexpr int kSlotOFloats = kDecodeConsumerWarps * G * kORowStride;
  static constexpr int kSlotMLFloats = 2 * kDecodeConsumerWarps * G;
  static constexpr int kSlotBytes = (kSlotOFloats + kSlotMLFloats) * 4 + 16;
  // [stages][slots][barriers][meta][flags (16 B)][pad to 16][receive barrier (16 B)]
  // [receive rows: cluster launches only, kRecvRowFloats per (split, row)]
  // barriers: full, empty, patch (per stage), slot full, slot empty
  static constexpr int kRecvBarOffset = (kStages * kStageBytes + kSlots * kSlotBytes +
                                         (3 * kStages + 2 * kSlots) * 8 +
                                         kStages * kDecodeMetaInts * 4 + 16 + 15) / 16 * 16;
  static constexpr int kRecvOffset = kRecvBarOffset + 16;
  static constexpr int kSmemBytes = kRecvOffset + 1024 /* alignment */;
  // A cluster launch of C splits adds C * G receive rows.
  static constexpr int kRecvBytesPerSplit = G * kRecvRowFloats * 4;
};

struct DecodeParams {
  const int32_t* block_tables;
  const int32_t* context_lens;
  __nv_bfloat16* out;
  int64_t out_stride_token;
  int64_t num_blocks;
  unsigned int* counters;        // [0] work counter, [1] finished-CTA counter
  unsigned int* split_counters;  // [batch * num_kv_heads]
  float* part_o;                 // [pairs, max_splits, g, 128]
  float* part_ml;                // [pairs, max_splits, g, 2]
  float scale_log2;
  int max_blocks;
  int batch;
  int num_kv_heads;
  int g;
  int block_size;
  int chunk_tokens;
  int max_splits;
  int total_items;
  // > 1: launched as clusters of `cluster` CTAs, CTA r of cluster c taking
  // split r of (row, kv head) pair c and sending its partial to rank 0
  // through distributed shared memory (no global partials or counters).
  int cluster;
  // 1: block_tables, context_lens, slot_mapping, the ring indices and the
  // cached K/V rows (other than the step's new ones) are not written by the
  // kernel this launch depends on, so a CTA's first item's metadata and its
  // first K/V tile are requested before the dependency wait (the fused
  // decode step's contract, when its caller vouches for it).
  int metadata_ready;
  // Fused decode step (optional, null when unused): the step's new K/V rows,
  // written by the producer warp right before the TMA that reads them, and
  // the KvChat query-window ring append.
  const uint4* new_k;           // [batch] rows of num_kv_heads*128 bf16
  const uint4* new_v;
  int64_t new_k_stride_vec;     // row strides in 16-byte units
  int64_t new_v_stride_vec;
  const int32_t* slot_mapping;  // [batch]
  uint4* k_cache_vec;           // the caches as 16-byte units (for the write)
  uint4* v_cache_vec;
  const uint4* q_vec;           // q rows for the ring append
  int64_t q_stride_token_vec;
  uint4* ring_vec;              // [slots, layers, W, Hq, 128] bf16, or null
  const int32_t* ring_slot_of_row;  // [batch], -1 = row not in a query window
  const int32_t* ring_pos_of_row;   // [batch]
  int64_t ring_layer_base_vec;      // offset of ring[0, layer_id] in 16-byte units
  int64_t ring_slot_stride_vec;     // ring[s] -> ring[s + 1]
  int ring_slots;
  int ring_window;
  int num_q_heads;
};

__device__ __forceinline__ void store_bf16x4(__nv_bfloat16* dst, float4 v) {
  uint2 u;
  u.x = pack_bf16x2(v.x, v.y);
  u.y = pack_bf16x2(v.z, v.w);
  *reinterpret_cast<uint2*>(dst) = u;
}

template <int G>
__global__ void __launch_bounds__(kDecodeThreads, 1)
paged_decode_kernel(const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v,
                    const __grid_constant__ CUtensorMap tm_q, const DecodeParams p) {
  using S = DecodeShape<G>;
  constexpr int kStages = S::kStages;
  constexpr int kSlots = S::kSlots;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* stage_mem = smem;
  uint8_t* slot_mem = smem + kStages * S::kStageBytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(slot_mem + kSlots * S::kSlotBytes);
  uint64_t* empty_bar = full_bar + kStages;
  uint64_t* patch_bar = empty_bar + kStages;  // TMA of a tile the producer patches
  uint64_t* slot_full = patch_bar + kStages;   // 128 consumer arrivals
  uint64_t* slot_empty = slot_full + kSlots;   // 1 merger arrival
  int* meta = reinterpret_cast<int*>(slot_empty + kSlots);
  volatile int* flags = meta + kStages * kDecodeMetaInts;  // [0] abort
  uint64_t* recv_bar = reinterpret_cast<uint64_t*>(smem + S::kRecvBarOffset);
  // cluster launches: the consumer warps' own merge (two phases, 128 arrivals)
  uint64_t* merge_bar = recv_bar + 1;
  float* recv = reinterpret_cast<float*>(smem + S::kRecvOffset);
  // Cluster split mode needs the launch's clusters; a launch that lost them
  // (%cluster_nctarank 1) merges its splits through global memory instead.
  const int csize = p.cluster;
  const bool cluster_mode = csize > 1 && static_cast<int>(cluster_nctarank()) == csize;

  auto slot_o = [&](int s) { return reinterpret_cast<float*>(slot_mem + s * S::kSlotBytes); };
  auto slot_m = [&](int s) { return slot_o(s) + S::kSlotOFloats; };
  auto slot_l = [&](int s) { return slot_m(s) + kDecodeConsumerWarps * G; };
  auto slot_hdr = [&](int s) {
    return reinterpret_cast<int*>(slot_l(s) + kDecodeConsumerWarps * G);  // [item, nsplit]
  };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), kDecodeConsumerWarps);
      mbar_init(smem_u32(&patch_bar[s]), 1);
    }
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(smem_u32(&slot_full[s]), kDecodeConsumerWarps * 32);
      mbar_init(smem_u32(&slot_empty[s]), 1);
    }
    // the leader's receive barrier: its own arrival (with the expected
    // bytes) plus the splits' asynchronous stores
    if (cluster_mode) {
      mbar_init(smem_u32(recv_bar), 1);
      mbar_init(smem_u32(merge_bar), kDecodeConsumerWarps * 32);
    }
    flags[0] = 0;
    fence_barrier_init();
  }
  if (warp == kDecodeProducerWarp && lane == 0) {
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
    prefetch_tmap(&tm_q);
  }
  __syncthreads();
  // No CTA stores to the leader's receive rows before its barrier exists.
  if (cluster_mode) cluster_sync_all();
  // Launched with programmatic stream serialisation: everything above
  // overlapped the previous kernel (typically the previous layer's decode);
  // after each role's grid_dependency_wait its writes (q / k / v rows, cache
  // rows, the reset workspace counters) are visible. The producer allows the
  // next kernel of the stream (the next layer's decode) to be scheduled right
  // after its own wait: those CTAs take free SMs, run their set-up (and, with
  // metadata_ready, their first metadata loads and first K/V tile) and wait
  // until this grid has finished, which hides a launch's latency in a chain
  // of small launches.

  const int Hk = p.num_kv_heads;
  const int g = p.g;
  const float NEG_INF = -INFINITY;

  if (warp == kDecodeProducerWarp) {
    // ------------------------------------------------------------ producer
    // The whole warp walks the loop; lane 0 grabs items and issues the TMA,
    // all lanes share the fused step's row copies.
    const bool leader = lane == 0;
    const uint64_t pol_stream = l2_policy_evict_first();
    const uint64_t pol_q = l2_policy_evict_last();
    const uint32_t q_bytes = static_cast<uint32_t>(2 * g * 128);
    const int row_vecs = Hk * (kDecodeHeadDim / 8);  // 16-byte units of one cache row
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    // armed[s] = parity + 1 of the last TMA transaction issued into stage s
    // that the producer has not yet seen released (0 = none outstanding).
    uint32_t armed[kStages];
#pragma unroll
    for (int s = 0; s < kStages; ++s) armed[s] = 0;
    // Items are grabbed one at a time, only when the ring has room for their
    // first tile: claiming the next item early lets a busy CTA hold work an
    // idle one could have taken, which lengthens the tail (measured slower).
    // A CTA's first item is fixed by its block index; later ones come from
    // the counter (offset by the grid size).
    // In a split-cluster launch CTA r of cluster c takes split r of pair c.
    int static_item = static_cast<int>(blockIdx.x);
    if (csize > 1)
      static_item = static_cast<int>(blockIdx.x) % csize * (Hk * p.batch) +
                    static_cast<int>(blockIdx.x) / csize;
    constexpr int kHeadVecs = kDecodeHeadDim / 8;  // 16-byte units of one head row
    // An item's metadata in one round, spread over the lanes: its length,
    // slot-mapping entry and query-window slot / position (lanes 0-3) and 32
    // block-table entries from its split's first block (one per lane).
    auto meta_loads = [&](int it, int& scalar, int& bt) {
      const int rest_ = it / Hk;
      const int b_ = rest_ % p.batch;
      const int s_ = rest_ / p.batch;
      scalar = 0;
      if (lane == 0) {
        scalar = ldg_nc_s32(p.context_lens + b_);
      } else if (lane == 1) {
        scalar = p.new_k != nullptr ? ldg_nc_s32(p.slot_mapping + b_) : -1;
      } else if (lane == 2 || lane == 3) {
        if (p.ring_vec != nullptr && s_ == 0)
          scalar = ldg_nc_s32((lane == 2 ? p.ring_slot_of_row : p.ring_pos_of_row) + b_);
      }
      const int blk0 = s_ * p.chunk_tokens / p.block_size;
      bt = -1;
      if (blk0 + lane < p.max_blocks)
        bt = ldg_nc_s32(p.block_tables + static_cast<int64_t>(b_) * p.max_blocks + blk0 + lane);
    };
    // Everything about an item that follows from its metadata (no data of
    // the kernel this launch depends on): computed before the dependency
    // wait for a CTA's first item when metadata_ready.
    struct ItemPlan {
      int item, kvh, b, s, t0, blk_first, bt_ent;
      int len, nsplit, t1, ntiles;
      int slot_new, ring_slot, ring_pos;
      int patch_row;  // >= 0: the new token's row inside the item's last tile
      int tile0_slot; // first slot of the item's first tile (or the zero-fill coordinate)
      bool skip;      // no such split
    };
    // Block index of the cache block holding token position `tok` of the row.
    auto block_of = [&](const ItemPlan& P, int tok) -> int {
      const int bi = tok / p.block_size - P.blk_first;
      int blk = __shfl_sync(0xffffffffu, P.bt_ent, bi & 31);
      if (bi >= 32)
        blk = __ldg(p.block_tables + static_cast<int64_t>(P.b) * p.max_blocks + tok / p.block_size);
      return blk;
    };
    // Slot of the tile starting at `tok` (fully out of range: TMA fills zeros).
    auto tile_slot = [&](const ItemPlan& P, int tok) -> int {
      const int blk = block_of(P, tok);
      const bool blk_ok = blk >= 0 && static_cast<int64_t>(blk) < p.num_blocks;
      if (!blk_ok && leader) raise_error(NKV_DEVERR_DECODE_BLOCK);
      return blk_ok ? blk * p.block_size + (tok % p.block_size) : -2 * kDecodeTileTokens;
    };
    auto make_plan = [&](int it, int scalar, int bt) -> ItemPlan {
      ItemPlan P;
      P.item = it;
      P.kvh = it % Hk;
      const int rest = it / Hk;
      P.b = rest % p.batch;
      P.s = rest / p.batch;
      P.t0 = P.s * p.chunk_tokens;
      P.blk_first = P.t0 / p.block_size;
      P.bt_ent = bt;
      int len = __shfl_sync(0xffffffffu, scalar, 0);
      // a length past the row's block table is clamped (and flagged) so that
      // no block-table read leaves the row
      if (len > p.max_blocks * p.block_size) {
        if (leader) raise_error(NKV_DEVERR_DECODE_BLOCK);
        len = p.max_blocks * p.block_size;
      }
      P.len = len;
      P.slot_new = __shfl_sync(0xffffffffu, scalar, 1);
      P.ring_slot = __shfl_sync(0xffffffffu, scalar, 2);
      P.ring_pos = __shfl_sync(0xffffffffu, scalar, 3);
      P.nsplit = len > 0 ? (len + p.chunk_tokens - 1) / p.chunk_tokens : 1;
      P.skip = P.s >= P.nsplit;
      P.t1 = min(P.t0 + p.chunk_tokens, len);
      P.ntiles = (len > 0 && !P.skip) ? (P.t1 - P.t0 + kDecodeTileTokens - 1) / kDecodeTileTokens : 0;
      // Fused slot write: the current token (position len - 1) lives in the
      // last split's last tile. Its K/V head slice goes to the cache and,
      // so that the tile's load need not wait for that write, into the
      // tile's shared-memory copy once the TMA has landed.
      P.patch_row = -1;
      if (p.new_k != nullptr && !P.skip && P.s == P.nsplit - 1 && P.ntiles > 0) {
        const int blk = block_of(P, len - 1);
        const bool blk_ok = blk >= 0 && static_cast<int64_t>(blk) < p.num_blocks;
        const int64_t want =
            blk_ok ? static_cast<int64_t>(blk) * p.block_size + (len - 1) % p.block_size : -1;
        if (P.slot_new >= 0 && P.slot_new == want) {
          P.patch_row = (len - 1) - (P.t0 + (P.ntiles - 1) * kDecodeTileTokens);
        } else if (P.slot_new != -1 && leader) {
          raise_error(NKV_DEVERR_STORE_SLOT);
        }
      }
      P.tile0_slot = P.ntiles > 0 ? tile_slot(P, P.t0) : 0;
      return P;
    };
    // With metadata_ready the first item's metadata is requested and planned
    // before the dependency wait: the kernel this launch depends on does not
    // write it (the contract of metadata_ready). In a launch with one item
    // per CTA (the latency-bound small batches) the item's first K/V tile is
    // requested then too -- that kernel writes no cache row this launch reads,
    // and the step's own new row is patched into the tile's shared-memory
    // copy after the wait -- and only the tile's q rows, which that kernel
    // may have written, after the wait, first thing. In larger launches,
    // whose previous kernel is still streaming at full bandwidth, the tile
    // is only hinted into L2 (demand loads there slowed that kernel's tail).
    const bool early = p.metadata_ready != 0 && static_item < p.total_items;
    ItemPlan pre;
    bool pre_tile = false;  // the first item's first tile is in flight (all but q)
    uint32_t pre_tb = 0;    // the barrier its transaction completes on
    if (early) {
      int sc0, bt0;
      meta_loads(static_item, sc0, bt0);
      pre = make_plan(static_item, sc0, bt0);
      if (p.total_items > static_cast<int>(gridDim.x)) {
        if (leader && pre.ntiles > 0 && pre.tile0_slot >= 0) {
          tma_prefetch_l2_3d(&tm_k, 0, pre.kvh, pre.tile0_slot);
          tma_prefetch_l2_3d(&tm_k, 64, pre.kvh, pre.tile0_slot);
          tma_prefetch_l2_3d(&tm_v, 0, pre.kvh, pre.tile0_slot);
          tma_prefetch_l2_3d(&tm_v, 64, pre.kvh, pre.tile0_slot);
        }
      } else if (!pre.skip && pre.ntiles > 0) {
        // stage 0, phase 0: free; the tile is the item's last when ntiles == 1
        pre_tb = smem_u32(pre.patch_row >= 0 && pre.ntiles == 1 ? &patch_bar[0] : &full_bar[0]);
        if (leader) {
          int* m = meta;
          m[0] = pre.item;
          m[1] = 0;
          m[2] = pre.ntiles;
          m[3] = min(kDecodeTileTokens, pre.t1 - pre.t0);
          m[4] = pre.nsplit;
          mbar_arrive_expect_tx(pre_tb, 4u * kHalfTileBytes + q_bytes);
          const uint32_t base = smem_u32(stage_mem);
          tma_load_3d(base + 0 * kHalfTileBytes, &tm_k, pre_tb, 0, pre.kvh, pre.tile0_slot, pol_stream);
          tma_load_3d(base + 1 * kHalfTileBytes, &tm_k, pre_tb, 64, pre.kvh, pre.tile0_slot, pol_stream);
          tma_load_3d(base + 2 * kHalfTileBytes, &tm_v, pre_tb, 0, pre.kvh, pre.tile0_slot, pol_stream);
          tma_load_3d(base + 3 * kHalfTileBytes, &tm_v, pre_tb, 64, pre.kvh, pre.tile0_slot, pol_stream);
        }
        pre_tile = true;
      }
    }
    grid_dependency_wait();
    if (pre_tile && leader) {
      const uint32_t qb = smem_u32(stage_mem) + 4 * kHalfTileBytes;
      tma_load_3d(qb, &tm_q, pre_tb, 0, pre.kvh * g, pre.b, pol_q);
      tma_load_3d(qb + S::kQHalfBytes, &tm_q, pre_tb, 64, pre.kvh * g, pre.b, pol_q);
    }
    allow_dependent_launch();
    bool first = true;
    // patch_armed[s] = parity + 1 of a patch-barrier transaction issued into
    // stage s and not yet waited for (only after an abort).
    uint32_t patch_armed[kStages];
    uint32_t patch_phase = 0;  // bit s: parity of stage s's next patch transaction
#pragma unroll
    for (int s = 0; s < kStages; ++s) patch_armed[s] = 0;
    while (ok) {
      int item = static_item;
      if (item < 0) {
        if (leader) item = static_cast<int>(gridDim.x + atomicAdd(&p.counters[0], 1u));
        item = __shfl_sync(0xffffffffu, item, 0);
      }
      static_item = -1;
      if (item >= p.total_items) break;
      ItemPlan P;
      const bool pre_first = first && pre_tile;  // its first tile is already requested
      if (first && early) {
        P = pre;
      } else {
        int sc, bt;
        meta_loads(item, sc, bt);
        P = make_plan(item, sc, bt);
      }
      first = false;
      if (P.skip) continue;
      // The data rows come from the kernel this launch depends on (after the
      // wait) and are needed only after the item's tiles are requested: the
      // new K/V head rows of the fused slot write (lanes 0-15 K, 16-31 V)
      // and the group's q rows for the KvChat query window.
      uint4 new_row = make_uint4(0u, 0u, 0u, 0u);
      if (P.patch_row >= 0) {
        const int64_t col = static_cast<int64_t>(P.kvh) * kHeadVecs + (lane & (kHeadVecs - 1));
        new_row = ldg_nc_v4(lane < kHeadVecs ? p.new_k + static_cast<int64_t>(P.b) * p.new_k_stride_vec + col
                                             : p.new_v + static_cast<int64_t>(P.b) * p.new_v_stride_vec + col);
      }
      constexpr int kQVecsPerLane = G >= 2 ? G / 2 : 1;
      const int q_vecs = g * kHeadVecs;  // the group's q rows
      const bool ring_append = p.ring_vec != nullptr && P.s == 0 && P.ring_slot >= 0;
      uint4 q_rows[kQVecsPerLane];
      if (ring_append) {
        const uint4* src = p.q_vec + static_cast<int64_t>(P.b) * p.q_stride_token_vec +
                           static_cast<int64_t>(P.kvh) * q_vecs;
#pragma unroll
        for (int i = 0; i < kQVecsPerLane; ++i)
          if (lane + 32 * i < q_vecs) q_rows[i] = ldg_nc_v4(src + lane + 32 * i);
      }
      const int kvh = P.kvh, b = P.b, t0 = P.t0, t1 = P.t1, ntiles = P.ntiles, nsplit = P.nsplit;
      // After a tile's loads are requested: the tile is armed, or -- the
      // item's last tile holding the step's new row -- the row goes to the
      // cache and into the tile's shared-memory copy once the TMA has landed,
      // and the producer releases the tile itself. false: the wait gave up.
      auto finish_tile = [&](bool patch, uint32_t fb) -> bool {
        if (!patch) {
          armed[stage] = phase + 1u;
          return true;
        }
        const uint32_t pp = (patch_phase >> stage) & 1u;
        patch_phase ^= 1u << stage;
        patch_armed[stage] = pp + 1u;
        // the new row to the cache (for later steps; nothing in this
        // launch reads that slot from global memory)
        {
          const int64_t col = static_cast<int64_t>(P.kvh) * kHeadVecs + (lane & (kHeadVecs - 1));
          uint4* gdst = lane < kHeadVecs ? p.k_cache_vec : p.v_cache_vec;
          gdst[static_cast<int64_t>(P.slot_new) * row_vecs + col] = new_row;
        }
        // every lane observes the transaction's completion before it
        // overwrites part of what the TMA wrote
        const bool landed = mbar_wait_bounded(smem_u32(&patch_bar[stage]), pp);
        if (!__all_sync(0xffffffffu, landed)) {
          if (leader) flags[0] = 1;
          return false;
        }
        patch_armed[stage] = 0;
        // lane u < 16: K dims [8u, 8u + 8) -> half u / 8, 16-byte chunk
        // u % 8 of the row's 128-byte swizzled line; lanes 16-31: V
        const int u = lane & (kHeadVecs - 1);
        uint8_t* dst = stage_mem + stage * S::kStageBytes +
                       ((lane < kHeadVecs ? 0 : 2) + (u >> 3)) * kHalfTileBytes +
                       swz128(static_cast<uint32_t>(P.patch_row), static_cast<uint32_t>(u & 7));
        *reinterpret_cast<uint4*>(dst) = new_row;
        __syncwarp();
        if (leader) mbar_arrive(fb);  // releases the tile (and the patch) to the consumers
        return true;
      };
      auto next_stage = [&]() {
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      };
      int j = 0;
      if (pre_first) {
        // the first tile was requested before the wait (ntiles > 0, stage 0)
        if (!finish_tile(P.patch_row >= 0 && ntiles == 1, smem_u32(&full_bar[stage]))) {
          ok = false;
          break;
        }
        next_stage();
        j = 1;
      }
      for (; j < ntiles || (j == 0 && ntiles == 0); ++j) {
        bool waited = true;
        if (leader) {
          waited = !flags[0] && mbar_wait_bounded(smem_u32(&empty_bar[stage]), phase ^ 1u);
          if (!waited) flags[0] = 1;
        }
        if (!__shfl_sync(0xffffffffu, waited ? 1 : 0, 0)) {
          ok = false;
          break;
        }
        armed[stage] = 0;
        const int tok = t0 + j * kDecodeTileTokens;
        if (leader) {
          int* m = meta + stage * kDecodeMetaInts;
          m[0] = item;
          m[1] = j;
          m[2] = ntiles;
          m[3] = ntiles > 0 ? min(kDecodeTileTokens, t1 - tok) : 0;
          m[4] = nsplit;
        }
        const uint32_t fb = smem_u32(&full_bar[stage]);
        if (ntiles == 0) {
          if (leader) mbar_arrive(fb);
        } else {
          const int slot = j == 0 ? P.tile0_slot : tile_slot(P, tok);
          const bool patch = P.patch_row >= 0 && j == ntiles - 1;
          // a patched tile's transaction completes on the patch barrier; the
          // producer releases the consumers itself after the patch
          const uint32_t tb = patch ? smem_u32(&patch_bar[stage]) : fb;
          const uint32_t base = smem_u32(stage_mem + stage * S::kStageBytes);
          if (leader) {
            const uint32_t bytes = 4u * kHalfTileBytes + (j == 0 ? q_bytes : 0u);
            mbar_arrive_expect_tx(tb, bytes);
            tma_load_3d(base + 0 * kHalfTileBytes, &tm_k, tb, 0, kvh, slot, pol_stream);
            tma_load_3d(base + 1 * kHalfTileBytes, &tm_k, tb, 64, kvh, slot, pol_stream);
            tma_load_3d(base + 2 * kHalfTileBytes, &tm_v, tb, 0, kvh, slot, pol_stream);
            tma_load_3d(base + 3 * kHalfTileBytes, &tm_v, tb, 64, kvh, slot, pol_stream);
            if (j == 0) {
              const uint32_t qb = base + 4 * kHalfTileBytes;
              tma_load_3d(qb, &tm_q, tb, 0, kvh * g, b, pol_q);
              tma_load_3d(qb + S::kQHalfBytes, &tm_q, tb, 64, kvh * g, b, pol_q);
            }
          }
          if (!finish_tile(patch, fb)) {
            ok = false;
            break;
          }
        }
        next_stage();
      }
      if (!ok) break;
      // KvChat: this step's query rows of the group join the row's window
      // (after the item's tiles are in flight: nothing in this launch reads them).
      if (ring_append) {
        if (P.ring_slot < p.ring_slots && P.ring_pos >= 0 && P.ring_pos < p.ring_window) {
          uint4* dst = p.ring_vec + p.ring_layer_base_vec + P.ring_slot * p.ring_slot_stride_vec +
                       static_cast<int64_t>(P.ring_pos) * p.num_q_heads * kHeadVecs +
                       static_cast<int64_t>(kvh) * q_vecs;
#pragma unroll
          for (int i = 0; i < kQVecsPerLane; ++i)
            if (lane + 32 * i < q_vecs) dst[lane + 32 * i] = q_rows[i];
        } else if (leader) {
          raise_error(NKV_DEVERR_RING_RANGE);
        }
      }
    }
    if (leader) {
      if (ok) {
        // End-of-work marker for the consumers.
        if (mbar_wait_bounded(smem_u32(&empty_bar[stage]), phase ^ 1u)) {
          armed[stage] = 0;  // released: its last transaction has completed
          meta[stage * kDecodeMetaInts + 0] = -1;
          mbar_arrive(smem_u32(&full_bar[stage]));
        } else {
          flags[0] = 1;
        }
      }
      // Drain: never leave the CTA with a bulk copy still writing its shared
      // memory (only matters after an abort; normally these return at once).
#pragma unroll
      for (int s = 0; s < kStages; ++s) {
        if (armed[s]) mbar_wait_bounded(smem_u32(&full_bar[s]), armed[s] - 1u);
        if (patch_armed[s]) mbar_wait_bounded(smem_u32(&patch_bar[s]), patch_armed[s] - 1u);
      }
      // The last CTA out resets the scheduler counters for the next call.
      __threadfence();
      const unsigned int prev = atomicAdd(&p.counters[1], 1u);
      if (prev == gridDim.x - 1) {
        atomicExch(&p.counters[0], 0u);
        atomicExch(&p.counters[1], 0u);
      }
    }
    return;
  }

  if (warp == kDecodeMergerWarp) {
    // -------------------------------------------------------------- merger
    grid_dependency_wait();  // before any global write (out, partials, counters)
    int slot = 0;
    uint32_t sphase = 0;
    const int d0 = 4 * lane;  // this lane's 4 dims
    while (true) {
      if (!mbar_wait_bounded(smem_u32(&slot_full[slot]), sphase)) {
        flags[0] = 1;
        break;
      }
      const int* hdr = slot_hdr(slot);
      const int item = hdr[0];
      if (item < 0) break;
      const int nsplit = hdr[1];
      const int kvh = item % Hk;
      const int rest = item / Hk;
      const int b = rest % p.batch;
      const int s = rest / p.batch;
      const int pair = b * Hk + kvh;
      const float* so = slot_o(slot);
      const float* sm = slot_m(slot);
      const float* sl = slot_l(slot);
      for (int row = 0; row < g; ++row) {
        float M = NEG_INF;
#pragma unroll
        for (int w = 0; w < kDecodeConsumerWarps; ++w) M = fmaxf(M, sm[w * G + row]);
        float L = 0.f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < kDecodeConsumerWarps; ++w) {
          const float mw = sm[w * G + row];
          const float f = (mw == NEG_INF) ? 0.f : fast_exp2(mw - M);
          L += sl[w * G + row] * f;
          const float4 ow =
              *reinterpret_cast<const float4*>(so + (w * G + row) * S::kORowStride + d0);
          acc.x += ow.x * f;
          acc.y += ow.y * f;
          acc.z += ow.z * f;
          acc.w += ow.w * f;
        }
        if (nsplit == 1) {
          const float inv = (L > 0.f) ? 1.f / L : 0.f;
          store_bf16x4(p.out + static_cast<int64_t>(b) * p.out_stride_token +
                           static_cast<int64_t>(kvh * g + row) * kDecodeHeadDim + d0,
                       make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv));
        } else {
          const int64_t pidx = (static_cast<int64_t>(pair) * p.max_splits + s) * g + row;
          *reinterpret_cast<float4*>(p.part_o + pidx * kDecodeHeadDim + d0) = acc;
          if (lane == 0) {
            *reinterpret_cast<float2*>(p.part_ml + pidx * 2) = make_float2(M, L);
          }
        }
      }
      // The slot's contents are consumed: hand it back before the global
      // hand-off so the consumers never wait on the split protocol.
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&slot_empty[slot]));
      if (nsplit > 1) {
        // __syncwarp orders the lanes' partial stores before lane 0's
        // gpu-scope release; the acquire half of the same atomic makes the
        // other splits' partials visible to the last arriver (and, through
        // the next __syncwarp, to all its lanes).
        __syncwarp();
        int last = 0;
        if (lane == 0) {
          const unsigned int prev = atomic_add_acq_rel_gpu(&p.split_counters[pair], 1u);
          last = (prev == static_cast<unsigned int>(nsplit - 1)) ? 1 : 0;
          if (last) atomicExch(&p.split_counters[pair], 0u);
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        __syncwarp();
        if (last && G <= 8 && nsplit <= 32) {
          // All rows at once, in two rounds of loads: every row's (m, l) of
          // split `lane`, then this lane's 4 dims of the rows' partial O,
          // 16 loads in flight per batch (a loop of dependent loads costs an
          // L2 round trip each, and the last arriver's merge is on the
          // launch's tail). The sums run in split order; M and L are
          // reduced by fixed butterflies, so the result is deterministic.
          constexpr int kRows = G <= 8 ? G : 8;
          constexpr int kB = 16 / kRows;  // splits per batch
          const int64_t base0 = static_cast<int64_t>(pair) * p.max_splits * g;
          float f_r[kRows], inv_r[kRows];
          {
            float ms_r[kRows], l_r[kRows];
#pragma unroll
            for (int row = 0; row < kRows; ++row) {
              ms_r[row] = NEG_INF;
              l_r[row] = 0.f;
              if (row < g && lane < nsplit) {
                const float2 ml = __ldcg(reinterpret_cast<const float2*>(
                    p.part_ml + (base0 + row + static_cast<int64_t>(lane) * g) * 2));
                ms_r[row] = ml.x;
                l_r[row] = ml.y;
              }
            }
#pragma unroll
            for (int row = 0; row < kRows; ++row) {
              float M = ms_r[row];
#pragma unroll
              for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
              const float f = (ms_r[row] != NEG_INF) ? fast_exp2(ms_r[row] - M) : 0.f;
              float lf = l_r[row] * f;
#pragma unroll
              for (int o = 16; o > 0; o >>= 1) lf += __shfl_xor_sync(0xffffffffu, lf, o);
              f_r[row] = f;
              inv_r[row] = (lf > 0.f) ? 1.f / lf : 0.f;
            }
          }
          float4 acc[kRows];
#pragma unroll
          for (int row = 0; row < kRows; ++row) acc[row] = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int k0 = 0; k0 < nsplit; k0 += kB) {
            float4 po[kRows][kB];
#pragma unroll
            for (int row = 0; row < kRows; ++row) {
#pragma unroll
              for (int u = 0; u < kB; ++u) {
                po[row][u] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (row < g && k0 + u < nsplit)
                  po[row][u] = __ldcg(reinterpret_cast<const float4*>(
                      p.part_o + (base0 + row + static_cast<int64_t>(k0 + u) * g) * kDecodeHeadDim +
                      d0));
              }
            }
#pragma unroll
            for (int row = 0; row < kRows; ++row) {
#pragma unroll
              for (int u = 0; u < kB; ++u) {
                const float fu = __shfl_sync(0xffffffffu, f_r[row], (k0 + u) & 31);
                if (k0 + u < nsplit) {
                  acc[row].x += po[row][u].x * fu;
                  acc[row].y += po[row][u].y * fu;
                  acc[row].z += po[row][u].z * fu;
                  acc[row].w += po[row][u].w * fu;
                }
              }
            }
          }
#pragma unroll
          for (int row = 0; row < kRows; ++row) {
            if (row < g) {
              const float inv = inv_r[row];
              store_bf16x4(p.out + static_cast<int64_t>(b) * p.out_stride_token +
                               static_cast<int64_t>(kvh * g + row) * kDecodeHeadDim + d0,
                           make_float4(acc[row].x * inv, acc[row].y * inv, acc[row].z * inv,
                                       acc[row].w * inv));
            }
          }
        } else if (last) {
          // Any group width and split count: two rounds of loads per row (the
          // splits' (m, l), one split per lane, then this lane's 4 dims of
          // every split's partial O, eight at a time), in split order.
          for (int row = 0; row < g; ++row) {
            const int64_t base = static_cast<int64_t>(pair) * p.max_splits * g + row;
            float ms0 = NEG_INF, l0 = 0.f;  // split `lane` (the first 32 splits)
            if (lane < nsplit) {
              const float2 ml = __ldcg(reinterpret_cast<const float2*>(
                  p.part_ml + (base + static_cast<int64_t>(lane) * g) * 2));
              ms0 = ml.x;
              l0 = ml.y;
            }
            float M = ms0;
            for (int c = 32; c < nsplit; c += 32)
              if (c + lane < nsplit)
                M = fmaxf(M, __ldcg(p.part_ml + (base + static_cast<int64_t>(c + lane) * g) * 2));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
            float L = 0.f;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int c = 0; c < nsplit; c += 32) {
              const int cnt = min(32, nsplit - c);
              float ms = ms0, lw = l0;
              if (c > 0) {
                ms = NEG_INF;
                lw = 0.f;
                if (lane < cnt) {
                  const float2 ml = __ldcg(reinterpret_cast<const float2*>(
                      p.part_ml + (base + static_cast<int64_t>(c + lane) * g) * 2));
                  ms = ml.x;
                  lw = ml.y;
                }
              }
              const float f = (lane < cnt && ms != NEG_INF) ? fast_exp2(ms - M) : 0.f;
              float lf = lw * f;
#pragma unroll
              for (int o = 16; o > 0; o >>= 1) lf += __shfl_xor_sync(0xffffffffu, lf, o);
              L += lf;
              for (int k0 = 0; k0 < cnt; k0 += 8) {
                float4 po[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                  po[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                  if (k0 + u < cnt)
                    po[u] = __ldcg(reinterpret_cast<const float4*>(
                        p.part_o + (base + static_cast<int64_t>(c + k0 + u) * g) * kDecodeHeadDim + d0));
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                  const float fu = __shfl_sync(0xffffffffu, f, (k0 + u) & 31);
                  if (k0 + u < cnt) {
                    acc.x += po[u].x * fu;
                    acc.y += po[u].y * fu;
                    acc.z += po[u].z * fu;
                    acc.w += po[u].w * fu;
                  }
                }
              }
            }
            const float inv = (L > 0.f) ? 1.f / L : 0.f;
            store_bf16x4(p.out + static_cast<int64_t>(b) * p.out_stride_token +
                             static_cast<int64_t>(kvh * g + row) * kDecodeHeadDim + d0,
                         make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv));
          }
        }
      }
      if (++slot == kSlots) {
        slot = 0;
        sphase ^= 1u;
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  grid_dependency_wait();
  const int cw = warp;
  const int gid = lane >> 2;
  const int tig = lane & 3;
  const float scale_log2 = p.scale_log2;

  // Group widths up to 8 compute the transposed products, S^T = K Q^T and
  // O^T = V^T P^T: the tokens (or dims) fill the 16 rows of each mma.sync
  // tile and the g heads its 8 columns, so a 2- to 8-head group costs half
  // the tensor-core instructions of the Q-on-rows form (whose 16 rows would
  // carry g heads). P^T reaches the B operand through movmatrix.
  constexpr bool kSwapAB = G <= 8;
  float o[16][4];
  float m_run[2], l_run[2];  // swap form: heads 2 tig + e; else rows gid (+ 8)
  uint32_t qa[8][4];

  int stage = 0;
  uint32_t phase = 0;
  int cslot = 0;
  uint32_t cphase = 0;
  // Hands the warp states of one item (or the end marker, item < 0) to the
  // merger through the next slot.
  // This warp's raw (m, l, O) rows into hand-off slot `sl`.
  auto write_state = [&](int sl) {
    if (kSwapAB) {
      // o[dm][c]: O^T rows dims 16 dm + gid (c 0, 1) and + 8 (c 2, 3),
      // columns heads 2 tig (c even) and 2 tig + 1 (c odd)
      float* so = slot_o(sl);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float l = l_run[e];
        l += __shfl_xor_sync(0xffffffffu, l, 4);
        l += __shfl_xor_sync(0xffffffffu, l, 8);
        l += __shfl_xor_sync(0xffffffffu, l, 16);
        const int h = 2 * tig + e;
        if (h < g) {
          if (gid == 0) {
            slot_m(sl)[cw * G + h] = m_run[e];
            slot_l(sl)[cw * G + h] = l;
          }
          float* dst = so + (cw * G + h) * S::kORowStride;
#pragma unroll
          for (int dm = 0; dm < 8; ++dm) {
            dst[16 * dm + gid] = o[dm][e];
            dst[16 * dm + 8 + gid] = o[dm][2 + e];
          }
        }
      }
    } else {
      constexpr int kRowSets = (G == 16) ? 2 : 1;
      float* so = slot_o(sl);
#pragma unroll
      for (int rs = 0; rs < kRowSets; ++rs) {
        float l = l_run[rs];
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        l += __shfl_xor_sync(0xffffffffu, l, 2);
        const int row = gid + 8 * rs;
        if (row < g) {
          if (tig == 0) {
            slot_m(sl)[cw * G + row] = m_run[rs];
            slot_l(sl)[cw * G + row] = l;
          }
          float* dst = so + (cw * G + row) * S::kORowStride;
#pragma unroll
          for (int n = 0; n < 16; ++n)
            *reinterpret_cast<float2*>(dst + 8 * n + 2 * tig) =
                make_float2(o[n][2 * rs], o[n][2 * rs + 1]);
        }
      }
    }
  };
  auto handoff = [&](int item, int nsplit) -> bool {
    if (!mbar_wait_bounded(smem_u32(&slot_empty[cslot]), cphase ^ 1u)) {
      flags[0] = 1;
      return false;
    }
    if (item >= 0) write_state(cslot);
    if (threadIdx.x == 0) {
      slot_hdr(cslot)[0] = item;
      slot_hdr(cslot)[1] = nsplit;
    }
    mbar_arrive(smem_u32(&slot_full[cslot]));
    if (++cslot == kSlots) {
      cslot = 0;
      cphase ^= 1u;
    }
    return true;
  };

  while (true) {
    if (!mbar_wait_bounded(smem_u32(&full_bar[stage]), phase)) {
      flags[0] = 1;
      break;
    }
    const int* m = meta + stage * kDecodeMetaInts;
    const int item = m[0];
    if (item < 0) {
      handoff(-1, 0);  // end marker for the merger
      break;
    }
    const int j = m[1];
    const int ntiles = m[2];
    const int nvalid = m[3];
    const int nsplit = m[4];
    const uint8_t* sbase = stage_mem + stage * S::kStageBytes;

    if (j == 0) {
#pragma unroll
      for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
      m_run[0] = m_run[1] = NEG_INF;
      l_run[0] = l_run[1] = 0.f;
      if (ntiles > 0) {
        const uint8_t* q0 = sbase + 4 * kHalfTileBytes;
        const uint8_t* q1 = q0 + S::kQHalfBytes;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint8_t* qh = (kk < 4) ? q0 : q1;
          const uint32_t c = 2u * (kk & 3);
          uint32_t a0 = 0, a1 = 0, a2 = 0, a3 = 0;
          if (gid < g) {
            a0 = *reinterpret_cast<const uint32_t*>(qh + swz128(gid, c) + 4 * tig);
            a2 = *reinterpret_cast<const uint32_t*>(qh + swz128(gid, c + 1) + 4 * tig);
          }
          if (G == 16 && gid + 8 < g) {
            a1 = *reinterpret_cast<const uint32_t*>(qh + swz128(gid + 8, c) + 4 * tig);
            a3 = *reinterpret_cast<const uint32_t*>(qh + swz128(gid + 8, c + 1) + 4 * tig);
          }
          qa[kk][0] = a0;
          qa[kk][1] = a1;
          qa[kk][2] = a2;
          qa[kk][3] = a3;
        }
      }
    }

    const int tok_base = cw * 32;
    if (kSwapAB && ntiles > 0 && tok_base < nvalid) {
      const uint32_t sK0 = smem_u32(sbase);
      const uint32_t sK1 = sK0 + kHalfTileBytes;
      const uint32_t sV0 = sK0 + 2 * kHalfTileBytes;
      const uint32_t sV1 = sK0 + 3 * kHalfTileBytes;
      const int mi = lane >> 3;
      // S^T = K Q^T: two 16-token m-tiles x 8 head columns, 8 k-steps of 16 dims
      float sacc[2][4];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) sacc[mt][0] = sacc[mt][1] = sacc[mt][2] = sacc[mt][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t sK = (kk < 4) ? sK0 : sK1;
        const uint32_t c = 2u * (kk & 3) + static_cast<uint32_t>(mi >> 1);
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          const uint32_t r = tok_base + 16 * mt + (mi & 1) * 8 + (lane & 7);
          uint32_t a0, a1, a2, a3;
          ldsm_x4(sK + swz128(r, c), a0, a1, a2, a3);
          mma_bf16_16816(sacc[mt], a0, a1, a2, a3, qa[kk][0], qa[kk][2]);
        }
      }
      // online softmax per head (column 2 tig + e) over this warp's tokens
      const bool partial = (tok_base + 32 > nvalid);
      float mx[2] = {NEG_INF, NEG_INF};
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float v = sacc[mt][c] * scale_log2;
          const int tk = tok_base + 16 * mt + 8 * (c >> 1) + gid;
          if (partial && tk >= nvalid) v = NEG_INF;
          sacc[mt][c] = v;
          mx[c & 1] = fmaxf(mx[c & 1], v);
        }
      }
      float alpha[2], m_use[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 4));
        mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 8));
        mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 16));
        const float m_new = fmaxf(m_run[e], mx[e]);
        m_use[e] = (m_new == NEG_INF) ? 0.f : m_new;
        alpha[e] = fast_exp2(m_run[e] - m_use[e]);
        m_run[e] = m_new;
      }
      float rsum[2] = {0.f, 0.f};
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float pv = fast_exp2(sacc[mt][c] - m_use[c & 1]);
          sacc[mt][c] = pv;
          rsum[c & 1] += pv;
        }
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) l_run[e] = l_run[e] * alpha[e] + rsum[e];
#pragma unroll
      for (int dm = 0; dm < 8; ++dm) {
        o[dm][0] *= alpha[0];
        o[dm][1] *= alpha[1];
        o[dm][2] *= alpha[0];
        o[dm][3] *= alpha[1];
      }
      // O^T += V^T P^T: 8 m-tiles of 16 dims, two 16-token k-steps
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const uint32_t b0 = movmatrix_trans(pack_bf16x2(sacc[jj][0], sacc[jj][1]));
        const uint32_t b1 = movmatrix_trans(pack_bf16x2(sacc[jj][2], sacc[jj][3]));
        uint32_t mask_lo = 0xffffffffu, mask_hi = 0xffffffffu;
        if (partial) {
          const int ta = tok_base + 16 * jj + 2 * tig;
          mask_lo = (ta < nvalid ? 0x0000ffffu : 0u) | (ta + 1 < nvalid ? 0xffff0000u : 0u);
          mask_hi = (ta + 8 < nvalid ? 0x0000ffffu : 0u) | (ta + 9 < nvalid ? 0xffff0000u : 0u);
        }
        const uint32_t r = tok_base + 16 * jj + (mi & 1) * 8 + (lane & 7);
#pragma unroll
        for (int dm = 0; dm < 8; ++dm) {
          const uint32_t c16 = 2 * dm + (mi >> 1);
          const uint32_t addr = ((c16 < 8) ? sV0 : sV1) + swz128(r, c16 & 7u);
          uint32_t v0, v1, v2, v3;
          ldsm_x4_trans(addr, v0, v1, v2, v3);
          // v0 / v1: tokens 0-7 / 8-15 of dims 16 dm..+7; v2 / v3: dims +8
          v0 &= mask_lo;
          v2 &= mask_lo;
          v1 &= mask_hi;
          v3 &= mask_hi;
          mma_bf16_16816(o[dm], v0, v2, v1, v3, b0, b1);
        }
      }
    } else if (!kSwapAB && ntiles > 0 && tok_base < nvalid) {
      const uint32_t sK0 = smem_u32(sbase);
      const uint32_t sK1 = sK0 + kHalfTileBytes;
      const uint32_t sV0 = sK0 + 2 * kHalfTileBytes;
      const uint32_t sV1 = sK0 + 3 * kHalfTileBytes;
      float sacc[4][4];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.f;
      // S = Q K^T over this warp's 32 tokens.
#pragma unroll
      for (int kp = 0; kp < 4; ++kp) {
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          const uint32_t r = tok_base + nt * 8 + (lane & 7);
          const uint32_t c16 = kp * 4 + (lane >> 3);
          const uint32_t addr = ((c16 < 8) ? sK0 : sK1) + swz128(r, c16 & 7u);
          uint32_t b0, b1, b2, b3;
          ldsm_x4(addr, b0, b1, b2, b3);
          mma_bf16_16816(sacc[nt], qa[2 * kp][0], qa[2 * kp][1], qa[2 * kp][2], qa[2 * kp][3],
                         b0, b1);
          mma_bf16_16816(sacc[nt], qa[2 * kp + 1][0], qa[2 * kp + 1][1], qa[2 * kp + 1][2],
                         qa[2 * kp + 1][3], b2, b3);
        }
      }
      const bool partial = (tok_base + 32 > nvalid);
      // Online softmax, rows gid (and gid + 8 when G == 16).
      constexpr int kRowSets = (G == 16) ? 2 : 1;
      float pr[4][4];
#pragma unroll
      for (int rs = 0; rs < kRowSets; ++rs) {
        float mx = NEG_INF;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            float v = sacc[nt][2 * rs + e] * scale_log2;
            const int tk = tok_base + nt * 8 + 2 * tig + e;
            if (partial && tk >= nvalid) v = NEG_INF;
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
        for (int nt = 0; nt < 4; ++nt) {
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
          o[n][2 * rs + 0] *= alpha;
          o[n][2 * rs + 1] *= alpha;
        }
      }
      // O += P V over the warp's two 16-token k-steps.
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const uint32_t a0 = pack_bf16x2(pr[2 * jj][0], pr[2 * jj][1]);
        const uint32_t a2 = pack_bf16x2(pr[2 * jj + 1][0], pr[2 * jj + 1][1]);
        const uint32_t a1 = (G == 16) ? pack_bf16x2(pr[2 * jj][2], pr[2 * jj][3]) : 0u;
        const uint32_t a3 = (G == 16) ? pack_bf16x2(pr[2 * jj + 1][2], pr[2 * jj + 1][3]) : 0u;
        uint32_t mask_lo = 0xffffffffu, mask_hi = 0xffffffffu;
        if (partial) {
          const int ta = tok_base + 16 * jj + 2 * tig;
          mask_lo = (ta < nvalid ? 0x0000ffffu : 0u) | (ta + 1 < nvalid ? 0xffff0000u : 0u);
          mask_hi = (ta + 8 < nvalid ? 0x0000ffffu : 0u) | (ta + 9 < nvalid ? 0xffff0000u : 0u);
        }
        const int mi = lane >> 3;
        const uint32_t r = tok_base + 16 * jj + (mi & 1) * 8 + (lane & 7);
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
    }

    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&empty_bar[stage]));
    if (++stage == kStages) {
      stage = 0;
      phase ^= 1u;
    }

    if (j + 1 < ntiles) continue;
    if (cluster_mode) {
      // A cluster launch gives each CTA one item: the consumer warps merge
      // their own states (no hand-off to the merger warp, which here only
      // receives the end marker) and send the split's rows to the leader's
      // receive rows, or, in the leader, gather the splits and write the
      // output. Slot 0 holds the warp states (the end marker's hand-off
      // writes only its header).
      write_state(0);
      // all four warps' states in place (a bounded wait: a warp that gave
      // up earlier leaves the others to time out, not to hang)
      mbar_arrive(smem_u32(merge_bar));
      if (!mbar_wait_bounded(smem_u32(merge_bar), 0)) {
        flags[0] = 1;
        continue;
      }
      const int kvh = item % Hk;
      const int rest = item / Hk;
      const int b = rest % p.batch;
      const int s = rest / p.batch;
      const int d0 = 4 * lane;
      const float* so = slot_o(0);
      const float* smv = slot_m(0);
      const float* slv = slot_l(0);
      for (int row = cw; row < g; row += kDecodeConsumerWarps) {
        float M = NEG_INF;
#pragma unroll
        for (int w = 0; w < kDecodeConsumerWarps; ++w) M = fmaxf(M, smv[w * G + row]);
        float L = 0.f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < kDecodeConsumerWarps; ++w) {
          const float mw = smv[w * G + row];
          const float f = (mw == NEG_INF) ? 0.f : fast_exp2(mw - M);
          L += slv[w * G + row] * f;
          const float4 ow =
              *reinterpret_cast<const float4*>(so + (w * G + row) * S::kORowStride + d0);
          acc.x += ow.x * f;
          acc.y += ow.y * f;
          acc.z += ow.z * f;
          acc.w += ow.w * f;
        }
        if (nsplit == 1) {
          const float inv = (L > 0.f) ? 1.f / L : 0.f;
          store_bf16x4(p.out + static_cast<int64_t>(b) * p.out_stride_token +
                           static_cast<int64_t>(kvh * g + row) * kDecodeHeadDim + d0,
                       make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv));
        } else if (s == 0) {
          float* r = recv + row * kRecvRowFloats;  // the leader's own split
          *reinterpret_cast<float4*>(r + d0) = acc;
          if (lane == 0) *reinterpret_cast<float2*>(r + kDecodeHeadDim) = make_float2(M, L);
        } else {
          // into the leader's receive rows, counted on its receive barrier
          const uint32_t dst = mapa_shared(smem_u32(recv + (s * G + row) * kRecvRowFloats), 0);
          const uint32_t rbar = mapa_shared(smem_u32(recv_bar), 0);
          st_async_f32x4(dst + 4 * d0, acc, rbar);
          if (lane == 0) st_async_f32x2(dst + 4 * kDecodeHeadDim, M, L, rbar);
        }
      }
      if (nsplit > 1 && s == 0) {
        // The leader expects the other splits' rows (splits past the row's
        // end send nothing), waits for them to land, then merges the splits
        // in order.
        // its own rows are visible to all its warps
        mbar_arrive(smem_u32(merge_bar));
        if (!mbar_wait_bounded(smem_u32(merge_bar), 1)) {
          flags[0] = 1;
          continue;
        }
        if (threadIdx.x == 0)
          mbar_arrive_expect_tx(smem_u32(recv_bar),
                                static_cast<uint32_t>((nsplit - 1) * g * (4 * kDecodeHeadDim + 8)));
        if (mbar_wait_cluster_bounded(smem_u32(recv_bar), 0)) {
          for (int row = cw; row < g; row += kDecodeConsumerWarps) {
            float M = NEG_INF;
            for (int s2 = 0; s2 < nsplit; ++s2)
              M = fmaxf(M, recv[(s2 * G + row) * kRecvRowFloats + kDecodeHeadDim]);
            float L = 0.f;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int s2 = 0; s2 < nsplit; ++s2) {
              const float* r = recv + (s2 * G + row) * kRecvRowFloats;
              const float ms = r[kDecodeHeadDim];
              const float f = (ms == NEG_INF) ? 0.f : fast_exp2(ms - M);
              L += r[kDecodeHeadDim + 1] * f;
              const float4 po = *reinterpret_cast<const float4*>(r + d0);
              acc.x += po.x * f;
              acc.y += po.y * f;
              acc.z += po.z * f;
              acc.w += po.w * f;
            }
            const float inv = (L > 0.f) ? 1.f / L : 0.f;
            store_bf16x4(p.out + static_cast<int64_t>(b) * p.out_stride_token +
                             static_cast<int64_t>(kvh * g + row) * kDecodeHeadDim + d0,
                         make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv));
          }
        } else {
          flags[0] = 1;
        }
      }
      continue;
    }
    if (!handoff(item, nsplit)) break;
  }
  // Consumers leave only after the producer's end marker (or an abort), so
  // every TMA transaction they waited on has completed.
}

}  // namespace nkv
