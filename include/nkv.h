/*
 * nkv.h -- C ABI of the B200 (sm_100a) attention hot path for nano-kvllm.
 *
 * The library (libnkv.so) replaces three pieces of the reference's attention
 * path with hand-written CUDA kernels:
 *
 *   1. the paged KV slot write        (Triton store_kvcache_kernel)
 *   2. paged decode attention         (flash_attn_with_kvcache, block-table form)
 *   3. KV-cache compression           (torch MyCompressCompact + SnapKV), both the
 *                                      periodic window form and KvChat's threshold
 *                                      S -> R form with its query window.
 *
 * Conventions shared by every entry point:
 *   - All tensor pointers are DEVICE pointers. 16-bit floating point data is
 *     bfloat16 and is passed as void*. Index tensors are int32.
 *   - Sizes and strides are host integers. Strides are counted in ELEMENTS.
 *   - The KV cache of one layer is laid out exactly like the reference's
 *     per-layer view kv_cache[0|1, layer] of shape
 *     [num_blocks, block_size, num_kv_heads, head_dim], contiguous, so a slot
 *     (block_id * block_size + offset) addresses a row of num_kv_heads*head_dim
 *     elements.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *     Every call is stream-ordered, performs no host synchronisation and
 *     allocates no device memory; scratch memory ("workspace") is owned and
 *     passed in by the caller.
 *   - Every call returns an nkv_status (0 = success). No C++ exception crosses
 *     this boundary. Device-side range checks never trap: they skip the bad
 *     access and set a bit in a sticky per-device error word that
 *     nkv_read_device_error() returns.
 */
#ifndef NKV_H_
#define NKV_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum nkv_status {
  NKV_OK = 0,
  NKV_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative size, bad stride */
  NKV_ERR_UNSUPPORTED = 2,      /* head_dim, block_size or group width outside the kernels' range */
  NKV_ERR_WORKSPACE = 3,        /* workspace missing or smaller than the *_workspace_size query */
  NKV_ERR_ALIGNMENT = 4,        /* pointer or stride not 16-byte aligned where TMA or 128-bit loads need it */
  NKV_ERR_CUDA = 5              /* CUDA launch / driver error (see nkv_last_cuda_error) */
} nkv_status;

/* Bits of the sticky device error word. */
#define NKV_DEVERR_STORE_SLOT      0x1u  /* slot_mapping entry outside [-1, num_slots) */
#define NKV_DEVERR_DECODE_BLOCK    0x2u  /* block_tables entry outside [0, num_blocks) on a live token, or a context length past max_blocks * block_size (clamped) */
#define NKV_DEVERR_WAIT_TIMEOUT    0x4u  /* a bounded mbarrier / cluster wait gave up */
#define NKV_DEVERR_COMPRESS_RANGE  0x8u  /* compression window or slot outside the cache */
#define NKV_DEVERR_RING_RANGE      0x10u /* query-window ring slot / position out of range */
#define NKV_DEVERR_PREFILL_RANGE   0x20u /* cu_seqlens / max_seqlen_q outside the tensors or the grid */
#define NKV_DEVERR_ROPE_POSITION   0x40u /* position outside the rotary cos/sin cache (clamped) */
#define NKV_DEVERR_LAUNCH_SHAPE    0x80u /* a kernel ran without the thread-block clusters it needs (nothing written) */

/* Human-readable name of a status code (static string). */
const char* nkv_status_string(int status);

/* ABI version of this header (major * 100 + minor). */
int nkv_abi_version(void);

/* Last CUDA runtime error code seen by an entry point on this thread (0 if none). */
int nkv_last_cuda_error(void);

/* Reads (and optionally clears) the sticky device error word of the current
 * device. This is the one call that synchronises: it copies 4 bytes to the
 * host. Meant for tests and debugging, not for the decode loop. */
int nkv_read_device_error(uint32_t* out_bits, int clear);

/* ------------------------------------------------------------------------ */
/* 1. store_kvcache                                                          */
/* Replaces: store_kvcache / store_kvcache_kernel,                           */
/*   nanokvllm/layers/attention.py:10-40 (same in KvChat/layers/attention.py:10-40). */
/* For each token i with s = slot_mapping[i] != -1:                          */
/*   k_cache[s, :, :] = key[i, :, :];  v_cache[s, :, :] = value[i, :, :]     */
/* key/value rows are num_kv_heads*head_dim contiguous elements starting at  */
/* key + i*key_stride (the reference asserts stride(1) == head_dim and       */
/* stride(-1) == 1; the row stride may be the qkv split stride).             */
/* num_tokens == 0 or num_slots == 0 is a no-op (the reference's warm-up     */
/* with empty caches, model_runner.py:97-131).                               */
int nkv_store_kvcache(const void* key, int64_t key_stride,
                      const void* value, int64_t value_stride,
                      void* k_cache, void* v_cache, int64_t num_slots,
                      const int32_t* slot_mapping, int32_t num_tokens,
                      int32_t num_kv_heads, int32_t head_dim, void* stream);

/* ------------------------------------------------------------------------ */
/* 2. Paged decode attention                                                 */
/* Replaces: flash_attn_with_kvcache(q.unsqueeze(1), k_cache, v_cache,       */
/*   cache_seqlens=context_lens, block_table=block_tables, softmax_scale,    */
/*   causal=True) at nanokvllm/layers/attention.py:104-107 and               */
/*   KvChat/layers/attention.py:113-116.                                     */
/* out[b, h, :] = softmax(scale * q[b,h] . K[b, h/g, t]^T, t < context_lens[b]) V */
/* with g = num_q_heads / num_kv_heads and keys found through                */
/* block_tables[b, t / block_size]. context_lens[b] == 0 writes zeros.       */
/* q rows: q + b*q_stride_token + h*q_stride_head (head_dim contiguous).     */
/* out rows: out + b*out_stride_token + h*head_dim.                          */
/* Supported: head_dim 128, block_size a multiple of 128, g in [1, 16],      */
/* batch * num_kv_heads <= 65536.                                            */
/* The workspace must be zero-filled once before its first use. Every call   */
/* leaves its counter region zeroed again (partial results elsewhere in the  */
/* buffer may stay), so one buffer serves all layers, shapes and CUDA graphs.*/
size_t nkv_paged_decode_workspace_size(int32_t batch, int32_t num_q_heads,
                                       int32_t num_kv_heads, int32_t head_dim,
                                       int32_t max_blocks, int32_t block_size);
int nkv_paged_decode(const void* q, int64_t q_stride_token, int64_t q_stride_head,
                     const void* k_cache, const void* v_cache, int64_t num_blocks,
                     const int32_t* block_tables, int32_t max_blocks,
                     const int32_t* context_lens,
                     void* out, int64_t out_stride_token,
                     int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                     int32_t head_dim, int32_t block_size, float softmax_scale,
                     void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* 2b. Fused decode step: slot write + optional query-window append + decode */
/* Replaces, in one launch, the decode-step sequence of                      */
/*   nanokvllm/layers/attention.py:72-73 (store_kvcache) and :104-107        */
/*   (flash_attn_with_kvcache), and for KvChat also the query-window append  */
/*   of KvChat/layers/attention.py:80-87.                                    */
/* Same result as nkv_store_kvcache(key, value, slot_mapping) [then          */
/* nkv_query_window_append] then nkv_paged_decode, for a decode step: one   */
/* new token per batch row, whose slot_mapping[b] is -1 or the slot of       */
/* position context_lens[b]-1 (how the reference's decode step builds it,    */
/* nanokvllm/engine/model_runner.py:194 and :279). Rows violating that are   */
/* not written and flag NKV_DEVERR_STORE_SLOT. The producer warp writes each */
/* kv head's new row to the cache and into the shared-memory copy of the     */
/* tile that holds it (after that tile's TMA has landed), so no second       */
/* launch or cross-CTA ordering is needed.                                   */
/* metadata_ready = 1 lets the launch read block_tables, context_lens,      */
/* slot_mapping, the ring indices and the cached K/V rows other than the     */
/* step's new ones before it waits for the kernel it depends on             */
/* (programmatic dependent launch): the caller vouches that the kernel       */
/* launched just before this call on the stream writes none of them (host    */
/* copies and earlier kernels are fine; a compression kernel that rewrites   */
/* context_lens or the cache right before, or a separate slot write of this  */
/* step's rows, is not). In a chain of decode launches that hides the        */
/* metadata loads and a CTA's first K/V tile behind the previous launch's    */
/* tail. 0 reads everything after the wait. q, key and value are always read */
/* after it.                                                                 */
/* ring may be NULL (no query window). Otherwise it is the KvChat ring       */
/* [num_ring_slots, num_layers, window_size, num_q_heads, head_dim]; row b   */
/* appends q[b] to ring[ring_slot_of_row[b], layer_id, ring_pos_of_row[b]]   */
/* when ring_slot_of_row[b] >= 0; q heads must then be contiguous            */
/* (q_stride_head == head_dim).                                              */
int nkv_decode_step(const void* q, int64_t q_stride_token, int64_t q_stride_head,
                    const void* key, int64_t key_stride, const void* value, int64_t value_stride,
                    const int32_t* slot_mapping,
                    void* k_cache, void* v_cache, int64_t num_blocks,
                    const int32_t* block_tables, int32_t max_blocks,
                    const int32_t* context_lens,
                    void* ring, int32_t num_ring_slots, int32_t num_layers,
                    int32_t window_size, int32_t layer_id,
                    const int32_t* ring_slot_of_row, const int32_t* ring_pos_of_row,
                    void* out, int64_t out_stride_token,
                    int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                    int32_t head_dim, int32_t block_size, float softmax_scale,
                    int32_t metadata_ready,
                    void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* 2c. Prefill / mixed-batch attention (variable-length, causal)            */
/* Replaces: flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k,     */
/*   max_seqlen_q, max_seqlen_k, softmax_scale, causal=True, block_table)    */
/*   at nanokvllm/layers/attention.py:96-102 and KvChat/layers/attention.py: */
/*   105-111 (metadata: nanokvllm/engine/model_runner.py:160-220).           */
/* Sequence b has Lq = cu_seqlens_q[b+1]-cu_seqlens_q[b] query rows (q/out   */
/* rows cu_seqlens_q[b] ..) and Lk = cu_seqlens_k[b+1]-cu_seqlens_k[b] keys.  */
/* out[t, h] = softmax(scale * q[t, h] K^T) V over the keys of kv head       */
/* h / g that query i (= t - cu_seqlens_q[b]) may see: all Lk keys, or with  */
/* causal != 0 keys j <= Lk - Lq + i (bottom-right aligned mask, as          */
/* flash-attn >= 2.1). A row that sees no key gets zeros.                    */
/* Keys: with block_tables (the paged cache [num_blocks, block_size, Hk, D], */
/* k_stride_token = v_stride_token = Hk*D, num_kv_rows = num_blocks *        */
/* block_size) key j of sequence b is row block_tables[b, j / block_size] *  */
/* block_size + j % block_size; with block_tables == NULL (prefill without a */
/* cached prefix) it is row cu_seqlens_k[b] + j of k / v [num_kv_rows, Hk, D].*/
/* max_seqlen_q sizes the grid and must be >= every Lq (rows violating it,   */
/* or cu_seqlens outside num_q_tokens / num_kv_rows / the block table, are   */
/* skipped and flag NKV_DEVERR_PREFILL_RANGE).                               */
/* Supported: head_dim 128, g = num_q_heads / num_kv_heads in [1, 128],      */
/* block_size 64 or a multiple of 128, heads of k / v / out contiguous       */
/* (stride D), out 16-byte aligned with out_stride_token a multiple of 8.    */
/* softmax_scale must be finite and > 0.                                     */
/* No workspace; nothing is allocated.                                       */
int nkv_paged_prefill(const void* q, int64_t q_stride_token, int64_t q_stride_head,
                      int64_t num_q_tokens,
                      const void* k, int64_t k_stride_token,
                      const void* v, int64_t v_stride_token, int64_t num_kv_rows,
                      const int32_t* block_tables, int32_t max_blocks, int32_t block_size,
                      const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k,
                      int32_t batch, int32_t max_seqlen_q, int32_t causal,
                      void* out, int64_t out_stride_token,
                      int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                      float softmax_scale, void* stream);

/* ------------------------------------------------------------------------ */
/* 2d. q/k RMSNorm + rotary embedding + slot write (one launch)             */
/* Replaces the per-layer sequence q_norm / k_norm / rotary_emb of          */
/*   nanokvllm/models/qwen3.py:109-113 and store_kvcache of                  */
/*   nanokvllm/layers/attention.py:72-73.                                    */
/* qkv: the qkv projection output [num_tokens, (Hq + 2 Hk) * head_dim] bf16 */
/* (row stride qkv_stride_token). For token t and head h:                   */
/*   q heads: q_out[t, h] = rope(rmsnorm(q[t, h]) * q_norm_weight)           */
/*   k heads: k = rope(rmsnorm(k[t, h]) * k_norm_weight), written to          */
/*            k_cache[slot_mapping[t], h] (and to k_out[t, h] if k_out is     */
/*            not NULL); v[t, h] is copied to v_cache[slot_mapping[t], h].    */
/* slot_mapping[t] == -1 skips the cache writes (graph padding); k_cache may */
/* be NULL (no cache yet, as the reference's warm-up). RMSNorm: fp32 mean of */
/* squares, bf16(x * rsqrt(var + eps)) * weight rounded to bf16 (the        */
/* reference module's rounding points, layers/layernorm.py:16-25). RoPE:     */
/* rotate-half with cos / sin from cos_sin_cache[positions[t]]               */
/* ([max_positions, head_dim] fp32: cos then sin, rotary_embedding.py:7-45). */
/* Positions outside the cache are clamped and flag NKV_DEVERR_ROPE_POSITION;*/
/* slots >= num_slots are not written and flag NKV_DEVERR_STORE_SLOT.       */
/* Supported: head_dim 128; all pointers 16-byte aligned, row strides       */
/* multiples of 8 elements.                                                  */
int nkv_qk_norm_rope_store(const void* qkv, int64_t qkv_stride_token, int32_t num_tokens,
                           const int64_t* positions, const float* cos_sin_cache,
                           int64_t max_positions, const void* q_norm_weight,
                           const void* k_norm_weight, float eps,
                           void* q_out, int64_t q_out_stride_token,
                           void* k_out, int64_t k_out_stride_token,
                           void* k_cache, void* v_cache, int64_t num_slots,
                           const int32_t* slot_mapping,
                           int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                           void* stream);

/* ------------------------------------------------------------------------ */
/* 2e. o_proj GEMM + tensor-parallel all-reduce in one kernel (decode sizes) */
/* Replaces RowParallelLinear.forward's F.linear + dist.all_reduce           */
/* (nanokvllm/layers/linear.py:151-155) for tokens <= 512:                   */
/*   y[t, :] = sum over ranks of x_rank[t, :] @ w_rank^T                    */
/* x [tokens, k] bf16 (row stride ldx), w [n, k] bf16 (the rank's weight     */
/* shard, row stride ldw), y [tokens, n] bf16 (row stride ldy). Each rank    */
/* writes its partial product, rounded to bf16 as F.linear's output is, to  */
/* its copy of a symmetric bf16 [tokens, n] buffer (part_local; part_mc =   */
/* the buffer's multicast address); after an in-kernel barrier every rank   */
/* sums its 1/world slice in fp32 through NVLink SHARP (multimem.ld_reduce  */
/* .acc::f32) and broadcasts the bf16 result into every rank's copy of a    */
/* symmetric bf16 [tokens, n] buffer (out_mc / out_local); after a second    */
/* barrier it copies the result to y. sig_mc / sig_local: a symmetric       */
/* uint32[2] of arrival counters (every CTA of every rank adds one per       */
/* barrier); flags: this rank's uint32[5] (the two barriers' counter         */
/* targets, the tiling of the last launch as (TN << 8) | S, the status word, */
/* the call's epoch); counters and flags zeroed once. Targets and epoch are  */
/* read and advanced on the device, so every rank must make the same        */
/* sequence of calls and a CUDA graph may replay them. Waits are bounded by  */
/* timeout_ns. A wait that gives up sets NKV_DEVERR_WAIT_TIMEOUT and ORs     */
/* into the status word which one (1 TMA ring, 2 MMA stage, 4 accumulator,   */
/* 8 cross-rank barrier); the data it guarded becomes NaN (a failed GEMM     */
/* sends NaN partials, a failed barrier leaves NaN in y), the targets are    */
/* not advanced, and the group must rebuild its buffers before calling again.*/
/* Needs k % 64 == 0,                                                       */
/* n % 32 == 0, 16-byte aligned x, w, y and buffers, row strides multiples  */
/* of 8. Cooperative launch of (n / TN) * S CTAs, TN in {32, 64, 128}        */
/* output columns per tile and S in {1, 2, 4} CTAs per tile (a cluster,      */
/* each CTA a K / S range, their fp32 partial tiles summed through          */
/* `workspace`, a 16-byte aligned device buffer of workspace_bytes: S > 1   */
/* needs S * ceil(tokens / 128) * 128 * n * 4 bytes, so 16 * 512 * n bytes   */
/* allow every S; with null or less, S = 1). The launch picks the pair that */
/* streams the fewest bytes per CTA and fits the GPU at once.               */
int nkv_oproj_allreduce(const void* x, int64_t ldx, const void* w, int64_t ldw, int32_t tokens,
                        int32_t k, int32_t n, void* part_mc, void* part_local, void* out_mc,
                        const void* out_local, void* sig_mc, void* sig_local, uint32_t* flags,
                        int32_t rank, int32_t world, uint64_t timeout_ns, void* workspace,
                        int64_t workspace_bytes, void* y, int64_t ldy, void* stream);

/* One-shot variant of the same replacement, without NVLink multicast: each  */
/* rank stores its bf16 partial (rounded as F.linear's output is) straight   */
/* from the GEMM epilogue into its slot of EVERY rank's receive buffer       */
/* (plain stores through peer mappings, NVLink for the other ranks), then    */
/* one in-kernel barrier, then every rank sums the world slots in rank order */
/* (fp32, so all ranks hold the same bf16 result) into y. recv_peers: device */
/* array of world pointers, rank q's receive buffer of                       */
/* [2 parities][world][slot_stride] bf16 (slot_stride >= tokens * n, a       */
/* multiple of 8); the parity alternates per call, so a rank's next call     */
/* never overwrites a slot a peer is still summing. sig_peers: device array  */
/* of world pointers to each rank's uint32[2] arrival counters (sig_local =  */
/* this rank's). flags, epoch, waits, limits, workspace and the             */
/* cooperative cluster launch as nkv_oproj_allreduce. Egress per rank:       */
/* (world - 1) x the partial, so it suits small TP groups.                  */
int nkv_oproj_allreduce_p2p(const void* x, int64_t ldx, const void* w, int64_t ldw,
                            int32_t tokens, int32_t k, int32_t n, void* const* recv_peers,
                            int64_t slot_stride, uint32_t* const* sig_peers, void* sig_local,
                            uint32_t* flags, int32_t rank, int32_t world, uint64_t timeout_ns,
                            void* workspace, int64_t workspace_bytes, void* y, int64_t ldy,
                            void* stream);

/* ------------------------------------------------------------------------ */
/* 3a. Periodic window compression (one layer, all selected sequences)       */
/* Replaces: MyCompressCompact, nanokvllm/layers/compress_utils.py:100-263,  */
/*   with get_tail_window_and_tail_slots (:9-72), gather_kv_by_slots (:75-97) */
/*   and SnapKV(window=obs_window) (nanokvllm/layers/CompressMethod.py:4-58). */
/* For selected sequence i (batch row b = selected_batch_indices[i]):        */
/*   L0 = base_context_lens[b]; the window is the last window_blocks FULL    */
/*   blocks before position L0; the last obs_window window tokens are kept    */
/*   and scored against q[b]; SnapKV keeps token 0, the top                   */
/*   keep_tokens-1-obs_window tokens by summed softmax importance (bf16      */
/*   rounding points of the reference, ties broken towards the lower index)  */
/*   and the obs_window last tokens; kept rows are compacted in place to the */
/*   first keep_tokens slots of the window, the partial tail block follows   */
/*   them, and context_lens[b] = L0 - window_blocks*block_size + keep_tokens. */
/* out_keep_idx (optional, [num_selected, keep_tokens]) receives the window-  */
/* relative kept indices; out_new_lens (optional, [num_selected]) the new     */
/* lengths; out_importance (optional, bf16 [num_selected, window_tokens -     */
/* obs_window]) the importance the top-k ranked (SnapKV's key_importance).    */
/* Needs num_kv_heads <= 8 (one thread-block cluster per sequence).          */
/* Entries of selected_batch_indices equal to -1 are skipped.                */
/* The caller guarantees what the reference asserts (full_blocks >=          */
/* window_blocks); rows violating it are skipped and flag                    */
/* NKV_DEVERR_COMPRESS_RANGE. The tail rows go to the slots after the last    */
/* kept slot in slot arithmetic, as the reference moves them; when           */
/* keep_tokens + tail exceeds the window they run into the next physical     */
/* block. Each sequence's own rows are read before that write, but two       */
/* sequences of one call whose escaped rows land in a block the other reads  */
/* are not ordered (the reference reads every row of the step first).        */
/* block_size must be a multiple of 64.                                      */
int nkv_window_compress(const void* q, int64_t q_stride_token,
                        void* k_cache, void* v_cache, int64_t num_blocks,
                        const int32_t* block_tables, int32_t max_blocks,
                        const int32_t* base_context_lens, int32_t* context_lens,
                        const int32_t* selected_batch_indices, int32_t num_selected,
                        int32_t window_blocks, int32_t keep_tokens, int32_t obs_window,
                        int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                        int32_t block_size, float softmax_scale,
                        int32_t* out_keep_idx, int32_t* out_new_lens, void* out_importance,
                        void* stream);

/* 3a'. Device-side selection of the rows a periodic compression step takes */
/* (the reference's host loop in prepare_decode, nanokvllm/engine/          */
/* model_runner.py:305-321), so the whole compression step can be captured  */
/* in a CUDA graph and replayed: row b (length context_lens[b]) is skipped   */
/* when its length mod block_size == block_size - 1, eligible when          */
/* tail_uncompressed[b] >= window_blocks * block_size and                    */
/* context_lens[b] / block_size >= window_blocks; the first topk eligible   */
/* rows in batch order go to out_selected[0, count), the rest of            */
/* out_selected[topk] is -1 (nkv_window_compress skips -1 entries, so it is  */
/* called with num_selected = topk). out_count [1] and out_base_lens        */
/* [batch] (a copy of context_lens: the base lengths nkv_window_compress    */
/* reads) may be NULL.                                                       */
int nkv_window_select(const int32_t* context_lens, const int32_t* tail_uncompressed,
                      int32_t batch, int32_t block_size, int32_t window_blocks, int32_t topk,
                      int32_t* out_selected, int32_t* out_count, int32_t* out_base_lens,
                      void* stream);

/* ------------------------------------------------------------------------ */
/* 3b. KvChat query window: append this step's queries of active sequences  */
/* Replaces: QueryWindowManager.append, KvChat/engine/query_window_manager.py:46-58 */
/* (the Python loop of per-sequence copy_ calls).                            */
/* ring is [num_ring_slots, num_layers, window_size, num_q_heads, head_dim]. */
/* For active row j: ring[ring_slot[j], layer_id, ring_pos[j], :, :] =        */
/*   q[batch_index[j], :, :]. All three index arrays live on the device so    */
/* the call can sit inside a captured CUDA graph.                            */
int nkv_query_window_append(const void* q, int64_t q_stride_token,
                            void* ring, int32_t num_ring_slots, int32_t num_layers,
                            int32_t window_size, int32_t layer_id,
                            const int32_t* batch_index, const int32_t* ring_slot,
                            const int32_t* ring_pos, int32_t num_active,
                            int32_t num_q_heads, int32_t head_dim, void* stream);

/* ------------------------------------------------------------------------ */
/* 3c. KvChat threshold compression S -> R (one layer)                       */
/* Replaces: MyCompressCompact, KvChat/layers/compress_utils.py:10-171, with */
/*   TritonGetKVForComp (:218-252) and SnapKV(window=W, num_keep=R-W-1)      */
/*   (KvChat/layers/CompressMethod.py:4-58).                                 */
/* For selected sequence i (row b): the source window is positions           */
/* [max(context_lens[b]-S, 0), +S); its first S-W keys are scored by the W   */
/* ring queries of ring slot ring_slot_of_selected[i] (all heads, all W      */
/* queries); SnapKV keeps token 0, the top R-W-1 and the last W; kept rows   */
/* are compacted to positions [0, R) of the sequence's block table and       */
/* context_lens[b] = R. out_keep_idx is optional ([num_selected, R]), and so */
/* is out_importance (bf16 [num_selected, S - W]: the importance ranked).    */
int nkv_threshold_compress(const void* ring, int32_t num_ring_slots, int32_t num_layers,
                           int32_t window_size, int32_t layer_id,
                           const int32_t* ring_slot_of_selected,
                           void* k_cache, void* v_cache, int64_t num_blocks,
                           const int32_t* block_tables, int32_t max_blocks,
                           int32_t* context_lens,
                           const int32_t* selected_batch_indices, int32_t num_selected,
                           int32_t compress_S, int32_t compress_R,
                           int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                           int32_t block_size, float softmax_scale,
                           int32_t* out_keep_idx, void* out_importance, void* stream);

/* ------------------------------------------------------------------------ */
/* 4. Paged decode without a caller-provided workspace                       */
/* No counterpart in the reference: an addition for callers that cannot      */
/* allocate device memory -- code that runs while a CUDA graph is being      */
/* captured, serving runtimes whose memory pool is sealed after start-up,    */
/* and plugin hosts that hand a kernel its inputs and outputs but no scratch */
/* buffer. It computes exactly what nkv_paged_decode computes, with the same */
/* arguments minus the workspace, and allocates nothing: its scratch is a    */
/* fixed array of NKV_STATIC_SCRATCH_BYTES in the library's device image,    */
/* present on every GPU that loads libnkv.so until the process exits.        */
/*   - A problem whose nkv_paged_decode_workspace_size exceeds               */
/*     NKV_STATIC_SCRATCH_BYTES is rejected with NKV_ERR_WORKSPACE before     */
/*     anything is launched (16 MiB covers e.g. batch 256 x 8 kv heads of    */
/*     8k-token contexts, 8.8 MB; use nkv_paged_decode for larger batches).  */
/*   - The first call on each device looks up the array's device address     */
/*     (cudaGetSymbolAddress with that device current); make that first call */
/*     outside any stream capture.                                           */
/*   - Every call on a device shares the one array and clears the counters   */
/*     it needs on `stream` before the launch. Calls that overlap on the GPU */
/*     (different streams without ordering between them) race on it.        */
#define NKV_STATIC_SCRATCH_BYTES (16u << 20)
int nkv_paged_decode_static_scratch(const void* q, int64_t q_stride_token, int64_t q_stride_head,
                                    const void* k_cache, const void* v_cache, int64_t num_blocks,
                                    const int32_t* block_tables, int32_t max_blocks,
                                    const int32_t* context_lens,
                                    void* out, int64_t out_stride_token,
                                    int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                                    int32_t head_dim, int32_t block_size, float softmax_scale,
                                    void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* NKV_H_ */
