/*
 * dsr_b200.h -- C ABI of the B200 (sm_100a) attention hot path of DeepSeekRPC.
 *
 * Every entry point takes plain device pointers, element counts and a
 * cudaStream_t passed as `void*` (NULL = legacy default stream).  The compute
 * entry points allocate no device memory (callers pass outputs and scratch),
 * never synchronize the stream and never read device data on the host; work is
 * enqueued on `stream` only.  The exceptions are the peer-exchange set-up calls
 * at the end of this header: dsr_p2p_alloc / dsr_p2p_free allocate and free the
 * exchange buffer (cudaMalloc / cudaFree) and dsr_p2p_open / dsr_p2p_close map
 * and unmap a peer's buffer (CUDA IPC), once per process, outside the step.
 *
 * Two error channels, as in the reference extension:
 *   - host return value: DSR_OK, or a negative code for argument / shape / bound
 *     violations (the reference raises them through TORCH_CHECK) and launch
 *     failures; dsr_last_error() returns the message for the calling thread.
 *   - device status word `err` (one int32 in device memory, zeroed by the
 *     caller): data-dependent errors, first error wins via atomicCAS.  Codes 1..3
 *     keep the reference meaning (native/operations.cu:44-158).
 *
 * Storage dtypes: BF16 values are passed as uint16_t bit patterns.
 */
#ifndef DSR_B200_H
#define DSR_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- device status codes (written to err[0]) ---------------------------- */
#define DSR_ERR_ID 1        /* invalid id, slot, block or visibility          */
#define DSR_ERR_NONFINITE 2 /* non-finite input, score or output              */
#define DSR_ERR_SCATTER 3   /* scatter bounds / duplicate / stale generation  */
#define DSR_ERR_TIMEOUT 4   /* a bounded device-side wait gave up (new code)  */

/* ---- host return codes --------------------------------------------------- */
#define DSR_OK 0
#define DSR_EINVAL (-1)  /* shape, dtype-size or bound violation             */
#define DSR_ECUDA (-2)   /* CUDA runtime / launch failure                    */
#define DSR_ENODEV (-3)  /* current device is not a compute-capability 10.x GPU */

/* Fixed geometry of the paged decode path (DeepSeek V3.2/V4 sparse MLA). */
#define DSR_BLOCK_TOKENS 64 /* tokens per paged pool block                   */
#define DSR_INDEX_DIM 128   /* index-key width                               */
#define DSR_KV_DIM 576      /* latent 512 + rope 64                          */
#define DSR_V_DIM 512       /* value width = leading latent columns          */
#define DSR_SWA_ROWS 128    /* sliding-window ring rows per sequence         */

/* ABI generation; the reference module returns 2 from abi_version()
 * (native/bindings.cpp:25). */
int dsr_abi_version(void);

/* Message of the last nonzero host return on this thread ("" if none). */
const char* dsr_last_error(void);

/* Returns DSR_OK when the current CUDA device is sm_100-class, else DSR_ENODEV. */
int dsr_device_check(void);

/* ===================== reference drop-in operations ======================= */

/* Replaces ds_index_scores / index_kernel (native/operations.cu:84-123,199-212).
 * q f32[rows,heads,128], keys bf16[capacity,128], weights f32[rows,heads],
 * ids i32[rows,columns], visible i32[rows] -> out f32[rows,columns].
 * out[r,c] = sum_h w[r,h]*max(q[r,h].keys[id],0); -inf for id==-1 or id>=visible[r].
 * Bounds widened from the reference: heads <= 64 (was 32), columns < 2^31
 * (was 8192), rows <= 65536 (was 4096). */
int dsr_index_scores(const float* q, const uint16_t* keys, const float* weights,
                     const int32_t* ids, const int32_t* visible, float* out, int32_t* err,
                     int64_t rows, int64_t heads, int64_t columns, int64_t capacity,
                     void* stream);

/* Replaces ds_sparse_attention / sparse_kernel (native/operations.cu:30-82,180-197).
 * q f32[rows,heads,width], window bf16[window_rows,width], source
 * bf16[source_rows,width], ids i32[rows,selected], sink f32[heads] ->
 * out f32[rows,heads,width]; online softmax whose initial state is (sink, 1, 0).
 * Bounds widened: width <= 576 (was 512), window_rows <= 65536 (was 8192),
 * source_rows < 2^31 (was 2^20), selected <= 65536 (was 4096). */
int dsr_sparse_attention(const float* q, const uint16_t* window, const uint16_t* source,
                         const int32_t* ids, const float* sink, float* out, int32_t* err,
                         int64_t rows, int64_t heads, int64_t width, int64_t window_rows,
                         int64_t source_rows, int64_t selected, float scale, void* stream);

/* Replaces ds_scatter_slots / scatter_kernel (native/operations.cu:144-161,227-243).
 * Generation-checked row scatter; does not modify `generations` (the caller
 * bumps them, reference cache_pool.py:309).  Width bound widened to 576. */
int dsr_scatter_slots(uint16_t* pool, const int64_t* generations, const int32_t* slots,
                      const int64_t* expected, const uint16_t* values, int32_t* err,
                      int64_t rows, int64_t width, int64_t capacity, void* stream);

/* Replaces ds_engram_decode / engram_kernel (native/operations.cu:125-142,214-225).
 * u8[rows,264] FP8-E4M3 x UE8M0 -> bf16[rows,256]. */
int dsr_engram_decode(const uint8_t* encoded, uint16_t* out, int32_t* err, int64_t rows,
                      void* stream);

/* ========================= exact top-k selection ========================== */

/* Replaces the streaming top-k of TiledIndexer._select + merge_ranked
 * (src/deepseekrpc/index_selection.py:9-19,79-124).
 * For each row r: among entries i < lengths[r] (and ids[r,i] >= 0 when `ids` is
 * given) select the k largest scores; equal scores prefer the lower id; -0.0
 * equals +0.0.  Output out_ids i32[rows,k]: the selected ids in ascending order,
 * padded with -1.  Optional out_scores f32[rows,k] holds the matching scores
 * (padding: -inf).  When `ids` is NULL the id of entry i is i + id_base.
 * When `ids` is given, valid ids must increase along each row (any -1 entries
 * are skipped).  k <= 8192; row_stride >= max length.
 * Scratch: dsr_topk_workspace_bytes(rows, row_stride) bytes, 256-byte aligned,
 * zero before its first use; every completed call leaves it zero again.  Calls
 * sharing a workspace must not overlap on the GPU. */
size_t dsr_topk_workspace_bytes(int64_t rows, int64_t row_stride);
int dsr_topk_select(const float* scores, const int32_t* ids, const int32_t* lengths,
                    int32_t* out_ids, float* out_scores, int32_t* err, int64_t rows,
                    int64_t row_stride, int64_t k, int64_t id_base, void* workspace,
                    size_t workspace_bytes, void* stream);

/* Allocation-free variant of dsr_topk_select.  No reference counterpart: it
 * serves hosts that cannot hand the library device memory per call.  Same
 * arguments, validation and results as dsr_topk_select, minus the workspace.
 * Scratch is a fixed DSR_TOPK_NOALLOC_BYTES array inside this library (one per
 * device); calls with dsr_topk_workspace_bytes(rows, row_stride) above it are
 * refused with DSR_EINVAL before any CUDA call (e.g. 8 rows x 131072 entries
 * fit, 16 rows x 131072 do not).  Nothing is allocated: a call outside stream
 * capture looks the array's address up (cudaGetSymbolAddress) on the current
 * device; a captured call reuses the address of the last uncaptured call on
 * that device, so make the first call on each device outside any stream
 * capture (after a device reset, make one more); each call clears the zero-initialised
 * part of the scratch with cudaMemsetAsync on `stream` before its kernels.
 * All calls on one device share the scratch: calls that overlap on the GPU
 * (different streams, or threads without ordering) race and must be
 * serialised by the caller. */
#define DSR_TOPK_NOALLOC_BYTES (16u << 20)
int dsr_topk_select_noalloc(const float* scores, const int32_t* ids, const int32_t* lengths,
                            int32_t* out_ids, float* out_scores, int32_t* err, int64_t rows,
                            int64_t row_stride, int64_t k, int64_t id_base, void* stream);

/* ======================== paged decode hot path =========================== */

/* Lightning-indexer scores over a paged BF16 index-key pool, tcgen05 tensor cores.
 * index_pool bf16[pool_blocks*64,128]; block_table i32[batch,table_stride]
 * (physical block of logical block j = positions 64j..64j+63);
 * visible i32[batch] keys per row (<= score_stride, else err 1); q f32[batch,heads,128]; weights
 * f32[batch,heads]; heads in {16,32,64}.
 * scores f32[batch,score_stride]: scores[b,p] for p < visible[b].
 * Replaces TiledIndexer's per-tile index_scores calls (index_selection.py:94-107)
 * for the dense (non-candidate) case. */
int dsr_indexer_decode(const float* q, const float* weights, const uint16_t* index_pool,
                       int64_t pool_blocks, const int32_t* block_table, int64_t table_stride,
                       const int32_t* visible, float* scores, int64_t score_stride,
                       int32_t* err, int64_t batch, int64_t heads, void* stream);

/* Lightning-indexer scores of a chunk of prefill queries against ONE sequence,
 * as a tcgen05 GEMM: each 128-key tile is contracted against a group of 128/heads
 * queries at once.  q f32[queries,heads,128]; weights f32[queries,heads];
 * index_pool and paging as above, block_table i32[table_len] the sequence's
 * blocks; visible i32[queries] keys query t sees (causal: its position + 1,
 * <= score_stride and <= table_len*64, else err 1); heads in {32,64}.
 * scores f32[queries,score_stride]: scores[t,p] for p < visible[t].  Queries
 * whose FP32 values are not BF16-exact are contracted as bf16(q) plus the
 * bf16 residual.  Replaces TiledIndexer's per-row tiles for prefill rows
 * (index_selection.py:79-107); the per-query top-k runs on the scores with
 * dsr_topk_select. */
int dsr_indexer_prefill(const float* q, const float* weights, const uint16_t* index_pool,
                        int64_t pool_blocks, const int32_t* block_table, int64_t table_len,
                        const int32_t* visible, float* scores, int64_t score_stride, int32_t* err,
                        int64_t queries, int64_t heads, void* stream);

/* Candidate-block mode of TiledIndexer (index_selection.py:62-90,108-123).
 * dsr_candidate_blocks: from a dense indexer's scores f32[rows,score_stride]
 * (entries < visible[r]), block scores = max over 8 consecutive positions (NaN
 * propagates), the block of position visible-1 pinned to +inf, and the `keep`
 * best blocks (ties: lower block id) -> out_blocks i32[rows,keep] ascending,
 * -1 padded.  dsr_candidate_select: a later indexer scores only the positions
 * of candidate_blocks i32[rows,ncand] (ascending, -1 padded, each block below
 * ceil(visible/8), at least one for a nonempty row; else status 1 and nothing
 * selected) below visible[r] and returns its top-k positions out_ids
 * i32[rows,k] ascending, -1 padded.  Scratch: the *_workspace_bytes() sizes,
 * 256-byte aligned, zero before first use. */
size_t dsr_candidate_blocks_workspace_bytes(int64_t rows, int64_t score_stride, int64_t keep);
int dsr_candidate_blocks(const float* scores, const int32_t* visible, int64_t rows,
                         int64_t score_stride, int64_t keep, int32_t* out_blocks, void* workspace,
                         size_t workspace_bytes, int32_t* err, void* stream);
size_t dsr_candidate_select_workspace_bytes(int64_t rows, int64_t ncand);
int dsr_candidate_select(const float* idx_q, const float* idx_w, int64_t idx_heads,
                         const uint16_t* index_pool, int64_t pool_blocks,
                         const int32_t* block_table, int64_t table_stride, const int32_t* visible,
                         const int32_t* candidate_blocks, int64_t ncand, int64_t k,
                         int32_t* out_ids, void* workspace, size_t workspace_bytes, int32_t* err,
                         int64_t rows, void* stream);

/* Sparse MLA decode attention over the SWA ring plus top-k selected pool rows.
 * q f32[batch,heads,576]; kv_pool bf16[pool_blocks*64,576]; block_table as above;
 * topk i32[batch,k] logical positions (ascending, -1 padded), each < visible[b];
 * swa bf16[batch,128,576] ring (row p%128 holds position p); swa_len i32[batch]
 * valid window rows (<= 128); sink f32[heads]; heads in {16,32,64,128}.
 * out f32[batch,heads,512] = softmax-with-sink weighted sum of the first 512
 * columns of the selected rows (reference sparse_kernel with V = K, restricted
 * to the value columns).  Scratch: workspace of dsr_mla_workspace_bytes(). */
size_t dsr_mla_workspace_bytes(int64_t batch, int64_t heads, int64_t k);
int dsr_sparse_mla_decode(const float* q, const uint16_t* kv_pool, int64_t pool_blocks,
                          const int32_t* block_table, int64_t table_stride,
                          const int32_t* visible, const int32_t* topk, int64_t k,
                          const uint16_t* swa, const int32_t* swa_len, const float* sink,
                          float scale, float* out, void* workspace, size_t workspace_bytes,
                          int32_t* err, int64_t batch, int64_t heads, void* stream);

/* Sparse MLA partial over ONE position shard, for sequence-sharded decode.
 * The pools, block table and swa hold this shard's positions
 * [id_base, id_base + visible[b]) (id_base a multiple of 64); topk holds the
 * GLOBAL selection (ids ascending, -1 padded): ids outside the shard are
 * skipped, not errors.  Outputs the unnormalised merged partial of the shard,
 * without the sink: out_o f32[batch,heads,512] = sum_i 2^{s_i - m} v_i,
 * out_m f32[batch,heads] = m (max of s_i, base-2 units: s_i = log2(e) * scale * q.k_i),
 * out_l f32[batch,heads] = sum_i 2^{s_i - m}; an empty shard gives m = -inf,
 * l = 0, o = 0.  dsr_lse_combine over the shards' partials with the sink
 * gives the full attention output.  Scratch: dsr_mla_workspace_bytes(). */
int dsr_sparse_mla_partial(const float* q, const uint16_t* kv_pool, int64_t pool_blocks,
                           const int32_t* block_table, int64_t table_stride,
                           const int32_t* visible, const int32_t* topk, int64_t k,
                           int64_t id_base, const uint16_t* swa, const int32_t* swa_len,
                           float scale, float* out_o, float* out_m, float* out_l,
                           void* workspace, size_t workspace_bytes, int32_t* err,
                           int64_t batch, int64_t heads, void* stream);

/* ===================== sequence-sharded decode (multi-GPU) ===================
 * Rank r of G holds positions [id_base, id_base + visible[b]) of every sequence
 * in its own pools.  Per step: dsr_indexer_topk_decode (local scores and top-k
 * with global ids and their scores) -> all-gather of the packed lists ->
 * dsr_topk_merge_lists (exact global top-k, same on every rank) ->
 * dsr_sparse_mla_partial (this rank's partial over its selected rows) ->
 * all-gather of the packed partials -> dsr_lse_combine_packed.  No reference
 * counterpart (the reference decodes on one GPU). */

/* Indexer scores -> exact top-k, chained on the device: out_ids i32[batch,k]
 * (id_base + position, ascending, -1 padded), out_scores (nullable)
 * f32[batch,k] their scores (-inf padding), scores_out (nullable)
 * f32[batch, round_up(max_visible,64)].  Arguments otherwise as
 * dsr_indexer_decode / dsr_topk_select.  Scratch as dsr_decode_step's. */
size_t dsr_indexer_topk_workspace_bytes(int64_t batch, int64_t max_visible);
int dsr_indexer_topk_decode(const float* idx_q, const float* idx_w, int64_t idx_heads,
                            const uint16_t* index_pool, int64_t pool_blocks,
                            const int32_t* block_table, int64_t table_stride,
                            const int32_t* visible, int64_t max_visible, int64_t k,
                            int64_t id_base, int32_t* out_ids, float* out_scores,
                            float* scores_out, void* workspace, size_t workspace_bytes,
                            int32_t* err, int64_t batch, void* stream);

/* Exact top-k of the union of per-shard ranked lists.  lists i32[world][2][rows][k]:
 * per shard the scores' bit patterns, then their ids (-1 padded); within a shard
 * ids increase, and every id of shard w is below every id of shard w+1.
 * out_ids i32[rows,k] ascending, -1 padded.  Scratch:
 * dsr_topk_merge_workspace_bytes(), 256-byte aligned, zero before first use. */
size_t dsr_topk_merge_workspace_bytes(int64_t rows, int64_t world, int64_t k);
int dsr_topk_merge_lists(const int32_t* lists, int64_t world, int64_t rows, int64_t k,
                         int32_t* out_ids, void* workspace, size_t workspace_bytes, int32_t* err,
                         void* stream);

/* Combine of the shards' partials in their exchange layout: packed
 * f32[world][o (batch*heads*512) | m (batch*heads) | l (batch*heads)] as written
 * by dsr_sparse_mla_partial into one buffer per rank; out f32[batch,heads,512]
 * with the sink counted once.  batch*heads must be even. */
int dsr_lse_combine_packed(const float* packed, int64_t world, const float* sink, float* out,
                           int32_t* err, int64_t batch, int64_t heads, void* stream);

/* Fused, generation-checked append of one KV row (576) and one index-key row
 * (128) per sequence into the paged pools and the SWA ring.  Replaces the two
 * DeviceRowPool.write calls of publish_source plus the SWA ring write
 * (attention_state.py:183-192, cache_pool.py:289-313, vllm_attention.py:261).
 * block_table i32[table_rows,table_stride]; seq i32[n] sequence of each new
 * row (< table_rows); positions i32[n] its logical position;
 * generations i64[pool_blocks*64] per physical row; expected i64[n].
 * A row is written only if its physical row is in bounds, not repeated by an
 * earlier row of the batch, generations[row]==expected[i] and both value rows
 * are finite; then generations[row] = expected[i]+1.  Otherwise err = 3
 * (bounds / duplicate / stale) or 2 (non-finite) and nothing of that row is
 * written.  swa (bf16[table_rows,128,576], row p%128) may be NULL; with it, a
 * row whose ring row (seq, p%128) repeats an earlier row's is refused too (3).
 * Rows that pass are written and bumped even if others fail: on a nonzero
 * status the caller rolls back or discards the whole batch, as the reference's
 * caller does after a failed scatter (cache_pool.py:304-313). */
int dsr_append_kv_index(uint16_t* kv_pool, uint16_t* index_pool, int64_t* generations,
                        int64_t pool_blocks, const int32_t* block_table, int64_t table_rows,
                        int64_t table_stride, const int32_t* seq, const int32_t* positions,
                        const int64_t* expected, const uint16_t* kv_values,
                        const uint16_t* index_values, uint16_t* swa, int32_t* err, int64_t n,
                        void* stream);

/* Log-sum-exp combine of attention partials: for each (b,h) the T partials
 * (m[b,t,h], l[b,t,h], o[b,t,h,:dv]), m in base-2 units, are merged; with a
 * sink (natural-log units) the result is normalised,
 * out[b,h,:] = sum_t o_t 2^{m_t-M} / (2^{log2(e) sink_h - M} + sum_t l_t 2^{m_t-M}),
 * otherwise (out_m,out_l,out) receive the merged unnormalised partial. */
int dsr_lse_combine(const float* part_o, const float* part_m, const float* part_l,
                    int64_t parts, const float* sink, float* out, float* out_m, float* out_l,
                    int32_t* err, int64_t batch, int64_t heads, int64_t dv, void* stream);

/* One decode step: indexer -> exact top-k -> sparse MLA attention -> combine.
 * Arguments as above; idx_q f32[batch,idx_heads,128], idx_w f32[batch,idx_heads];
 * topk_out i32[batch,k] receives the selection; scores_out (nullable)
 * f32[batch,score_stride].  Scratch: dsr_decode_workspace_bytes() bytes, 256-byte
 * aligned, zero before its first use (every completed call leaves the parts
 * that must start at zero cleared again); calls sharing it must not overlap. */
size_t dsr_decode_workspace_bytes(int64_t batch, int64_t max_visible, int64_t heads,
                                  int64_t k);
/* Kernels one dsr_decode_step (or _ring) call enqueues for this shape on the
 * current device: 1 when every attention tile unit (tile, sequence, head group)
 * gets a CTA of its own, so the attention and the combine run inside the
 * cooperative indexer launch after the selection; else 3 (indexer with the
 * selection, sparse MLA, combine). */
int dsr_decode_step_launches(int64_t batch, int64_t heads, int64_t idx_heads, int64_t k);
int dsr_decode_step(const float* idx_q, const float* idx_w, int64_t idx_heads,
                    const uint16_t* index_pool, const float* q, const uint16_t* kv_pool,
                    int64_t heads, int64_t pool_blocks, const int32_t* block_table,
                    int64_t table_stride, const int32_t* visible, int64_t max_visible,
                    int64_t k, const uint16_t* swa, const int32_t* swa_len,
                    const float* sink, float scale, float* out, int32_t* topk_out,
                    float* scores_out, void* workspace, size_t workspace_bytes,
                    int32_t* err, int64_t batch, void* stream);

/* ---------------------------------------------------------------------------
 * Ring-offset pools: the reference's own pool layout.  The reference keeps one
 * DeviceRowPool per (kind, layer) -- sources (KV rows), index_keys, windows
 * (the 128-row SWA ring) -- each a flat [slots, width] tensor in which logical
 * row p lives at slot (p + offset) % slots, offset = a hash of (run, role,
 * kind, layer) (src/deepseekrpc/cache_pool.py:24-113, bootstrap.py:185-192).
 * These entry points address such pools directly.  Per sequence b a ring
 * descriptor i64[3] = {first row, slots, offset} places its region at rows
 * [first, first + slots) of the pool tensor (first = 0, one sequence per pool,
 * is the reference's case); position p is at row first + (p + offset) % slots.
 * A descriptor is valid when slots > 0, 0 <= offset < slots and
 * first + slots <= the pool's rows; an invalid one, or visible[b] > slots,
 * gives status 1.  Offsets need not be multiples of 64 and a sequence may wrap
 * around the end of its slots.  Everything else is as in the paged forms.
 * ------------------------------------------------------------------------- */

/* dsr_indexer_decode over a ring-offset index-key pool bf16[pool_rows, 128];
 * ring i64[batch][3].  Replaces TiledIndexer.select's per-tile index_scores
 * over DeviceRowPool.physical() slots (index_selection.py:94-107). */
int dsr_indexer_decode_ring(const float* q, const float* weights, const uint16_t* index_pool,
                            int64_t pool_rows, const int64_t* ring, const int32_t* visible,
                            float* scores, int64_t score_stride, int32_t* err, int64_t batch,
                            int64_t heads, void* stream);

/* dsr_sparse_mla_decode over a ring-offset KV pool bf16[kv_rows, 576] (kv_ring
 * i64[batch][3]); the SWA window is the sequence's last swa_len[b] positions,
 * read from an SWA row pool bf16[swa_rows, 576] through swa_ring i64[batch][3]
 * (the reference's 128-slot windows pools: slots 128).  Replaces forward_mqa's
 * staging + physical() translation + sparse_attention (vllm_attention.py:231-262). */
int dsr_sparse_mla_decode_ring(const float* q, const uint16_t* kv_pool, int64_t kv_rows,
                               const int64_t* kv_ring, const int32_t* visible, const int32_t* topk,
                               int64_t k, const uint16_t* swa_pool, int64_t swa_rows,
                               const int64_t* swa_ring, const int32_t* swa_len, const float* sink,
                               float scale, float* out, void* workspace, size_t workspace_bytes,
                               int32_t* err, int64_t batch, int64_t heads, void* stream);

/* dsr_decode_step over ring-offset pools: index keys (index_ring), KV rows
 * (kv_ring) and the SWA window (swa_ring), each pool with its own offsets.
 * Workspace: dsr_decode_workspace_bytes(). */
int dsr_decode_step_ring(const float* idx_q, const float* idx_w, int64_t idx_heads,
                         const uint16_t* index_pool, int64_t index_rows, const int64_t* index_ring,
                         const float* q, const uint16_t* kv_pool, int64_t kv_rows,
                         const int64_t* kv_ring, int64_t heads, const int32_t* visible,
                         int64_t max_visible, int64_t k, const uint16_t* swa_pool, int64_t swa_rows,
                         const int64_t* swa_ring, const int32_t* swa_len, const float* sink,
                         float scale, float* out, int32_t* topk_out, float* scores_out,
                         void* workspace, size_t workspace_bytes, int32_t* err, int64_t batch,
                         void* stream);

/* dsr_append_kv_index over ring-offset pools, each with its own generations:
 * the KV row of (seq[i], positions[i]) goes to kv_pool at its kv_ring row, the
 * index row to index_pool at its index_ring row.  A row is written only if both
 * rows are in bounds, neither repeats an earlier row's target in its pool,
 * kv_generations[kv row] == kv_expected[i], index_generations[index row] ==
 * index_expected[i] and both value rows are finite; then both generations are
 * bumped to expected + 1.  Otherwise status 3 (bounds / repeat / stale) or 2
 * (non-finite) and nothing of that row is written.  Replaces publish_source's
 * two DeviceRowPool.write calls (attention_state.py:183-192); the SWA windows
 * pool stays the caller's (DeviceRowPool.write over dsr_pool_write).
 * sequences = the rows of each ring descriptor array. */
int dsr_append_kv_index_ring(uint16_t* kv_pool, int64_t kv_rows, const int64_t* kv_ring,
                             int64_t* kv_generations, const int64_t* kv_expected,
                             uint16_t* index_pool, int64_t index_rows, const int64_t* index_ring,
                             int64_t* index_generations, const int64_t* index_expected,
                             int64_t sequences, const int32_t* seq, const int32_t* positions,
                             const uint16_t* kv_values, const uint16_t* index_values, int32_t* err,
                             int64_t n, void* stream);

/* ---------------------------------------------------------------------------
 * Row-pool transactions and snapshot row streaming (DeviceRowPool,
 * cache_pool.py:156-360; StageSnapshot._gpu, snapshot_state.py:205-216;
 * snapshot_restore.py:158-165).  data bf16[slots, width] (width <= 576),
 * generations i64[slots], undo bf16[undo_rows, width].  All four are single
 * launches with no host synchronisation; device status in *err:
 * DSR_ERR_SCATTER (bounds / repeated slot / generation mismatch), DSR_ERR_NONFINITE,
 * DSR_ERR_ID (snapshot row not live).
 *  - dsr_pool_write: a batch of 1..64 rows.  The whole batch is checked first;
 *    every in-bounds target row is copied to undo[undo_start + i]; a valid batch
 *    is then written and its generations set to expected + 1, a refused one
 *    writes nothing else (restoring its undo rows leaves the pool unchanged).
 *  - dsr_pool_rollback: `count` rejected mutations in journal order (slot,
 *    previous generation, undo row); each slot ends with the backup of its
 *    earliest rejected mutation (the reference restores newest first).
 *  - dsr_pool_gather: a snapshot tile of 1..1024 logical rows (slot =
 *    (logical + offset) % slots) into out bf16[rows, width]; generations
 *    (nullable) must be live; non-finite payload is refused.
 *  - dsr_pool_restore: a snapshot tile into fresh rows (generation 0, no
 *    repeated slot), generations set to 1; a refused tile writes nothing.
 * ------------------------------------------------------------------------- */
int dsr_pool_write(uint16_t* data, int64_t* generations, int64_t slots, int64_t width,
                   const int32_t* slot_ids, const int64_t* expected, const uint16_t* values,
                   int64_t rows, uint16_t* undo, int64_t undo_rows, int64_t undo_start,
                   int32_t* err, void* stream);
int dsr_pool_rollback(uint16_t* data, int64_t* generations, int64_t slots, int64_t width,
                      const uint16_t* undo, int64_t undo_rows, const int32_t* slot_ids,
                      const int64_t* previous, const int32_t* undo_index, int64_t count,
                      int32_t* err, void* stream);
int dsr_pool_gather(const uint16_t* data, const int64_t* generations, int64_t slots, int64_t width,
                    int64_t offset, const int64_t* logical, int64_t rows, uint16_t* out,
                    int32_t* err, void* stream);
int dsr_pool_restore(uint16_t* data, int64_t* generations, int64_t slots, int64_t width,
                     int64_t offset, const int64_t* logical, const uint16_t* values, int64_t rows,
                     int32_t* err, void* stream);

/* ---------------------------------------------------------------------------
 * NVLink peer exchange for the sequence-sharded step (one process per GPU).
 * Replaces the collective library's all_gather at the two exchange points of a
 * decode step (torch.distributed.all_gather_into_tensor in the reference-style
 * host plumbing): rank r's payload lands in slot r of every rank's exchange
 * buffer through CUDA IPC peer mappings, written with plain stores; arrival
 * counters (system-scope release/acquire) signal completion, and the waiting
 * side gives up after a bounded time with DSR_ERR_TIMEOUT in *err.
 * Buffer layout: 256 control bytes, then world slots of slot_bytes
 * (slot r at byte 256 + r * slot_bytes).  Every rank allocates one buffer per
 * exchange (dsr_p2p_alloc, zeroed), shares the 64-byte IPC handle with its
 * peers, and maps theirs (dsr_p2p_open).  buffers[w] is rank w's buffer as
 * mapped in this process (buffers[rank] the local one); the host array is read
 * at launch.  All ranks must issue the same exchanges in the same order.
 * After DSR_ERR_TIMEOUT the receive slots may hold a mix of steps: every rank
 * frees and re-creates its exchange buffers before the next exchange.
 * ------------------------------------------------------------------------- */
#define DSR_P2P_MAX_WORLD 8
#define DSR_P2P_HANDLE_BYTES 64
size_t dsr_p2p_buffer_bytes(int64_t world, int64_t slot_bytes);
int dsr_p2p_alloc(size_t bytes, void** buffer, uint8_t* ipc_handle);
int dsr_p2p_open(const uint8_t* ipc_handle, void** peer_buffer);
int dsr_p2p_close(void* peer_buffer);
int dsr_p2p_free(void* buffer);
int dsr_p2p_allgather(const void* payload, int64_t payload_bytes, void* const* buffers,
                      int64_t rank, int64_t world, int64_t slot_bytes, int64_t chunks,
                      int32_t* err, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DSR_B200_H */
