// One sparse-attention decode step: indexer scores -> exact top-k -> sparse MLA
// attention -> LSE combine.  When the step's attention tiles fit one per SM, a
// single cooperative launch does all four; otherwise the indexer launch (scores
// and top-k) is followed by the MLA and combine kernels, chained with
// programmatic dependent launch so each prologue overlaps its predecessor.
// Replaces, per layer, the host loop of AttentionState.select ->
// TiledIndexer.select (index_selection.py:79-124) followed by forward_mqa's id
// assembly and sparse_attention call (vllm_attention.py:231-262).
#include "common.cuh"
#include "host_common.h"
#include "select.cuh"

namespace {
inline int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }
}  // namespace

extern "C" size_t dsr_decode_workspace_bytes(int64_t batch, int64_t max_visible, int64_t heads,
                                             int64_t k) {
  const int64_t stride = round_up(max_visible > 0 ? max_visible : 1, 64);
  return round_up(int64_t(dsr::select_workspace_bytes(batch, k)), 256) + dsr::select_group_bytes(batch, stride) +
         size_t(batch) * size_t(stride) * 4 + dsr::mla_query_image_bytes(batch, heads) +
         dsr::mla_workspace_bytes(batch, heads, k) + 256;
}

namespace dsr {
namespace {

// The step over any pool addressing: index keys through `ix`, KV rows through
// `kv`, the SWA window from the [batch, 128, 576] ring (swa_ring == nullptr) or
// from an SWA row pool through swa_ring.
int decode_step(const float* idx_q, const float* idx_w, int64_t idx_heads, const uint16_t* index_pool,
                const PoolAddr& ix, const float* q, const uint16_t* kv_pool, const PoolAddr& kv, int64_t heads,
                const int32_t* visible, int64_t max_visible, int64_t k, const uint16_t* swa,
                const int64_t* swa_ring, int64_t swa_rows, const int32_t* swa_len, const float* sink, float scale,
                float* out, int32_t* topk_out, float* scores_out, void* workspace, size_t workspace_bytes,
                int32_t* err, int64_t batch, void* stream) {
  DSR_REQUIRE(workspace != nullptr, "decode_step: workspace is required");
  DSR_REQUIRE(scores_out == nullptr || aligned16(scores_out), "decode_step: scores_out must be 16-byte aligned");
  DSR_REQUIRE(max_visible > 0 && max_visible <= (int64_t(1) << 31) - 64,
              "decode_step: max_visible %lld outside [1, 2^31 - 64]", (long long)max_visible);
  const size_t need = dsr_decode_workspace_bytes(batch, max_visible, heads, k);
  DSR_REQUIRE(workspace_bytes >= need, "decode_step: workspace %zu < %zu bytes", workspace_bytes,
              need);
  DSR_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255u) == 0,
              "decode_step: workspace must be 256-byte aligned");
  const int64_t stride = round_up(max_visible, 64);
  // [selection state (zero between calls) | group maxima | scores | MLA query image | MLA partials]
  uint8_t* sel_ws = static_cast<uint8_t*>(workspace);
  const size_t sel_bytes = size_t(round_up(int64_t(select_workspace_bytes(batch, k)), 256));
  const size_t group_bytes = select_group_bytes(batch, stride);
  uint8_t* ws = sel_ws + sel_bytes + group_bytes;
  workspace_bytes -= sel_bytes + group_bytes;
  float* scores = scores_out != nullptr ? scores_out : reinterpret_cast<float*>(ws);
  uint16_t* q_img = reinterpret_cast<uint16_t*>(ws + size_t(batch) * stride * 4);
  uint8_t* mla_ws = ws + size_t(batch) * stride * 4 + mla_query_image_bytes(batch, heads);
  const size_t mla_bytes =
      workspace_bytes - size_t(batch) * stride * 4 - mla_query_image_bytes(batch, heads);
  const cudaStream_t s = as_stream(stream);
  SelectArgs sel;
  int rc = select_args(&sel, sel_ws, batch, k, 0, topk_out, nullptr);
  if (rc != DSR_OK) return rc;
  sel.gmax = reinterpret_cast<uint16_t*>(sel_ws + sel_bytes);
  sel.gstride = select_group_stride(stride);
  // When every attention tile unit gets a CTA of its own, one cooperative launch
  // does the whole step: scores, exact top-k, attention tiles and combine.
  // Otherwise the indexer launch scores, selects and converts the MLA query into
  // the BF16 image the MLA kernels load, and those follow.
  MlaFuseLaunch plan;  // launch parameters are copied at the launch
  rc = plan_fused_mla(&plan, indexer_attention_room(idx_heads), q, kv_pool, kv, visible, topk_out, swa, swa_ring,
                      swa_rows, swa_len, sink, scale, out, mla_ws, mla_bytes, err, batch, heads, k);
  if (rc != DSR_OK) return rc;
  if (plan.args.units > 0)
    return launch_indexer_decode(idx_q, idx_w, index_pool, ix, visible, scores, stride, err, batch, idx_heads, s,
                                 false, nullptr, nullptr, 0, nullptr, &sel, &plan);
  rc = launch_indexer_decode(idx_q, idx_w, index_pool, ix, visible, scores, stride, err, batch, idx_heads, s,
                             false, q, q_img, heads, nullptr, &sel);
  if (rc != DSR_OK) return rc;
  return launch_mla_decode(q, kv_pool, kv, visible, topk_out, k, swa, swa_ring, swa_rows, swa_len, sink, scale,
                           out, mla_ws, mla_bytes, err, batch, heads, s, true, q_img);
}

}  // namespace
}  // namespace dsr

extern "C" int dsr_decode_step_launches(int64_t batch, int64_t heads, int64_t idx_heads, int64_t k) {
  const int units = dsr::fused_mla_units(dsr::indexer_attention_room(idx_heads), batch, heads, k);
  return units > 0 ? 1 : 3;
}

extern "C" int dsr_decode_step(const float* idx_q, const float* idx_w, int64_t idx_heads,
                               const uint16_t* index_pool, const float* q,
                               const uint16_t* kv_pool, int64_t heads, int64_t pool_blocks,
                               const int32_t* block_table, int64_t table_stride,
                               const int32_t* visible, int64_t max_visible, int64_t k,
                               const uint16_t* swa, const int32_t* swa_len, const float* sink,
                               float scale, float* out, int32_t* topk_out, float* scores_out,
                               void* workspace, size_t workspace_bytes, int32_t* err,
                               int64_t batch, void* stream) {
  using namespace dsr;
  clear_error();
  PoolAddr pa;
  const int rc = paged_addr(&pa, block_table, table_stride, pool_blocks, "decode_step");
  if (rc != DSR_OK) return rc;
  DSR_REQUIRE(max_visible <= table_stride * 64, "decode_step: max_visible %lld beyond the table capacity %lld",
              (long long)max_visible, (long long)(table_stride * 64));
  return decode_step(idx_q, idx_w, idx_heads, index_pool, pa, q, kv_pool, pa, heads, visible, max_visible, k, swa,
                     nullptr, 0, swa_len, sink, scale, out, topk_out, scores_out, workspace, workspace_bytes, err,
                     batch, stream);
}

extern "C" int dsr_decode_step_ring(const float* idx_q, const float* idx_w, int64_t idx_heads,
                                    const uint16_t* index_pool, int64_t index_rows, const int64_t* index_ring,
                                    const float* q, const uint16_t* kv_pool, int64_t kv_rows,
                                    const int64_t* kv_ring, int64_t heads, const int32_t* visible,
                                    int64_t max_visible, int64_t k, const uint16_t* swa_pool, int64_t swa_rows,
                                    const int64_t* swa_ring, const int32_t* swa_len, const float* sink,
                                    float scale, float* out, int32_t* topk_out, float* scores_out,
                                    void* workspace, size_t workspace_bytes, int32_t* err, int64_t batch,
                                    void* stream) {
  using namespace dsr;
  clear_error();
  PoolAddr ix, kv;
  int rc = ring_addr(&ix, index_ring, index_rows, "decode_step_ring (index pool)");
  if (rc != DSR_OK) return rc;
  rc = ring_addr(&kv, kv_ring, kv_rows, "decode_step_ring (KV pool)");
  if (rc != DSR_OK) return rc;
  DSR_REQUIRE(swa_ring != nullptr, "decode_step_ring: null SWA ring descriptors");
  return decode_step(idx_q, idx_w, idx_heads, index_pool, ix, q, kv_pool, kv, heads, visible, max_visible, k,
                     swa_pool, swa_ring, swa_rows, swa_len, sink, scale, out, topk_out, scores_out, workspace,
                     workspace_bytes, err, batch, stream);
}

// Indexer scores -> exact top-k with the scores of the chosen entries, the
// indexer's histogram handed to the top-k kernel and the two launches chained by
// programmatic dependent launch (the per-shard selection of sequence-sharded
// decode, and the dense TiledIndexer.select of index_selection.py:79-124).
extern "C" size_t dsr_indexer_topk_workspace_bytes(int64_t batch, int64_t max_visible) {
  const int64_t stride = round_up(max_visible > 0 ? max_visible : 1, 64);
  return round_up(int64_t(dsr::select_workspace_bytes(batch, 8192)), 256) + dsr::select_group_bytes(batch, stride) +
         size_t(batch) * size_t(stride) * 4 + 256;
}

extern "C" int dsr_indexer_topk_decode(const float* idx_q, const float* idx_w, int64_t idx_heads,
                                       const uint16_t* index_pool, int64_t pool_blocks,
                                       const int32_t* block_table, int64_t table_stride,
                                       const int32_t* visible, int64_t max_visible, int64_t k,
                                       int64_t id_base, int32_t* out_ids, float* out_scores,
                                       float* scores_out, void* workspace, size_t workspace_bytes,
                                       int32_t* err, int64_t batch, void* stream) {
  using namespace dsr;
  clear_error();
  DSR_REQUIRE(workspace != nullptr, "indexer_topk: workspace is required");
  DSR_REQUIRE(scores_out == nullptr || aligned16(scores_out), "indexer_topk: scores_out must be 16-byte aligned");
  DSR_REQUIRE(max_visible > 0 && max_visible <= table_stride * 64,
              "indexer_topk: max_visible %lld outside [1, table capacity %lld]",
              (long long)max_visible, (long long)(table_stride * 64));
  const size_t need = dsr_indexer_topk_workspace_bytes(batch, max_visible);
  DSR_REQUIRE(workspace_bytes >= need, "indexer_topk: workspace %zu < %zu bytes", workspace_bytes,
              need);
  DSR_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255u) == 0,
              "indexer_topk: workspace must be 256-byte aligned");
  DSR_REQUIRE(id_base >= 0 && id_base + max_visible < (int64_t(1) << 31) - 1,
              "indexer_topk: id_base %lld + visible keys exceed int32 ids", (long long)id_base);
  const int64_t stride = round_up(max_visible, 64);
  // [selection state (zero between calls) | group maxima | scores]
  uint8_t* sel_ws = static_cast<uint8_t*>(workspace);
  const size_t sel_bytes = size_t(round_up(int64_t(select_workspace_bytes(batch, 8192)), 256));
  const size_t group_bytes = select_group_bytes(batch, stride);
  float* scores =
      scores_out != nullptr ? scores_out : reinterpret_cast<float*>(sel_ws + sel_bytes + group_bytes);
  const cudaStream_t s = as_stream(stream);
  PoolAddr pa;
  int rc = paged_addr(&pa, block_table, table_stride, pool_blocks, "indexer_topk");
  if (rc != DSR_OK) return rc;
  SelectArgs sel;
  rc = select_args(&sel, sel_ws, batch, k, id_base, out_ids, out_scores);
  if (rc != DSR_OK) return rc;
  sel.gmax = reinterpret_cast<uint16_t*>(sel_ws + sel_bytes);
  sel.gstride = select_group_stride(stride);
  return launch_indexer_decode(idx_q, idx_w, index_pool, pa, visible, scores, stride, err, batch, idx_heads, s,
                               false, nullptr, nullptr, 0, nullptr, &sel);
}
