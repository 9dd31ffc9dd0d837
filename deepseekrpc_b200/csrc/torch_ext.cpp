// Thin PyTorch extension `deepseekrpc_cuda` over the C ABI of libdsr_b200.so.
//
// The four reference ops keep the names, argument order, return convention and
// TORCH_CHECK validation of native/bindings.cpp:20-26 / native/operations.cu:180-243
// (with the bounds widened to the DeepSeek-V3.2/V4 geometry); abi_version() is 2.
// New entry points expose the paged decode path.  Outputs are allocated with
// the caching allocator on the input's device; work runs on the current stream.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <vector>

#include "dsr_b200.h"

namespace {

void check(const at::Tensor& t, at::ScalarType dtype, const at::Tensor& anchor) {
  TORCH_CHECK(t.is_cuda() && t.device() == anchor.device(), "all inputs require the same CUDA device");
  TORCH_CHECK(t.scalar_type() == dtype && t.is_contiguous(), "input dtype/contiguity mismatch");
}

void check_cache(const at::Tensor& value, const at::Tensor& anchor) {
  TORCH_CHECK(value.scalar_type() == at::kBFloat16, "cache storage must be unquantized BF16");
  check(value, value.scalar_type(), anchor);
}

void ok(int rc) { TORCH_CHECK(rc == DSR_OK, dsr_last_error()); }

void* current_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

const uint16_t* bf16(const at::Tensor& t) { return reinterpret_cast<const uint16_t*>(t.data_ptr()); }
uint16_t* bf16_mut(at::Tensor& t) { return reinterpret_cast<uint16_t*>(t.data_ptr()); }

at::Tensor status_like(const at::Tensor& anchor) {
  return at::zeros({1}, anchor.options().dtype(at::kInt));
}

}  // namespace

// ---------------------------------------------------------------- reference ops

std::vector<at::Tensor> ds_sparse_attention(at::Tensor q, at::Tensor window, at::Tensor source,
                                            at::Tensor indices, at::Tensor sink, double scale) {
  check(q, at::kFloat, q);
  check_cache(window, q);
  check_cache(source, q);
  check(indices, at::kInt, q);
  check(sink, at::kFloat, q);
  TORCH_CHECK(q.dim() == 3 && q.size(0) > 0 && q.size(0) <= 65536 && q.size(1) > 0 && q.size(1) <= 128,
              "invalid bounded query shape");
  const auto width = q.size(2);
  TORCH_CHECK(width > 0 && width <= 576 && window.dim() == 2 && source.dim() == 2 &&
                  window.size(1) == width && source.size(1) == width && window.size(0) <= 65536,
              "KV dimensions/capacity differ from bounded query");
  TORCH_CHECK(indices.dim() == 2 && indices.size(0) == q.size(0) && indices.size(1) <= 65536 &&
                  sink.dim() == 1 && sink.size(0) == q.size(1),
              "invalid sparse indices/sink shape");
  TORCH_CHECK(std::isfinite(static_cast<float>(scale)) && static_cast<float>(scale) > 0.0f,
              "invalid attention scale");
  const c10::cuda::CUDAGuard guard(q.device());
  auto out = at::empty_like(q);
  auto error = status_like(q);
  ok(dsr_sparse_attention(q.data_ptr<float>(), bf16(window), bf16(source), indices.data_ptr<int32_t>(),
                          sink.data_ptr<float>(), out.data_ptr<float>(), error.data_ptr<int32_t>(),
                          q.size(0), q.size(1), width, window.size(0), source.size(0),
                          indices.size(1), static_cast<float>(scale), current_stream()));
  return {out, error};
}

std::vector<at::Tensor> ds_index_scores(at::Tensor q, at::Tensor keys, at::Tensor weights,
                                        at::Tensor indices, at::Tensor visible) {
  check(q, at::kFloat, q);
  check_cache(keys, q);
  check(weights, at::kFloat, q);
  check(indices, at::kInt, q);
  check(visible, at::kInt, q);
  TORCH_CHECK(q.dim() == 3 && q.size(0) > 0 && q.size(0) <= 65536 && q.size(1) > 0 && q.size(1) <= 64 &&
                  q.size(2) == 128 && keys.dim() == 2 && keys.size(1) == 128,
              "invalid index query/key shape");
  TORCH_CHECK(weights.dim() == 2 && weights.size(0) == q.size(0) && weights.size(1) == q.size(1) &&
                  visible.dim() == 1 && visible.size(0) == q.size(0) && indices.dim() == 2 &&
                  indices.size(0) == q.size(0) && indices.size(1) > 0,
              "invalid bounded index tile");
  const c10::cuda::CUDAGuard guard(q.device());
  auto out = at::empty(indices.sizes(), q.options());
  auto error = status_like(q);
  ok(dsr_index_scores(q.data_ptr<float>(), bf16(keys), weights.data_ptr<float>(),
                      indices.data_ptr<int32_t>(), visible.data_ptr<int32_t>(), out.data_ptr<float>(),
                      error.data_ptr<int32_t>(), q.size(0), q.size(1), indices.size(1), keys.size(0),
                      current_stream()));
  return {out, error};
}

std::vector<at::Tensor> ds_engram_decode(at::Tensor encoded) {
  check(encoded, at::kByte, encoded);
  TORCH_CHECK(encoded.dim() == 2 && encoded.size(0) > 0 && encoded.size(0) <= 1024 && encoded.size(1) == 264,
              "encoded Engram rows must be bounded [rows,264] uint8");
  const c10::cuda::CUDAGuard guard(encoded.device());
  auto out = at::empty({encoded.size(0), 256}, encoded.options().dtype(at::kBFloat16));
  auto error = status_like(encoded);
  ok(dsr_engram_decode(encoded.data_ptr<uint8_t>(), bf16_mut(out), error.data_ptr<int32_t>(),
                       encoded.size(0), current_stream()));
  return {out, error};
}

at::Tensor ds_scatter_slots(at::Tensor pool, at::Tensor generations, at::Tensor slots,
                            at::Tensor expected_generations, at::Tensor values) {
  check_cache(pool, pool);
  check(generations, at::kLong, pool);
  check(slots, at::kInt, pool);
  check(expected_generations, at::kLong, pool);
  check_cache(values, pool);
  TORCH_CHECK(pool.dim() == 2 && pool.size(1) > 0 && pool.size(1) <= 576 && generations.dim() == 1 &&
                  generations.size(0) == pool.size(0),
              "invalid cache/generation pool");
  TORCH_CHECK(slots.dim() == 1 && slots.size(0) > 0 && slots.size(0) <= 4096 &&
                  expected_generations.dim() == 1 && expected_generations.size(0) == slots.size(0) &&
                  values.dim() == 2 && values.size(0) == slots.size(0) && values.size(1) == pool.size(1),
              "invalid cache update rows");
  const c10::cuda::CUDAGuard guard(pool.device());
  auto error = status_like(pool);
  ok(dsr_scatter_slots(bf16_mut(pool), generations.data_ptr<int64_t>(), slots.data_ptr<int32_t>(),
                       expected_generations.data_ptr<int64_t>(), bf16(values), error.data_ptr<int32_t>(),
                       slots.size(0), pool.size(1), pool.size(0), current_stream()));
  return error;
}

// ---------------------------------------------------------------- new entry points

std::vector<at::Tensor> ds_topk_select(at::Tensor scores, at::Tensor lengths, int64_t k,
                                       c10::optional<at::Tensor> ids, int64_t id_base,
                                       bool return_scores) {
  check(scores, at::kFloat, scores);
  check(lengths, at::kInt, scores);
  TORCH_CHECK(scores.dim() == 2 && lengths.dim() == 1 && lengths.size(0) == scores.size(0),
              "topk_select: scores [rows, n] and lengths [rows] expected");
  if (ids) {
    check(*ids, at::kInt, scores);
    TORCH_CHECK(ids->sizes() == scores.sizes(), "topk_select: ids must match scores");
  }
  const c10::cuda::CUDAGuard guard(scores.device());
  auto out = at::empty({scores.size(0), k}, scores.options().dtype(at::kInt));
  at::Tensor out_scores = return_scores ? at::empty({scores.size(0), k}, scores.options()) : at::Tensor();
  auto error = status_like(scores);
  const size_t ws_bytes = dsr_topk_workspace_bytes(scores.size(0), scores.size(1));
  auto ws = at::zeros({int64_t(ws_bytes)}, scores.options().dtype(at::kByte));
  ok(dsr_topk_select(scores.data_ptr<float>(), ids ? ids->data_ptr<int32_t>() : nullptr,
                     lengths.data_ptr<int32_t>(), out.data_ptr<int32_t>(),
                     return_scores ? out_scores.data_ptr<float>() : nullptr, error.data_ptr<int32_t>(),
                     scores.size(0), scores.size(1), k, id_base, ws.data_ptr(), ws_bytes,
                     current_stream()));
  if (return_scores) return {out, error, out_scores};
  return {out, error};
}

std::vector<at::Tensor> ds_indexer_decode(at::Tensor q, at::Tensor weights, at::Tensor index_pool,
                                          at::Tensor block_table, at::Tensor visible,
                                          int64_t score_stride) {
  check(q, at::kFloat, q);
  check(weights, at::kFloat, q);
  check_cache(index_pool, q);
  check(block_table, at::kInt, q);
  check(visible, at::kInt, q);
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 128 && weights.dim() == 2 && weights.size(0) == q.size(0) &&
                  weights.size(1) == q.size(1),
              "indexer_decode: q [batch, heads, 128] and weights [batch, heads] expected");
  TORCH_CHECK(index_pool.dim() == 2 && index_pool.size(1) == 128 && index_pool.size(0) % 64 == 0,
              "indexer_decode: index_pool [blocks*64, 128] expected");
  TORCH_CHECK(block_table.dim() == 2 && block_table.size(0) == q.size(0) && visible.dim() == 1 &&
                  visible.size(0) == q.size(0),
              "indexer_decode: block_table [batch, blocks] and visible [batch] expected");
  const c10::cuda::CUDAGuard guard(q.device());
  auto scores = at::empty({q.size(0), score_stride}, q.options());
  auto error = status_like(q);
  ok(dsr_indexer_decode(q.data_ptr<float>(), weights.data_ptr<float>(), bf16(index_pool),
                        index_pool.size(0) / 64, block_table.data_ptr<int32_t>(), block_table.size(1),
                        visible.data_ptr<int32_t>(), scores.data_ptr<float>(), score_stride,
                        error.data_ptr<int32_t>(), q.size(0), q.size(1), current_stream()));
  return {scores, error};
}

std::vector<at::Tensor> ds_sparse_mla_decode(at::Tensor q, at::Tensor kv_pool, at::Tensor block_table,
                                             at::Tensor visible, at::Tensor topk, at::Tensor swa,
                                             at::Tensor swa_len, at::Tensor sink, double scale) {
  check(q, at::kFloat, q);
  check_cache(kv_pool, q);
  check(block_table, at::kInt, q);
  check(visible, at::kInt, q);
  check(topk, at::kInt, q);
  check_cache(swa, q);
  check(swa_len, at::kInt, q);
  check(sink, at::kFloat, q);
  const int64_t batch = q.size(0), heads = q.size(1);
  TORCH_CHECK(q.dim() == 3 && q.size(2) == DSR_KV_DIM, "sparse_mla_decode: q [batch, heads, 576] expected");
  TORCH_CHECK(kv_pool.dim() == 2 && kv_pool.size(1) == DSR_KV_DIM && kv_pool.size(0) % 64 == 0,
              "sparse_mla_decode: kv_pool [blocks*64, 576] expected");
  TORCH_CHECK(block_table.dim() == 2 && block_table.size(0) == batch && topk.dim() == 2 &&
                  topk.size(0) == batch && visible.size(0) == batch && swa_len.size(0) == batch &&
                  swa.dim() == 3 && swa.size(0) == batch && swa.size(1) == DSR_SWA_ROWS &&
                  swa.size(2) == DSR_KV_DIM && sink.dim() == 1 && sink.size(0) == heads,
              "sparse_mla_decode: inconsistent shapes");
  const c10::cuda::CUDAGuard guard(q.device());
  const int64_t k = topk.size(1);
  auto out = at::empty({batch, heads, DSR_V_DIM}, q.options());
  const size_t ws_bytes = dsr_mla_workspace_bytes(batch, heads, k);
  auto ws = at::empty({int64_t(ws_bytes)}, q.options().dtype(at::kByte));
  auto error = status_like(q);
  ok(dsr_sparse_mla_decode(q.data_ptr<float>(), bf16(kv_pool), kv_pool.size(0) / 64,
                           block_table.data_ptr<int32_t>(), block_table.size(1),
                           visible.data_ptr<int32_t>(), topk.data_ptr<int32_t>(), k, bf16(swa),
                           swa_len.data_ptr<int32_t>(), sink.data_ptr<float>(), static_cast<float>(scale),
                           out.data_ptr<float>(), ws.data_ptr(), ws_bytes, error.data_ptr<int32_t>(),
                           batch, heads, current_stream()));
  return {out, error};
}

at::Tensor ds_append_kv_index(at::Tensor kv_pool, at::Tensor index_pool, at::Tensor generations,
                              at::Tensor block_table, at::Tensor seq, at::Tensor positions,
                              at::Tensor expected, at::Tensor kv_values, at::Tensor index_values,
                              c10::optional<at::Tensor> swa) {
  check_cache(kv_pool, kv_pool);
  check_cache(index_pool, kv_pool);
  check(generations, at::kLong, kv_pool);
  check(block_table, at::kInt, kv_pool);
  check(seq, at::kInt, kv_pool);
  check(positions, at::kInt, kv_pool);
  check(expected, at::kLong, kv_pool);
  check_cache(kv_values, kv_pool);
  check_cache(index_values, kv_pool);
  const int64_t n = seq.size(0);
  TORCH_CHECK(kv_pool.dim() == 2 && kv_pool.size(1) == DSR_KV_DIM && index_pool.dim() == 2 &&
                  index_pool.size(1) == DSR_INDEX_DIM && kv_pool.size(0) == index_pool.size(0) &&
                  kv_pool.size(0) % 64 == 0 && generations.dim() == 1 &&
                  generations.size(0) == kv_pool.size(0),
              "append_kv_index: pools [blocks*64, 576/128] and generations [blocks*64] expected");
  TORCH_CHECK(block_table.dim() == 2 && positions.size(0) == n && expected.size(0) == n &&
                  kv_values.dim() == 2 && kv_values.size(0) == n && kv_values.size(1) == DSR_KV_DIM &&
                  index_values.dim() == 2 && index_values.size(0) == n &&
                  index_values.size(1) == DSR_INDEX_DIM,
              "append_kv_index: inconsistent row shapes");
  if (swa) {
    check_cache(*swa, kv_pool);
    TORCH_CHECK(swa->dim() == 3 && swa->size(0) == block_table.size(0) && swa->size(1) == DSR_SWA_ROWS &&
                    swa->size(2) == DSR_KV_DIM,
                "append_kv_index: swa [sequences, 128, 576] expected");
  }
  const c10::cuda::CUDAGuard guard(kv_pool.device());
  auto error = status_like(kv_pool);
  ok(dsr_append_kv_index(bf16_mut(kv_pool), bf16_mut(index_pool), generations.data_ptr<int64_t>(),
                         kv_pool.size(0) / 64, block_table.data_ptr<int32_t>(), block_table.size(0),
                         block_table.size(1), seq.data_ptr<int32_t>(), positions.data_ptr<int32_t>(),
                         expected.data_ptr<int64_t>(), bf16(kv_values), bf16(index_values),
                         swa ? bf16_mut(*swa) : nullptr, error.data_ptr<int32_t>(), n,
                         current_stream()));
  return error;
}

std::vector<at::Tensor> ds_lse_combine(at::Tensor part_o, at::Tensor part_m, at::Tensor part_l,
                                       c10::optional<at::Tensor> sink) {
  check(part_o, at::kFloat, part_o);
  check(part_m, at::kFloat, part_o);
  check(part_l, at::kFloat, part_o);
  TORCH_CHECK(part_o.dim() == 4 && part_m.dim() == 3 && part_l.sizes() == part_m.sizes() &&
                  part_o.size(0) == part_m.size(0) && part_o.size(1) == part_m.size(1) &&
                  part_o.size(2) == part_m.size(2),
              "lse_combine: part_o [batch, parts, heads, dv], part_m/part_l [batch, parts, heads]");
  const int64_t batch = part_o.size(0), parts = part_o.size(1), heads = part_o.size(2), dv = part_o.size(3);
  const c10::cuda::CUDAGuard guard(part_o.device());
  auto out = at::empty({batch, heads, dv}, part_o.options());
  auto error = status_like(part_o);
  if (sink) {
    check(*sink, at::kFloat, part_o);
    TORCH_CHECK(sink->dim() == 1 && sink->size(0) == heads, "lse_combine: sink [heads] expected");
    ok(dsr_lse_combine(part_o.data_ptr<float>(), part_m.data_ptr<float>(), part_l.data_ptr<float>(),
                       parts, sink->data_ptr<float>(), out.data_ptr<float>(), nullptr, nullptr,
                       error.data_ptr<int32_t>(), batch, heads, dv, current_stream()));
    return {out, error};
  }
  auto m = at::empty({batch, heads}, part_o.options());
  auto l = at::empty({batch, heads}, part_o.options());
  ok(dsr_lse_combine(part_o.data_ptr<float>(), part_m.data_ptr<float>(), part_l.data_ptr<float>(), parts,
                     nullptr, out.data_ptr<float>(), m.data_ptr<float>(), l.data_ptr<float>(),
                     error.data_ptr<int32_t>(), batch, heads, dv, current_stream()));
  return {out, m, l, error};
}

std::vector<at::Tensor> ds_decode_step(at::Tensor idx_q, at::Tensor idx_w, at::Tensor index_pool,
                                       at::Tensor q, at::Tensor kv_pool, at::Tensor block_table,
                                       at::Tensor visible, int64_t max_visible, int64_t k, at::Tensor swa,
                                       at::Tensor swa_len, at::Tensor sink, double scale,
                                       bool return_scores) {
  check(idx_q, at::kFloat, q);
  check(idx_w, at::kFloat, q);
  check_cache(index_pool, q);
  check(q, at::kFloat, q);
  check_cache(kv_pool, q);
  check(block_table, at::kInt, q);
  check(visible, at::kInt, q);
  check_cache(swa, q);
  check(swa_len, at::kInt, q);
  check(sink, at::kFloat, q);
  const int64_t batch = q.size(0), heads = q.size(1);
  TORCH_CHECK(idx_q.dim() == 3 && idx_q.size(0) == batch && idx_q.size(2) == 128 && idx_w.dim() == 2 &&
                  idx_w.size(0) == batch && idx_w.size(1) == idx_q.size(1),
              "decode_step: idx_q [batch, idx_heads, 128], idx_w [batch, idx_heads] expected");
  TORCH_CHECK(q.dim() == 3 && q.size(2) == DSR_KV_DIM && kv_pool.size(1) == DSR_KV_DIM &&
                  index_pool.size(1) == DSR_INDEX_DIM && kv_pool.size(0) == index_pool.size(0) &&
                  kv_pool.size(0) % 64 == 0,
              "decode_step: pool geometry mismatch");
  TORCH_CHECK(block_table.dim() == 2 && block_table.size(0) == batch && visible.size(0) == batch &&
                  swa.dim() == 3 && swa.size(0) == batch && swa_len.size(0) == batch &&
                  sink.size(0) == heads,
              "decode_step: inconsistent batch shapes");
  const c10::cuda::CUDAGuard guard(q.device());
  auto out = at::empty({batch, heads, DSR_V_DIM}, q.options());
  auto topk = at::empty({batch, k}, q.options().dtype(at::kInt));
  const int64_t stride = (max_visible + 63) / 64 * 64;
  at::Tensor scores = return_scores ? at::empty({batch, stride}, q.options()) : at::Tensor();
  const size_t ws_bytes = dsr_decode_workspace_bytes(batch, max_visible, heads, k);
  auto ws = at::zeros({int64_t(ws_bytes)}, q.options().dtype(at::kByte));
  auto error = status_like(q);
  ok(dsr_decode_step(idx_q.data_ptr<float>(), idx_w.data_ptr<float>(), idx_q.size(1), bf16(index_pool),
                     q.data_ptr<float>(), bf16(kv_pool), heads, kv_pool.size(0) / 64,
                     block_table.data_ptr<int32_t>(), block_table.size(1), visible.data_ptr<int32_t>(),
                     max_visible, k, bf16(swa), swa_len.data_ptr<int32_t>(), sink.data_ptr<float>(),
                     static_cast<float>(scale), out.data_ptr<float>(), topk.data_ptr<int32_t>(),
                     return_scores ? scores.data_ptr<float>() : nullptr, ws.data_ptr(), ws_bytes,
                     error.data_ptr<int32_t>(), batch, current_stream()));
  if (return_scores) return {out, topk, error, scores};
  return {out, topk, error};
}

// ---- ring-offset pools (the reference's DeviceRowPool layout): rings i64[batch, 3]
void check_ring(const at::Tensor& ring, int64_t batch, const at::Tensor& anchor, const char* what) {
  check(ring, at::kLong, anchor);
  TORCH_CHECK(ring.dim() == 2 && ring.size(0) == batch && ring.size(1) == 3, what,
              ": ring descriptors [batch, 3] = (first row, slots, offset) expected");
}

std::vector<at::Tensor> ds_indexer_decode_ring(at::Tensor q, at::Tensor weights, at::Tensor index_pool,
                                               at::Tensor ring, at::Tensor visible, int64_t score_stride) {
  check(q, at::kFloat, q);
  check(weights, at::kFloat, q);
  check_cache(index_pool, q);
  check(visible, at::kInt, q);
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 128 && weights.dim() == 2 && weights.size(0) == q.size(0) &&
                  weights.size(1) == q.size(1) && index_pool.dim() == 2 && index_pool.size(1) == 128 &&
                  visible.dim() == 1 && visible.size(0) == q.size(0),
              "indexer_decode_ring: q [batch, heads, 128], weights [batch, heads], index_pool [rows, 128], "
              "visible [batch] expected");
  check_ring(ring, q.size(0), q, "indexer_decode_ring");
  const c10::cuda::CUDAGuard guard(q.device());
  auto scores = at::empty({q.size(0), score_stride}, q.options());
  auto error = status_like(q);
  ok(dsr_indexer_decode_ring(q.data_ptr<float>(), weights.data_ptr<float>(), bf16(index_pool),
                             index_pool.size(0), ring.data_ptr<int64_t>(), visible.data_ptr<int32_t>(),
                             scores.data_ptr<float>(), score_stride, error.data_ptr<int32_t>(), q.size(0),
                             q.size(1), current_stream()));
  return {scores, error};
}

std::vector<at::Tensor> ds_sparse_mla_decode_ring(at::Tensor q, at::Tensor kv_pool, at::Tensor kv_ring,
                                                  at::Tensor visible, at::Tensor topk, at::Tensor swa_pool,
                                                  at::Tensor swa_ring, at::Tensor swa_len, at::Tensor sink,
                                                  double scale) {
  check(q, at::kFloat, q);
  check_cache(kv_pool, q);
  check(visible, at::kInt, q);
  check(topk, at::kInt, q);
  check_cache(swa_pool, q);
  check(swa_len, at::kInt, q);
  check(sink, at::kFloat, q);
  const int64_t batch = q.size(0), heads = q.size(1);
  TORCH_CHECK(q.dim() == 3 && q.size(2) == DSR_KV_DIM && kv_pool.dim() == 2 && kv_pool.size(1) == DSR_KV_DIM &&
                  swa_pool.dim() == 2 && swa_pool.size(1) == DSR_KV_DIM && topk.dim() == 2 &&
                  topk.size(0) == batch && visible.size(0) == batch && swa_len.size(0) == batch &&
                  sink.dim() == 1 && sink.size(0) == heads,
              "sparse_mla_decode_ring: inconsistent shapes");
  check_ring(kv_ring, batch, q, "sparse_mla_decode_ring (KV pool)");
  check_ring(swa_ring, batch, q, "sparse_mla_decode_ring (SWA pool)");
  const c10::cuda::CUDAGuard guard(q.device());
  const int64_t k = topk.size(1);
  auto out = at::empty({batch, heads, DSR_V_DIM}, q.options());
  const size_t ws_bytes = dsr_mla_workspace_bytes(batch, heads, k);
  auto ws = at::empty({int64_t(ws_bytes)}, q.options().dtype(at::kByte));
  auto error = status_like(q);
  ok(dsr_sparse_mla_decode_ring(q.data_ptr<float>(), bf16(kv_pool), kv_pool.size(0), kv_ring.data_ptr<int64_t>(),
                                visible.data_ptr<int32_t>(), topk.data_ptr<int32_t>(), k, bf16(swa_pool),
                                swa_pool.size(0), swa_ring.data_ptr<int64_t>(), swa_len.data_ptr<int32_t>(),
                                sink.data_ptr<float>(), static_cast<float>(scale), out.data_ptr<float>(),
                                ws.data_ptr(), ws_bytes, error.data_ptr<int32_t>(), batch, heads,
                                current_stream()));
  return {out, error};
}

std::vector<at::Tensor> ds_decode_step_ring(at::Tensor idx_q, at::Tensor idx_w, at::Tensor index_pool,
                                            at::Tensor index_ring, at::Tensor q, at::Tensor kv_pool,
                                            at::Tensor kv_ring, at::Tensor visible, int64_t max_visible, int64_t k,
                                            at::Tensor swa_pool, at::Tensor swa_ring, at::Tensor swa_len,
                                            at::Tensor sink, double scale, bool return_scores) {
  check(idx_q, at::kFloat, q);
  check(idx_w, at::kFloat, q);
  check_cache(index_pool, q);
  check(q, at::kFloat, q);
  check_cache(kv_pool, q);
  check(visible, at::kInt, q);
  check_cache(swa_pool, q);
  check(swa_len, at::kInt, q);
  check(sink, at::kFloat, q);
  const int64_t batch = q.size(0), heads = q.size(1);
  TORCH_CHECK(idx_q.dim() == 3 && idx_q.size(0) == batch && idx_q.size(2) == 128 && idx_w.dim() == 2 &&
                  idx_w.size(0) == batch && idx_w.size(1) == idx_q.size(1),
              "decode_step_ring: idx_q [batch, idx_heads, 128], idx_w [batch, idx_heads] expected");
  TORCH_CHECK(q.dim() == 3 && q.size(2) == DSR_KV_DIM && kv_pool.dim() == 2 && kv_pool.size(1) == DSR_KV_DIM &&
                  index_pool.dim() == 2 && index_pool.size(1) == DSR_INDEX_DIM && swa_pool.dim() == 2 &&
                  swa_pool.size(1) == DSR_KV_DIM,
              "decode_step_ring: pool geometry mismatch");
  TORCH_CHECK(visible.size(0) == batch && swa_len.size(0) == batch && sink.size(0) == heads,
              "decode_step_ring: inconsistent batch shapes");
  check_ring(index_ring, batch, q, "decode_step_ring (index pool)");
  check_ring(kv_ring, batch, q, "decode_step_ring (KV pool)");
  check_ring(swa_ring, batch, q, "decode_step_ring (SWA pool)");
  const c10::cuda::CUDAGuard guard(q.device());
  auto out = at::empty({batch, heads, DSR_V_DIM}, q.options());
  auto topk = at::empty({batch, k}, q.options().dtype(at::kInt));
  const int64_t stride = (max_visible + 63) / 64 * 64;
  at::Tensor scores = return_scores ? at::empty({batch, stride}, q.options()) : at::Tensor();
  const size_t ws_bytes = dsr_decode_workspace_bytes(batch, max_visible, heads, k);
  auto ws = at::zeros({int64_t(ws_bytes)}, q.options().dtype(at::kByte));
  auto error = status_like(q);
  ok(dsr_decode_step_ring(idx_q.data_ptr<float>(), idx_w.data_ptr<float>(), idx_q.size(1), bf16(index_pool),
                          index_pool.size(0), index_ring.data_ptr<int64_t>(), q.data_ptr<float>(), bf16(kv_pool),
                          kv_pool.size(0), kv_ring.data_ptr<int64_t>(), heads, visible.data_ptr<int32_t>(),
                          max_visible, k, bf16(swa_pool), swa_pool.size(0), swa_ring.data_ptr<int64_t>(),
                          swa_len.data_ptr<int32_t>(), sink.data_ptr<float>(), static_cast<float>(scale),
                          out.data_ptr<float>(), topk.data_ptr<int32_t>(),
                          return_scores ? scores.data_ptr<float>() : nullptr, ws.data_ptr(), ws_bytes,
                          error.data_ptr<int32_t>(), batch, current_stream()));
  if (return_scores) return {out, topk, error, scores};
  return {out, topk, error};
}

at::Tensor ds_append_kv_index_ring(at::Tensor kv_pool, at::Tensor kv_ring, at::Tensor kv_generations,
                                   at::Tensor kv_expected, at::Tensor index_pool, at::Tensor index_ring,
                                   at::Tensor index_generations, at::Tensor index_expected, at::Tensor seq,
                                   at::Tensor positions, at::Tensor kv_values, at::Tensor index_values) {
  check_cache(kv_pool, kv_pool);
  check_cache(index_pool, kv_pool);
  check(kv_generations, at::kLong, kv_pool);
  check(index_generations, at::kLong, kv_pool);
  check(kv_expected, at::kLong, kv_pool);
  check(index_expected, at::kLong, kv_pool);
  check(seq, at::kInt, kv_pool);
  check(positions, at::kInt, kv_pool);
  check_cache(kv_values, kv_pool);
  check_cache(index_values, kv_pool);
  const int64_t n = seq.size(0), sequences = kv_ring.size(0);
  TORCH_CHECK(kv_pool.dim() == 2 && kv_pool.size(1) == DSR_KV_DIM && index_pool.dim() == 2 &&
                  index_pool.size(1) == DSR_INDEX_DIM && kv_generations.dim() == 1 &&
                  kv_generations.size(0) == kv_pool.size(0) && index_generations.dim() == 1 &&
                  index_generations.size(0) == index_pool.size(0),
              "append_kv_index_ring: pools [rows, 576/128] with generations [rows] expected");
  TORCH_CHECK(positions.size(0) == n && kv_expected.size(0) == n && index_expected.size(0) == n &&
                  kv_values.dim() == 2 && kv_values.size(0) == n && kv_values.size(1) == DSR_KV_DIM &&
                  index_values.dim() == 2 && index_values.size(0) == n && index_values.size(1) == DSR_INDEX_DIM,
              "append_kv_index_ring: inconsistent row shapes");
  check_ring(kv_ring, sequences, kv_pool, "append_kv_index_ring (KV pool)");
  check_ring(index_ring, sequences, kv_pool, "append_kv_index_ring (index pool)");
  const c10::cuda::CUDAGuard guard(kv_pool.device());
  auto error = status_like(kv_pool);
  ok(dsr_append_kv_index_ring(bf16_mut(kv_pool), kv_pool.size(0), kv_ring.data_ptr<int64_t>(),
                              kv_generations.data_ptr<int64_t>(), kv_expected.data_ptr<int64_t>(),
                              bf16_mut(index_pool), index_pool.size(0), index_ring.data_ptr<int64_t>(),
                              index_generations.data_ptr<int64_t>(), index_expected.data_ptr<int64_t>(), sequences,
                              seq.data_ptr<int32_t>(), positions.data_ptr<int32_t>(), bf16(kv_values),
                              bf16(index_values), error.data_ptr<int32_t>(), n, current_stream()));
  return error;
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("sparse_attention", &ds_sparse_attention);
  m.def("index_scores", &ds_index_scores);
  m.def("engram_decode", &ds_engram_decode);
  m.def("scatter_slots", &ds_scatter_slots);
  m.def("abi_version", [] { return dsr_abi_version(); });
  m.def("topk_select", &ds_topk_select, py::arg("scores"), py::arg("lengths"), py::arg("k"),
        py::arg("ids") = py::none(), py::arg("id_base") = 0, py::arg("return_scores") = false);
  m.def("indexer_decode", &ds_indexer_decode);
  m.def("sparse_mla_decode", &ds_sparse_mla_decode);
  m.def("append_kv_index", &ds_append_kv_index, py::arg("kv_pool"), py::arg("index_pool"),
        py::arg("generations"), py::arg("block_table"), py::arg("seq"), py::arg("positions"),
        py::arg("expected"), py::arg("kv_values"), py::arg("index_values"), py::arg("swa") = py::none());
  m.def("lse_combine", &ds_lse_combine, py::arg("part_o"), py::arg("part_m"), py::arg("part_l"),
        py::arg("sink") = py::none());
  m.def("decode_step", &ds_decode_step, py::arg("idx_q"), py::arg("idx_w"), py::arg("index_pool"),
        py::arg("q"), py::arg("kv_pool"), py::arg("block_table"), py::arg("visible"),
        py::arg("max_visible"), py::arg("k"), py::arg("swa"), py::arg("swa_len"), py::arg("sink"),
        py::arg("scale"), py::arg("return_scores") = false);
  m.def("indexer_decode_ring", &ds_indexer_decode_ring, py::arg("q"), py::arg("weights"), py::arg("index_pool"),
        py::arg("ring"), py::arg("visible"), py::arg("score_stride"));
  m.def("sparse_mla_decode_ring", &ds_sparse_mla_decode_ring, py::arg("q"), py::arg("kv_pool"),
        py::arg("kv_ring"), py::arg("visible"), py::arg("topk"), py::arg("swa_pool"), py::arg("swa_ring"),
        py::arg("swa_len"), py::arg("sink"), py::arg("scale"));
  m.def("decode_step_ring", &ds_decode_step_ring, py::arg("idx_q"), py::arg("idx_w"), py::arg("index_pool"),
        py::arg("index_ring"), py::arg("q"), py::arg("kv_pool"), py::arg("kv_ring"), py::arg("visible"),
        py::arg("max_visible"), py::arg("k"), py::arg("swa_pool"), py::arg("swa_ring"), py::arg("swa_len"),
        py::arg("sink"), py::arg("scale"), py::arg("return_scores") = false);
  m.def("append_kv_index_ring", &ds_append_kv_index_ring, py::arg("kv_pool"), py::arg("kv_ring"),
        py::arg("kv_generations"), py::arg("kv_expected"), py::arg("index_pool"), py::arg("index_ring"),
        py::arg("index_generations"), py::arg("index_expected"), py::arg("seq"), py::arg("positions"),
        py::arg("kv_values"), py::arg("index_values"));
}
