// Fused, generation-checked append of new KV (576) and index-key (128) rows into
// the paged pools and the per-sequence SWA ring.
//
// Reference path being fused: publish_source writes the KV source pool and the
// index-key pool with two DeviceRowPool.write calls (attention_state.py:183-192),
// each a checked scatter_slots followed by a generation bump
// (cache_pool.py:299-310, native/operations.cu:144-161); forward_mqa then writes
// the SWA ring (vllm_attention.py:261).  Checks kept: physical bounds, no
// repeated target in one batch (for the SWA ring: no repeated ring row, as the
// reference's 128-slot windows pool refuses), generation equal to the expected
// value, finite BF16 payload.  Difference (documented in the C ABI): a failing
// row writes nothing at all, instead of the reference's element-wise partial
// write, and the rows that pass are written and bumped even when another row of
// the batch fails (the reference bumps a batch only when all of it passed).
#include "common.cuh"
#include "host_common.h"

namespace dsr {
namespace {

__device__ __forceinline__ int64_t physical_row(const int32_t* block_table, int64_t table_stride,
                                                int64_t table_rows, int64_t pool_blocks, int32_t s,
                                                int32_t p) {
  if (s < 0 || s >= table_rows || p < 0 || (p >> 6) >= table_stride) return -1;
  const int64_t blk = block_table[int64_t(s) * table_stride + (p >> 6)];
  if (blk < 0 || blk >= pool_blocks) return -1;
  return blk * 64 + (p & 63);
}

__global__ void __launch_bounds__(128) append_kernel(
    uint16_t* __restrict__ kv_pool, uint16_t* __restrict__ index_pool,
    int64_t* __restrict__ generations, int64_t pool_blocks, const int32_t* __restrict__ block_table,
    int64_t table_stride, int64_t table_rows, const int32_t* __restrict__ seq,
    const int32_t* __restrict__ positions, const int64_t* __restrict__ expected,
    const uint16_t* __restrict__ kv_values, const uint16_t* __restrict__ index_values,
    uint16_t* __restrict__ swa, int32_t* err) {
  __shared__ int reject;
  const int i = blockIdx.x;
  pdl_wait();
  const int32_t s = seq[i], p = positions[i];
  const int64_t row = physical_row(block_table, table_stride, table_rows, pool_blocks, s, p);
  if (threadIdx.x == 0) reject = row < 0 ? DSR_ERR_SCATTER : 0;
  __syncthreads();
  if (row >= 0) {
    // an earlier row of the batch with the same physical row, or (with the SWA
    // ring) the same sequence and ring row p % 128, refuses this one
    for (int j = threadIdx.x; j < i; j += blockDim.x) {
      const int32_t sj = seq[j], pj = positions[j];
      if (physical_row(block_table, table_stride, table_rows, pool_blocks, sj, pj) == row ||
          (swa != nullptr && sj == s && ((pj ^ p) & (DSR_SWA_ROWS - 1)) == 0))
        atomicCAS(&reject, 0, DSR_ERR_SCATTER);
    }
    if (threadIdx.x == 0 && generations[row] != expected[i]) atomicCAS(&reject, 0, DSR_ERR_SCATTER);
  }
  __syncthreads();
  if (reject == 0) {
    const uint16_t* kv = kv_values + int64_t(i) * DSR_KV_DIM;
    const uint16_t* ix = index_values + int64_t(i) * DSR_INDEX_DIM;
    bool bad = false;
    for (int d = threadIdx.x; d < DSR_KV_DIM; d += blockDim.x) bad |= (kv[d] & 0x7f80) == 0x7f80;
    for (int d = threadIdx.x; d < DSR_INDEX_DIM; d += blockDim.x) bad |= (ix[d] & 0x7f80) == 0x7f80;
    if (bad) atomicCAS(&reject, 0, DSR_ERR_NONFINITE);
  }
  __syncthreads();
  if (reject != 0) {
    if (threadIdx.x == 0) flag(err, reject);
    return;
  }
  const uint32_t* kv32 = reinterpret_cast<const uint32_t*>(kv_values + int64_t(i) * DSR_KV_DIM);
  const uint32_t* ix32 = reinterpret_cast<const uint32_t*>(index_values + int64_t(i) * DSR_INDEX_DIM);
  uint32_t* kvd = reinterpret_cast<uint32_t*>(kv_pool + row * DSR_KV_DIM);
  uint32_t* ixd = reinterpret_cast<uint32_t*>(index_pool + row * DSR_INDEX_DIM);
  uint32_t* swd = swa != nullptr
                      ? reinterpret_cast<uint32_t*>(swa + (int64_t(s) * DSR_SWA_ROWS + (p & 127)) * DSR_KV_DIM)
                      : nullptr;
  for (int d = threadIdx.x; d < DSR_KV_DIM / 2; d += blockDim.x) {
    const uint32_t v = kv32[d];
    kvd[d] = v;
    if (swd != nullptr) swd[d] = v;
  }
  for (int d = threadIdx.x; d < DSR_INDEX_DIM / 2; d += blockDim.x) ixd[d] = ix32[d];
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    generations[row] = expected[i] + 1;
  }
  pdl_launch_dependents();
}

}  // namespace
}  // namespace dsr

extern "C" int dsr_append_kv_index(uint16_t* kv_pool, uint16_t* index_pool, int64_t* generations,
                                   int64_t pool_blocks, const int32_t* block_table,
                                   int64_t table_rows, int64_t table_stride, const int32_t* seq,
                                   const int32_t* positions, const int64_t* expected,
                                   const uint16_t* kv_values, const uint16_t* index_values,
                                   uint16_t* swa, int32_t* err, int64_t n, void* stream) {
  using namespace dsr;
  clear_error();
  DSR_REQUIRE(kv_pool && index_pool && generations && block_table && seq && positions && expected &&
                  kv_values && index_values && err,
              "append_kv_index: null pointer");
  DSR_REQUIRE(n > 0 && n <= 4096, "append_kv_index: rows %lld outside [1, 4096]", (long long)n);
  DSR_REQUIRE(pool_blocks > 0 && table_rows > 0 && table_stride > 0,
              "append_kv_index: invalid pool/table");
  DSR_REQUIRE(((reinterpret_cast<uintptr_t>(kv_values) | reinterpret_cast<uintptr_t>(index_values) |
                reinterpret_cast<uintptr_t>(kv_pool) | reinterpret_cast<uintptr_t>(index_pool) |
                reinterpret_cast<uintptr_t>(swa)) & 3u) == 0,
              "append_kv_index: rows must be 4-byte aligned");
  append_kernel<<<unsigned(n), 128, 0, as_stream(stream)>>>(
      kv_pool, index_pool, generations, pool_blocks, block_table, table_stride, table_rows, seq,
      positions, expected, kv_values, index_values, swa, err);
  return launch_status("append_kv_index launch");
}
