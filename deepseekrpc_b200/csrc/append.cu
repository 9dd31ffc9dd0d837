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

// Target rows of one appended row in the KV and the index pool (-1: outside).
__device__ __forceinline__ void append_rows(const PoolAddr& kv, const PoolAddr& ix, int64_t nseq, int32_t s,
                                            int32_t p, int64_t& kv_row, int64_t& ix_row) {
  kv_row = ix_row = -1;
  if (s < 0 || s >= nseq || p < 0) return;
  kv_row = addr_row(kv, s, p);
  ix_row = addr_row(ix, s, p);
  if (kv_row >= kv.rows) kv_row = -1;
  if (ix_row >= ix.rows) ix_row = -1;
}

// One CTA per appended row.  Paged mode: both pools share the block table and one
// generation per physical row (ix_gens == nullptr).  Ring mode: each pool has its
// own ring, generations and expected values, as the reference's source and
// index-key pools do.
__global__ void __launch_bounds__(128) append_kernel(
    uint16_t* __restrict__ kv_pool, const PoolAddr kv, int64_t* __restrict__ kv_gens,
    const int64_t* __restrict__ kv_expected, uint16_t* __restrict__ index_pool, const PoolAddr ix,
    int64_t* __restrict__ ix_gens, const int64_t* __restrict__ ix_expected, int64_t nseq,
    const int32_t* __restrict__ seq, const int32_t* __restrict__ positions,
    const uint16_t* __restrict__ kv_values, const uint16_t* __restrict__ index_values,
    uint16_t* __restrict__ swa, int32_t* err) {
  __shared__ int reject;
  const int i = blockIdx.x;
  pdl_wait();
  const int32_t s = seq[i], p = positions[i];
  int64_t kv_row, ix_row;
  append_rows(kv, ix, nseq, s, p, kv_row, ix_row);
  const bool in = kv_row >= 0 && ix_row >= 0;
  if (threadIdx.x == 0) reject = in ? 0 : DSR_ERR_SCATTER;
  __syncthreads();
  if (in) {
    // an earlier row of the batch with the same target row in either pool, or
    // (with the SWA ring) the same sequence and ring row p % 128, refuses this one
    for (int j = threadIdx.x; j < i; j += blockDim.x) {
      const int32_t sj = seq[j], pj = positions[j];
      int64_t kj, ij;
      append_rows(kv, ix, nseq, sj, pj, kj, ij);
      if ((kj >= 0 && kj == kv_row) || (ij >= 0 && ij == ix_row) ||
          (swa != nullptr && sj == s && ((pj ^ p) & (DSR_SWA_ROWS - 1)) == 0))
        atomicCAS(&reject, 0, DSR_ERR_SCATTER);
    }
    if (threadIdx.x == 0 && kv_gens[kv_row] != kv_expected[i]) atomicCAS(&reject, 0, DSR_ERR_SCATTER);
    if (threadIdx.x == 0 && ix_gens != nullptr && ix_gens[ix_row] != ix_expected[i])
      atomicCAS(&reject, 0, DSR_ERR_SCATTER);
  }
  __syncthreads();
  if (reject == 0) {
    const uint16_t* kvv = kv_values + int64_t(i) * DSR_KV_DIM;
    const uint16_t* ixv = index_values + int64_t(i) * DSR_INDEX_DIM;
    bool bad = false;
    for (int d = threadIdx.x; d < DSR_KV_DIM; d += blockDim.x) bad |= (kvv[d] & 0x7f80) == 0x7f80;
    for (int d = threadIdx.x; d < DSR_INDEX_DIM; d += blockDim.x) bad |= (ixv[d] & 0x7f80) == 0x7f80;
    if (bad) atomicCAS(&reject, 0, DSR_ERR_NONFINITE);
  }
  __syncthreads();
  if (reject != 0) {
    if (threadIdx.x == 0) flag(err, reject);
    return;
  }
  const uint32_t* kv32 = reinterpret_cast<const uint32_t*>(kv_values + int64_t(i) * DSR_KV_DIM);
  const uint32_t* ix32 = reinterpret_cast<const uint32_t*>(index_values + int64_t(i) * DSR_INDEX_DIM);
  uint32_t* kvd = reinterpret_cast<uint32_t*>(kv_pool + kv_row * DSR_KV_DIM);
  uint32_t* ixd = reinterpret_cast<uint32_t*>(index_pool + ix_row * DSR_INDEX_DIM);
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
    kv_gens[kv_row] = kv_expected[i] + 1;
    if (ix_gens != nullptr) ix_gens[ix_row] = ix_expected[i] + 1;
  }
  pdl_launch_dependents();
}

int launch_append(uint16_t* kv_pool, const PoolAddr& kv, int64_t* kv_gens, const int64_t* kv_expected,
                  uint16_t* index_pool, const PoolAddr& ix, int64_t* ix_gens, const int64_t* ix_expected,
                  int64_t nseq, const int32_t* seq, const int32_t* positions, const uint16_t* kv_values,
                  const uint16_t* index_values, uint16_t* swa, int32_t* err, int64_t n, void* stream,
                  const char* what) {
  DSR_REQUIRE(kv_pool && index_pool && kv_gens && kv_expected && seq && positions && kv_values && index_values &&
                  err,
              "%s: null pointer", what);
  DSR_REQUIRE(n > 0 && n <= 4096, "%s: rows %lld outside [1, 4096]", what, (long long)n);
  DSR_REQUIRE(nseq > 0, "%s: no sequences", what);
  DSR_REQUIRE(((reinterpret_cast<uintptr_t>(kv_values) | reinterpret_cast<uintptr_t>(index_values) |
                reinterpret_cast<uintptr_t>(kv_pool) | reinterpret_cast<uintptr_t>(index_pool) |
                reinterpret_cast<uintptr_t>(swa)) & 3u) == 0,
              "%s: rows must be 4-byte aligned", what);
  append_kernel<<<unsigned(n), 128, 0, as_stream(stream)>>>(kv_pool, kv, kv_gens, kv_expected, index_pool, ix,
                                                            ix_gens, ix_expected, nseq, seq, positions, kv_values,
                                                            index_values, swa, err);
  return launch_status("append launch");
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
  PoolAddr pa;
  const int rc = paged_addr(&pa, block_table, table_stride, pool_blocks, "append_kv_index");
  if (rc != DSR_OK) return rc;
  DSR_REQUIRE(table_rows > 0, "append_kv_index: invalid pool/table");
  return launch_append(kv_pool, pa, generations, expected, index_pool, pa, nullptr, nullptr, table_rows, seq,
                       positions, kv_values, index_values, swa, err, n, stream, "append_kv_index");
}

extern "C" int dsr_append_kv_index_ring(uint16_t* kv_pool, int64_t kv_rows, const int64_t* kv_ring,
                                        int64_t* kv_generations, const int64_t* kv_expected,
                                        uint16_t* index_pool, int64_t index_rows, const int64_t* index_ring,
                                        int64_t* index_generations, const int64_t* index_expected,
                                        int64_t sequences, const int32_t* seq, const int32_t* positions,
                                        const uint16_t* kv_values, const uint16_t* index_values, int32_t* err,
                                        int64_t n, void* stream) {
  using namespace dsr;
  clear_error();
  PoolAddr kv, ix;
  int rc = ring_addr(&kv, kv_ring, kv_rows, "append_kv_index_ring (KV pool)");
  if (rc != DSR_OK) return rc;
  rc = ring_addr(&ix, index_ring, index_rows, "append_kv_index_ring (index pool)");
  if (rc != DSR_OK) return rc;
  DSR_REQUIRE(index_generations && index_expected, "append_kv_index_ring: null pointer");
  return launch_append(kv_pool, kv, kv_generations, kv_expected, index_pool, ix, index_generations, index_expected,
                       sequences, seq, positions, kv_values, index_values, nullptr, err, n, stream,
                       "append_kv_index_ring");
}
