// Device transactions of a BF16 row pool (the reference's DeviceRowPool,
// cache_pool.py:156-360) and the snapshot row streaming by logical id
// (snapshot_state.py:205-216, snapshot_restore.py:158-165).
//
//   pool_write_kernel     one batch of <= 64 rows (DeviceRowPool.write, cache_pool.py:289-310):
//                         the whole batch is validated first (physical bounds, no repeated
//                         slot, generation == expected, finite BF16 payload), every in-bounds
//                         target row is copied into the undo log, and only a valid batch is
//                         written and its generations bumped (expected + 1).  One launch, no
//                         host synchronisation; a refused batch writes nothing but its backup,
//                         so the reference's recovery (finish with nothing accepted) restores
//                         the unchanged rows.
//   pool_rollback_kernel  rejected mutations in journal order (DeviceRowPool.finish,
//                         cache_pool.py:336-352): the reference restores them newest first, so
//                         a slot ends with the backup and previous generation of its EARLIEST
//                         rejected mutation; here each mutation restores only if no earlier
//                         rejected one names the same slot, all in parallel.
//   pool_gather_kernel    snapshot tile: rows of logical ids (slot = (logical + offset) % slots)
//                         into a contiguous [n, width] tile, a live generation required and
//                         non-finite payload refused (StageSnapshot._gpu).
//   pool_restore_kernel   snapshot restore tile into fresh rows (DeviceRowPool.restore_rows,
//                         cache_pool.py:255-274): slots unique and generation 0, then the
//                         rows are written and their generations set to 1.
// Status codes: DSR_ERR_SCATTER for bounds / repeats / generation mismatches (as the
// reference's scatter), DSR_ERR_NONFINITE for non-finite payload, DSR_ERR_ID for a
// snapshot row that is not live.
#include "common.cuh"
#include "host_common.h"

namespace dsr {
namespace {

constexpr int kPoolThreads = 512;
constexpr int kPoolMaxWrite = 64;      // rows per write batch (cache_pool.py:74)
constexpr int kPoolMaxRestore = 1024;  // rows per snapshot tile (snapshot_state.py:207)
constexpr int kPoolMaxWidth = 576;
constexpr int kPoolMaxRollback = 4096;  // undo capacity bound (cache_pool.py:31)

__device__ __forceinline__ bool bf16_nonfinite(uint16_t v) { return (v & 0x7f80u) == 0x7f80u; }

// Copies `width` BF16 values; 16-byte pieces when every row start is 16-byte aligned.
__device__ __forceinline__ void copy_row(uint16_t* dst, const uint16_t* src, int width, bool vec) {
  if (vec) {
    for (int d = threadIdx.x; d < width / 8; d += blockDim.x)
      reinterpret_cast<uint4*>(dst)[d] = reinterpret_cast<const uint4*>(src)[d];
  } else {
    for (int d = threadIdx.x; d < width; d += blockDim.x) dst[d] = src[d];
  }
}

__global__ void __launch_bounds__(kPoolThreads) pool_write_kernel(
    uint16_t* __restrict__ data, int64_t* __restrict__ generations, int64_t slots, int width,
    const int32_t* __restrict__ slot_ids, const int64_t* __restrict__ expected,
    const uint16_t* __restrict__ values, uint16_t* __restrict__ undo, int64_t undo_start, int n,
    bool vec, int32_t* err) {
  __shared__ int32_t sl[kPoolMaxWrite];
  __shared__ int reject;
  pdl_wait();
  if (threadIdx.x == 0) reject = 0;
  if (threadIdx.x < n) sl[threadIdx.x] = slot_ids[threadIdx.x];
  __syncthreads();
  // ---- the whole batch first: bounds, repeats, generations, payload
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int32_t s = sl[i];
    bool bad = s < 0 || s >= slots;
    for (int j = 0; j < i && !bad; ++j) bad = sl[j] == s;
    if (!bad) bad = generations[s] != expected[i];
    if (bad) atomicCAS(&reject, 0, DSR_ERR_SCATTER);
  }
  bool nonfinite = false;
  for (int64_t e = threadIdx.x; e < int64_t(n) * width; e += blockDim.x) nonfinite |= bf16_nonfinite(values[e]);
  if (nonfinite) atomicCAS(&reject, 0, DSR_ERR_NONFINITE);
  __syncthreads();
  // ---- undo backup of every in-bounds target row (always: a refused batch is
  // recovered by restoring its rows, which must then hold their current bytes)
  for (int i = 0; i < n; ++i) {
    const int32_t s = sl[i];
    if (s >= 0 && s < slots)
      copy_row(undo + (undo_start + i) * width, data + int64_t(s) * width, width, vec);
  }
  __syncthreads();
  if (reject != 0) {
    if (threadIdx.x == 0) flag(err, reject);
    return;
  }
  // ---- the batch
  for (int i = 0; i < n; ++i) copy_row(data + int64_t(sl[i]) * width, values + int64_t(i) * width, width, vec);
  for (int i = threadIdx.x; i < n; i += blockDim.x) generations[sl[i]] = expected[i] + 1;
}

__global__ void __launch_bounds__(kPoolThreads) pool_rollback_kernel(
    uint16_t* __restrict__ data, int64_t* __restrict__ generations, int64_t slots, int width,
    const uint16_t* __restrict__ undo, int64_t undo_rows, const int32_t* __restrict__ slot_ids,
    const int64_t* __restrict__ previous, const int32_t* __restrict__ undo_index, int m, bool vec,
    int32_t* err) {
  __shared__ int restore;
  pdl_wait();
  const int i = blockIdx.x;
  const int32_t s = slot_ids[i];
  const int32_t u = undo_index[i];
  if (threadIdx.x == 0) restore = (s >= 0 && s < slots && u >= 0 && u < undo_rows) ? 1 : -1;
  __syncthreads();
  if (restore < 0) {
    if (threadIdx.x == 0) flag(err, DSR_ERR_SCATTER);
    return;
  }
  // an earlier rejected mutation of the same slot holds the older state
  for (int j = threadIdx.x; j < i; j += blockDim.x)
    if (slot_ids[j] == s) restore = 0;
  __syncthreads();
  if (!restore) return;
  copy_row(data + int64_t(s) * width, undo + int64_t(u) * width, width, vec);
  if (threadIdx.x == 0) generations[s] = previous[i];
}

__global__ void __launch_bounds__(256) pool_gather_kernel(
    const uint16_t* __restrict__ data, const int64_t* __restrict__ generations, int64_t slots,
    int width, int64_t offset, const int64_t* __restrict__ logical, uint16_t* __restrict__ out,
    bool vec, int32_t* err) {
  __shared__ int bad;
  pdl_wait();
  const int i = blockIdx.x;
  const int64_t lg = logical[i];
  const int64_t s = lg >= 0 ? (lg + offset) % slots : -1;
  if (threadIdx.x == 0) bad = (s < 0 || (generations != nullptr && generations[s] <= 0)) ? DSR_ERR_ID : 0;
  __syncthreads();
  if (bad) {
    if (threadIdx.x == 0) flag(err, bad);
    return;
  }
  const uint16_t* src = data + s * width;
  uint16_t* dst = out + int64_t(i) * width;
  bool nonfinite = false;
  for (int d = threadIdx.x; d < width; d += blockDim.x) {
    const uint16_t v = src[d];
    nonfinite |= bf16_nonfinite(v);
    dst[d] = v;
  }
  (void)vec;
  if (nonfinite) flag(err, DSR_ERR_NONFINITE);
}

__global__ void __launch_bounds__(kPoolThreads) pool_restore_kernel(
    uint16_t* __restrict__ data, int64_t* __restrict__ generations, int64_t slots, int width,
    int64_t offset, const int64_t* __restrict__ logical, const uint16_t* __restrict__ values, int n,
    bool vec, int32_t* err) {
  __shared__ int64_t sl[kPoolMaxRestore];
  __shared__ int reject;
  pdl_wait();
  if (threadIdx.x == 0) reject = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int64_t lg = logical[i];
    sl[i] = lg >= 0 ? (lg + offset) % slots : -1;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int64_t s = sl[i];
    bool bad = s < 0 || generations[s] != 0;
    for (int j = 0; j < i && !bad; ++j) bad = sl[j] == s;
    if (bad) atomicCAS(&reject, 0, DSR_ERR_SCATTER);
  }
  __syncthreads();
  if (reject != 0) {
    if (threadIdx.x == 0) flag(err, reject);
    return;
  }
  for (int i = 0; i < n; ++i) copy_row(data + sl[i] * width, values + int64_t(i) * width, width, vec);
  for (int i = threadIdx.x; i < n; i += blockDim.x) generations[sl[i]] = 1;
}

bool rows_vec(int width, const void* a, const void* b, const void* c) {
  const uintptr_t m = reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                      reinterpret_cast<uintptr_t>(c);
  return width % 8 == 0 && (m & 15u) == 0;
}

}  // namespace
}  // namespace dsr

extern "C" int dsr_pool_write(uint16_t* data, int64_t* generations, int64_t slots, int64_t width,
                              const int32_t* slot_ids, const int64_t* expected, const uint16_t* values,
                              int64_t rows, uint16_t* undo, int64_t undo_rows, int64_t undo_start,
                              int32_t* err, void* stream) {
  dsr::clear_error();
  DSR_REQUIRE(data && generations && slot_ids && expected && values && undo && err, "pool_write: null pointer");
  DSR_REQUIRE(slots > 0 && slots <= (int64_t(1) << 31) - 1, "pool_write: slots outside [1, 2^31)");
  DSR_REQUIRE(width > 0 && width <= dsr::kPoolMaxWidth, "pool_write: width outside [1, 576]");
  DSR_REQUIRE(rows >= 1 && rows <= dsr::kPoolMaxWrite, "pool_write: batch of %lld rows outside [1, 64]",
              (long long)rows);
  DSR_REQUIRE(undo_start >= 0 && undo_start + rows <= undo_rows, "pool_write: undo log capacity exhausted");
  const bool vec = dsr::rows_vec(int(width), data, values, undo);
  dsr::pool_write_kernel<<<1, dsr::kPoolThreads, 0, dsr::as_stream(stream)>>>(
      data, generations, slots, int(width), slot_ids, expected, values, undo, undo_start, int(rows), vec, err);
  return dsr::launch_status("pool_write launch");
}

extern "C" int dsr_pool_rollback(uint16_t* data, int64_t* generations, int64_t slots, int64_t width,
                                 const uint16_t* undo, int64_t undo_rows, const int32_t* slot_ids,
                                 const int64_t* previous, const int32_t* undo_index, int64_t count,
                                 int32_t* err, void* stream) {
  dsr::clear_error();
  DSR_REQUIRE(data && generations && undo && err, "pool_rollback: null pointer");
  DSR_REQUIRE(width > 0 && width <= dsr::kPoolMaxWidth, "pool_rollback: width outside [1, 576]");
  DSR_REQUIRE(count >= 0 && count <= dsr::kPoolMaxRollback, "pool_rollback: count outside [0, 4096]");
  if (count == 0) return DSR_OK;
  DSR_REQUIRE(slot_ids && previous && undo_index, "pool_rollback: null mutation arrays");
  const bool vec = dsr::rows_vec(int(width), data, undo, undo);
  dsr::pool_rollback_kernel<<<unsigned(count), 256, 0, dsr::as_stream(stream)>>>(
      data, generations, slots, int(width), undo, undo_rows, slot_ids, previous, undo_index, int(count), vec, err);
  return dsr::launch_status("pool_rollback launch");
}

extern "C" int dsr_pool_gather(const uint16_t* data, const int64_t* generations, int64_t slots, int64_t width,
                               int64_t offset, const int64_t* logical, int64_t rows, uint16_t* out,
                               int32_t* err, void* stream) {
  dsr::clear_error();
  DSR_REQUIRE(data && logical && out && err, "pool_gather: null pointer");
  DSR_REQUIRE(slots > 0 && width > 0 && width <= dsr::kPoolMaxWidth && offset >= 0 && offset < slots,
              "pool_gather: invalid pool geometry");
  DSR_REQUIRE(rows >= 1 && rows <= dsr::kPoolMaxRestore, "pool_gather: tile of %lld rows outside [1, 1024]",
              (long long)rows);
  dsr::pool_gather_kernel<<<unsigned(rows), 256, 0, dsr::as_stream(stream)>>>(
      data, generations, slots, int(width), offset, logical, out, false, err);
  return dsr::launch_status("pool_gather launch");
}

extern "C" int dsr_pool_restore(uint16_t* data, int64_t* generations, int64_t slots, int64_t width,
                                int64_t offset, const int64_t* logical, const uint16_t* values, int64_t rows,
                                int32_t* err, void* stream) {
  dsr::clear_error();
  DSR_REQUIRE(data && generations && logical && values && err, "pool_restore: null pointer");
  DSR_REQUIRE(slots > 0 && width > 0 && width <= dsr::kPoolMaxWidth && offset >= 0 && offset < slots,
              "pool_restore: invalid pool geometry");
  DSR_REQUIRE(rows >= 1 && rows <= dsr::kPoolMaxRestore, "pool_restore: tile of %lld rows outside [1, 1024]",
              (long long)rows);
  const bool vec = dsr::rows_vec(int(width), data, values, values);
  dsr::pool_restore_kernel<<<1, dsr::kPoolThreads, 0, dsr::as_stream(stream)>>>(
      data, generations, slots, int(width), offset, logical, values, int(rows), vec, err);
  return dsr::launch_status("pool_restore launch");
}
