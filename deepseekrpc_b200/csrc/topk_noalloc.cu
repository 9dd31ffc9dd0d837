// Allocation-free entry point for the exact top-k selection.
//
// Same kernels and results as dsr_topk_select; the scratch is a fixed array in
// this library's device memory instead of a caller-provided workspace, so a
// host that cannot hand out device memory (or wants none allocated per call)
// can still run the selection.  Nothing here calls an allocating routine: the
// array is part of the module image, its address comes from
// cudaGetSymbolAddress on the current device, and the leading part that the kernels expect to be
// zero (histograms, tickets, candidate counts) is cleared with cudaMemsetAsync
// on the caller's stream before every launch.
#include <mutex>

#include "common.cuh"
#include "host_common.h"

namespace {

constexpr size_t kNoAllocScratchBytes = DSR_TOPK_NOALLOC_BYTES;
static_assert(kNoAllocScratchBytes % 256 == 0, "scratch size must keep 256-byte alignment");

static __device__ __align__(256) uint8_t g_topk_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_addr[kMaxDevices] = {};

// Address of this device's scratch array.  Outside stream capture it is looked
// up again on every call (a device reset reloads the module and may move the
// array); during capture the address recorded by the last uncaptured call on
// this device is used, since a lookup may load the module, which capture forbids.
int scratch_address(cudaStream_t stream, void** out) {
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return dsr::fail(DSR_ECUDA, "topk_select_noalloc: cudaGetDevice: %s",
                                         cudaGetErrorString(e));
  if (device < 0 || device >= kMaxDevices)
    return dsr::fail(DSR_EINVAL, "topk_select_noalloc: device ordinal %d beyond %d", device,
                     kMaxDevices - 1);
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  e = cudaStreamIsCapturing(stream, &capture);
  if (e != cudaSuccess) return dsr::fail(DSR_ECUDA, "topk_select_noalloc: capture status: %s",
                                         cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (capture == cudaStreamCaptureStatusNone) {
    void* addr = nullptr;
    e = cudaGetSymbolAddress(&addr, g_topk_scratch);
    if (e != cudaSuccess) return dsr::fail(DSR_ECUDA, "topk_select_noalloc: scratch address: %s",
                                           cudaGetErrorString(e));
    g_scratch_addr[device] = addr;
  } else if (g_scratch_addr[device] == nullptr) {
    return dsr::fail(DSR_EINVAL,
                     "topk_select_noalloc: the first call on device %d must come before any stream capture",
                     device);
  }
  *out = g_scratch_addr[device];
  return DSR_OK;
}

}  // namespace

extern "C" int dsr_topk_select_noalloc(const float* scores, const int32_t* ids,
                                       const int32_t* lengths, int32_t* out_ids,
                                       float* out_scores, int32_t* err, int64_t rows,
                                       int64_t row_stride, int64_t k, int64_t id_base,
                                       void* stream) {
  using namespace dsr;
  clear_error();
  // size limits first, before any CUDA call
  DSR_REQUIRE(rows > 0 && rows <= 65535, "topk_select_noalloc: rows %lld outside [1, 65535]",
              (long long)rows);
  DSR_REQUIRE(row_stride > 0 && row_stride <= (int64_t(1) << 31) - 1,
              "topk_select_noalloc: invalid row stride");
  const size_t need = topk_workspace_bytes(rows, row_stride);
  DSR_REQUIRE(need <= kNoAllocScratchBytes,
              "topk_select_noalloc: %lld rows x %lld entries need %zu scratch bytes > %zu",
              (long long)rows, (long long)row_stride, need, kNoAllocScratchBytes);
  DSR_REQUIRE(scores && lengths && out_ids && err, "topk_select_noalloc: null pointer");
  DSR_REQUIRE(k > 0 && k <= 8192, "topk_select_noalloc: k %lld outside [1, 8192]", (long long)k);
  DSR_REQUIRE(id_base >= 0 && id_base + row_stride < (int64_t(1) << 31) - 1,
              "topk_select_noalloc: id_base %lld + row stride exceeds int32 ids", (long long)id_base);
  const cudaStream_t s = as_stream(stream);
  void* scratch = nullptr;
  int rc = scratch_address(s, &scratch);
  if (rc != DSR_OK) return rc;
  const cudaError_t e = cudaMemsetAsync(scratch, 0, topk_zeroed_prefix_bytes(rows, row_stride), s);
  if (e != cudaSuccess) return fail(DSR_ECUDA, "topk_select_noalloc: clear: %s", cudaGetErrorString(e));
  return launch_topk(scores, ids, lengths, out_ids, out_scores, err, rows, row_stride, k, id_base,
                     scratch, kNoAllocScratchBytes, s, false, false);
}
