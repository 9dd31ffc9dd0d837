// Host-side helpers: per-thread error messages, device queries, tensor maps.
#include "host_common.h"

#include <map>
#include <mutex>
#include <utility>

namespace dsr {

namespace {
thread_local std::string g_message;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}
}  // namespace

int fail(int code, const char* fmt, ...) {
  char buffer[512];
  va_list args;
  va_start(args, fmt);
  vsnprintf(buffer, sizeof(buffer), fmt, args);
  va_end(args);
  g_message = buffer;
  return code;
}

void clear_error() { g_message.clear(); }

int launch_status(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(DSR_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  return DSR_OK;
}

int sm_count() {
  static int counts[64] = {0};
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return 148;
  if (device < 0 || device >= 64) return 148;
  if (counts[device] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0)
      n = 148;
    counts[device] = n;
  }
  return counts[device];
}

int set_max_smem_raw(const void* fn, int bytes, const char* what) {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return fail(DSR_ECUDA, "%s: no current CUDA device", what);
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, int> limit;  // largest limit set so far
  std::lock_guard<std::mutex> lock(mu);
  int& have = limit[{device, fn}];
  if (have >= bytes) return DSR_OK;
  const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess)
    return fail(DSR_ECUDA, "%s: shared-memory attribute: %s", what, cudaGetErrorString(e));
  have = bytes;
  return DSR_OK;
}

int paged_addr(PoolAddr* a, const int32_t* table, int64_t stride, int64_t pool_blocks, const char* what) {
  if (table == nullptr) return fail(DSR_EINVAL, "%s: null block table", what);
  if (stride <= 0 || stride * 64 > (int64_t(1) << 31) - 1)
    return fail(DSR_EINVAL, "%s: block-table stride %lld outside [1, 2^25)", what, (long long)stride);
  if (pool_blocks <= 0 || pool_blocks * 64 > (int64_t(1) << 31) - 1)
    return fail(DSR_EINVAL, "%s: pool blocks %lld outside [1, 2^25)", what, (long long)pool_blocks);
  *a = PoolAddr{table, stride, nullptr, pool_blocks * 64};
  return DSR_OK;
}

int ring_addr(PoolAddr* a, const int64_t* ring, int64_t rows, const char* what) {
  if (ring == nullptr) return fail(DSR_EINVAL, "%s: null ring descriptors", what);
  if (rows <= 0 || rows > (int64_t(1) << 31) - 1)
    return fail(DSR_EINVAL, "%s: pool rows %lld outside [1, 2^31)", what, (long long)rows);
  *a = PoolAddr{nullptr, 0, ring, rows};
  return DSR_OK;
}

int encode_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                        uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(DSR_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {inner * 2};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t elem[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                        strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DSR_ECUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return DSR_OK;
}

}  // namespace dsr

extern "C" const char* dsr_last_error(void) { return dsr::g_message.c_str(); }

extern "C" int dsr_abi_version(void) { return 2; }

extern "C" int dsr_device_check(void) {
  int device = 0, major = 0;
  if (cudaGetDevice(&device) != cudaSuccess)
    return dsr::fail(DSR_ENODEV, "no CUDA device is available");
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess)
    return dsr::fail(DSR_ENODEV, "cannot query the compute capability");
  if (major != 10)
    return dsr::fail(DSR_ENODEV, "this build targets sm_100a; device %d is sm_%d.x", device, major);
  return DSR_OK;
}
