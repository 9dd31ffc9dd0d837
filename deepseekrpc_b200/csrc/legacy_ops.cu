// Reference drop-in operations (index_scores, sparse_attention, scatter_slots,
// engram_decode) with the reference's exact data semantics and error codes,
// FP32 arithmetic, and the bounds widened to the DeepSeek-V3.2/V4 geometry.
//
// Reference: native/operations.cu:30-243 (kernels and entry points).
#include "common.cuh"
#include "host_common.h"

#include <math_constants.h>

namespace dsr {
namespace {

// ---------------------------------------------------------------------------
// index_scores (operations.cu:84-123)
// One block scores 64 columns of one row.  q is staged transposed (qT[d][h])
// so that lane l reads heads l and l+32 without bank conflicts; the 64 keys
// are staged as fp32 rows and read by broadcast.
// ---------------------------------------------------------------------------
constexpr int kIdxKeys = 64;
constexpr int kIdxDim = 128;

__global__ void __launch_bounds__(256) legacy_index_kernel(
    const float* __restrict__ q, const uint16_t* __restrict__ keys,
    const float* __restrict__ weights, const int32_t* __restrict__ ids,
    const int32_t* __restrict__ visible, float* __restrict__ out, int32_t* err, int heads,
    int64_t columns, int64_t capacity) {
  extern __shared__ float smem[];
  float* qT = smem;                         // [128][64]
  float* ks = qT + kIdxDim * 64;            // [64][128]
  float* w = ks + kIdxKeys * kIdxDim;       // [64]
  int* status = reinterpret_cast<int*>(w + 64);  // [64]: 0 score, 1 -inf, 2 -inf + error

  const int row = blockIdx.y;
  const int64_t col0 = static_cast<int64_t>(blockIdx.x) * kIdxKeys;
  const int vis = visible[row];
  const bool bad_visible = vis < 0 || static_cast<int64_t>(vis) > capacity;

  for (int i = threadIdx.x; i < heads * kIdxDim; i += blockDim.x) {
    const int h = i / kIdxDim, d = i % kIdxDim;
    qT[d * 64 + h] = q[(static_cast<int64_t>(row) * heads + h) * kIdxDim + d];
  }
  for (int h = threadIdx.x; h < 64; h += blockDim.x) w[h] = h < heads ? weights[row * heads + h] : 0.f;
  if (threadIdx.x < kIdxKeys) {
    const int64_t col = col0 + threadIdx.x;
    int st = 1;
    if (col < columns) {
      const int64_t id = ids[static_cast<int64_t>(row) * columns + col];
      if (bad_visible) st = 2;
      else if (id == -1 || (id >= 0 && id < capacity && id >= vis)) st = 1;
      else if (id < 0 || id >= capacity) st = 2;
      else st = 0;
    }
    status[threadIdx.x] = st;
  }
  __syncthreads();
  // Stage valid keys (bf16 -> fp32); 16 threads per key, 8 elements each.
  for (int i = threadIdx.x; i < kIdxKeys * 16; i += blockDim.x) {
    const int j = i >> 4, part = i & 15;
    float* dst = ks + j * kIdxDim + part * 8;
    if (status[j] == 0) {
      const int64_t id = ids[static_cast<int64_t>(row) * columns + col0 + j];
      const uint4 v = *reinterpret_cast<const uint4*>(keys + id * kIdxDim + part * 8);
      const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        dst[2 * t] = __uint_as_float(words[t] << 16);
        dst[2 * t + 1] = __uint_as_float(words[t] & 0xffff0000u);
      }
    } else {
#pragma unroll
      for (int t = 0; t < 8; ++t) dst[t] = 0.f;
    }
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h0 = lane, h1 = lane + 32;
  float acc0[8], acc1[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc0[j] = acc1[j] = 0.f;
  const float* kw = ks + warp * 8 * kIdxDim;
#pragma unroll 2
  for (int d = 0; d < kIdxDim; d += 4) {
    float qa[4], qb[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      qa[t] = qT[(d + t) * 64 + h0];
      qb[t] = qT[(d + t) * 64 + h1];
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 kv = *reinterpret_cast<const float4*>(kw + j * kIdxDim + d);
      acc0[j] = fmaf(qa[0], kv.x, acc0[j]);
      acc0[j] = fmaf(qa[1], kv.y, acc0[j]);
      acc0[j] = fmaf(qa[2], kv.z, acc0[j]);
      acc0[j] = fmaf(qa[3], kv.w, acc0[j]);
      acc1[j] = fmaf(qb[0], kv.x, acc1[j]);
      acc1[j] = fmaf(qb[1], kv.y, acc1[j]);
      acc1[j] = fmaf(qb[2], kv.z, acc1[j]);
      acc1[j] = fmaf(qb[3], kv.w, acc1[j]);
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int slot = warp * 8 + j;
    const int64_t col = col0 + slot;
    const int st = status[slot];
    if (col >= columns) continue;  // warp-uniform
    if (st != 0) {
      if (lane == 0) {
        if (st == 2) flag(err, DSR_ERR_ID);
        out[static_cast<int64_t>(row) * columns + col] = -CUDART_INF_F;
      }
      continue;
    }
    float term = 0.f;
    if (h0 < heads) {
      if (!isfinite(acc0[j]) || !isfinite(w[h0])) flag(err, DSR_ERR_NONFINITE);
      term = fmaxf(acc0[j], 0.f) * w[h0];
    }
    if (h1 < heads) {
      if (!isfinite(acc1[j]) || !isfinite(w[h1])) flag(err, DSR_ERR_NONFINITE);
      term += fmaxf(acc1[j], 0.f) * w[h1];
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) term += __shfl_xor_sync(0xffffffffu, term, off);
    if (lane == 0) {
      if (!isfinite(term)) flag(err, DSR_ERR_NONFINITE);
      out[static_cast<int64_t>(row) * columns + col] = term;
    }
  }
}

// ---------------------------------------------------------------------------
// sparse_attention (operations.cu:30-82)
// Block = 8 warps = 8 heads of one query row.  Selected rows are staged 32 at a
// time (fp32-converted on use, padded stride so lane-per-row reads are
// conflict free); each warp keeps its head's online-softmax state, starting
// from (sink, 1, 0) exactly as the reference.
// ---------------------------------------------------------------------------
constexpr int kAttChunk = 32;
constexpr int kAttMaxWidth = 576;

__global__ void __launch_bounds__(256) legacy_sparse_kernel(
    const float* __restrict__ q, const uint16_t* __restrict__ window,
    const uint16_t* __restrict__ source, const int32_t* __restrict__ ids,
    const float* __restrict__ sink, float* __restrict__ out, int32_t* err, int heads, int width,
    int64_t window_rows, int64_t source_rows, int64_t selected, float scale) {
  extern __shared__ uint32_t att_smem[];
  const int pitch = width / 2 + 1;  // 32-bit words per staged row (odd => conflict free)
  uint32_t* rows = att_smem;                                         // [32][pitch]
  float* qs = reinterpret_cast<float*>(rows + kAttChunk * pitch);    // [8][width]
  int* valid = reinterpret_cast<int*>(qs + 8 * width);               // [32]

  const int row = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = blockIdx.y * 8 + warp;
  const bool active = head < heads;
  const int words = width / 2;  // width is even (checked on the host)

  for (int i = threadIdx.x; i < 8 * width; i += blockDim.x) {
    const int hh = blockIdx.y * 8 + i / width;
    qs[i] = hh < heads ? q[(static_cast<int64_t>(row) * heads + hh) * width + i % width] : 0.f;
  }
  float m = 0.f, l = 1.f;
  if (active) {
    m = sink[head];
    if (!isfinite(m)) {
      if (lane == 0) flag(err, DSR_ERR_NONFINITE);
      m = 0.f;
    }
  }
  // lane owns columns 2*lane + 64*i (+1)
  constexpr int kPairs = (kAttMaxWidth + 63) / 64;  // 9
  float acc[2 * kPairs];
#pragma unroll
  for (int i = 0; i < 2 * kPairs; ++i) acc[i] = 0.f;
  const float* qh = qs + warp * width;
  const int64_t total = window_rows + source_rows;

  for (int64_t c0 = 0; c0 < selected; c0 += kAttChunk) {
    __syncthreads();
    if (threadIdx.x < kAttChunk) {
      const int64_t c = c0 + threadIdx.x;
      int v = 0;
      if (c < selected) {
        const int64_t id = ids[static_cast<int64_t>(row) * selected + c];
        if (id != -1) {
          if (id < 0 || id >= total) flag(err, DSR_ERR_ID);
          else v = 1;
        }
      }
      valid[threadIdx.x] = v;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < kAttChunk * words; i += blockDim.x) {
      const int j = i / words, wd = i % words;
      uint32_t value = 0;
      if (valid[j]) {
        const int64_t id = ids[static_cast<int64_t>(row) * selected + c0 + j];
        const uint16_t* src = id < window_rows ? window + id * width : source + (id - window_rows) * width;
        value = reinterpret_cast<const uint32_t*>(src)[wd];
      }
      rows[j * pitch + wd] = value;
    }
    __syncthreads();
    if (!active) continue;
    // score of row `lane`
    float s = -CUDART_INF_F;
    const bool mine = valid[lane] != 0;
    if (mine) {
      float dot = 0.f;
      const uint32_t* r = rows + lane * pitch;
      for (int wd = 0; wd < words; ++wd) {
        const uint32_t v = r[wd];
        const float2 qq = *reinterpret_cast<const float2*>(qh + 2 * wd);
        dot = fmaf(qq.x, __uint_as_float(v << 16), dot);
        dot = fmaf(qq.y, __uint_as_float(v & 0xffff0000u), dot);
      }
      s = dot * scale;
      if (!isfinite(s)) flag(err, DSR_ERR_NONFINITE);
    }
    const unsigned any = __ballot_sync(0xffffffffu, mine);
    if (!any) continue;
    float cmax = mine ? s : -CUDART_INF_F;
#pragma unroll
    for (int off = 16; off; off >>= 1) cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, off));
    const float next = fmaxf(m, cmax);
    const float keep = expf(m - next);
    const float p = mine ? expf(s - next) : 0.f;
    float psum = p;
#pragma unroll
    for (int off = 16; off; off >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
    l = l * keep + psum;
#pragma unroll
    for (int i = 0; i < 2 * kPairs; ++i) acc[i] *= keep;
    for (int j = 0; j < kAttChunk; ++j) {
      if (!((any >> j) & 1u)) continue;
      const float pj = __shfl_sync(0xffffffffu, p, j);
      const uint32_t* r = rows + j * pitch;
#pragma unroll
      for (int i = 0; i < kPairs; ++i) {
        const int wd = lane + 32 * i;
        if (wd < words) {
          const uint32_t v = r[wd];
          acc[2 * i] = fmaf(pj, __uint_as_float(v << 16), acc[2 * i]);
          acc[2 * i + 1] = fmaf(pj, __uint_as_float(v & 0xffff0000u), acc[2 * i + 1]);
        }
      }
    }
    m = next;
  }
  if (!active) return;
  float* o = out + (static_cast<int64_t>(row) * heads + head) * width;
#pragma unroll
  for (int i = 0; i < kPairs; ++i) {
    const int wd = lane + 32 * i;
    if (wd < words) {
      const float a = acc[2 * i] / l, b = acc[2 * i + 1] / l;
      if (!isfinite(a) || !isfinite(b)) flag(err, DSR_ERR_NONFINITE);
      o[2 * wd] = a;
      o[2 * wd + 1] = b;
    }
  }
}

// ---------------------------------------------------------------------------
// scatter_slots (operations.cu:144-161)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) legacy_scatter_kernel(
    uint16_t* __restrict__ pool, const int64_t* __restrict__ generations,
    const int32_t* __restrict__ slots, const int64_t* __restrict__ expected,
    const uint16_t* __restrict__ values, int32_t* err, int rows, int width, int64_t capacity) {
  __shared__ int duplicate;
  const int row = blockIdx.x;
  const int64_t slot = slots[row];
  if (threadIdx.x == 0) duplicate = 0;
  __syncthreads();
  for (int prev = threadIdx.x; prev < row; prev += blockDim.x)
    if (slots[prev] == slot) atomicOr(&duplicate, 1);
  __syncthreads();
  const bool in_bounds = slot >= 0 && slot < capacity;
  if (!in_bounds || duplicate || generations[slot] != expected[row]) {
    if (threadIdx.x == 0) flag(err, DSR_ERR_SCATTER);
    return;
  }
  for (int d = threadIdx.x; d < width; d += blockDim.x) {
    const uint16_t v = values[static_cast<int64_t>(row) * width + d];
    if ((v & 0x7f80) == 0x7f80) flag(err, DSR_ERR_NONFINITE);
    else pool[slot * width + d] = v;
  }
}

// ---------------------------------------------------------------------------
// engram_decode (operations.cu:125-142): FP8 E4M3 x UE8M0 -> BF16
// ---------------------------------------------------------------------------
__global__ void legacy_engram_kernel(const uint8_t* __restrict__ encoded, uint16_t* __restrict__ out,
                                     int32_t* err, int64_t elements) {
  const int64_t index = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (index >= elements) return;
  const int64_t row = index / 256;
  const int dim = static_cast<int>(index % 256);
  const uint8_t bits = encoded[row * 264 + dim], scale = encoded[row * 264 + 256 + dim / 32];
  const int exponent = (bits >> 3) & 15, mantissa = bits & 7;
  if ((exponent == 15 && mantissa == 7) || scale == 255) {
    flag(err, DSR_ERR_NONFINITE);
    out[index] = 0;
    return;
  }
  // E4M3: subnormal m*2^-9, normal (1+m/8)*2^(e-7); UE8M0: 2^(s-127) (byte 0 = 2^-127).
  float value = exponent == 0 ? ldexpf(static_cast<float>(mantissa), -9)
                              : ldexpf(1.0f + mantissa / 8.0f, exponent - 7);
  if (bits & 128) value = -value;
  value *= ldexpf(1.0f, static_cast<int>(scale) - 127);
  if (!isfinite(value)) flag(err, DSR_ERR_NONFINITE);
  const __nv_bfloat16 rounded = __float2bfloat16_rn(value);
  if (!isfinite(__bfloat162float(rounded))) flag(err, DSR_ERR_NONFINITE);
  out[index] = __bfloat16_as_ushort(rounded);
}

}  // namespace
}  // namespace dsr

using namespace dsr;

extern "C" int dsr_index_scores(const float* q, const uint16_t* keys, const float* weights,
                                const int32_t* ids, const int32_t* visible, float* out,
                                int32_t* err, int64_t rows, int64_t heads, int64_t columns,
                                int64_t capacity, void* stream) {
  clear_error();
  DSR_REQUIRE(q && keys && weights && ids && visible && out && err, "index_scores: null pointer");
  DSR_REQUIRE(rows > 0 && rows <= 65536 && heads > 0 && heads <= 64,
              "invalid index query/key shape: rows %lld heads %lld (rows<=65536, heads<=64)",
              (long long)rows, (long long)heads);
  DSR_REQUIRE(columns > 0 && columns <= (int64_t(1) << 31) - 1 && capacity >= 0 &&
                  capacity <= (int64_t(1) << 31) - 1,
              "invalid bounded index tile: columns %lld capacity %lld", (long long)columns,
              (long long)capacity);
  DSR_REQUIRE(aligned16(keys), "index keys must be 16-byte aligned");
  const int64_t blocks_x = (columns + kIdxKeys - 1) / kIdxKeys;
  DSR_REQUIRE(blocks_x <= 2147483647LL, "too many index columns");
  const size_t smem = (kIdxDim * 64 + kIdxKeys * kIdxDim + 64 + 64) * sizeof(float);
  {
    const int rc = set_max_smem(legacy_index_kernel, smem, "index_scores");
    if (rc != DSR_OK) return rc;
  }
  legacy_index_kernel<<<dim3(unsigned(blocks_x), unsigned(rows)), 256, smem, as_stream(stream)>>>(
      q, keys, weights, ids, visible, out, err, int(heads), columns, capacity);
  return launch_status("index_scores launch");
}

extern "C" int dsr_sparse_attention(const float* q, const uint16_t* window, const uint16_t* source,
                                    const int32_t* ids, const float* sink, float* out, int32_t* err,
                                    int64_t rows, int64_t heads, int64_t width, int64_t window_rows,
                                    int64_t source_rows, int64_t selected, float scale,
                                    void* stream) {
  clear_error();
  DSR_REQUIRE(q && window && source && ids && sink && out && err, "sparse_attention: null pointer");
  DSR_REQUIRE(rows > 0 && rows <= 65536 && heads > 0 && heads <= 128,
              "invalid bounded query shape: rows %lld heads %lld", (long long)rows,
              (long long)heads);
  DSR_REQUIRE(width > 0 && width <= kAttMaxWidth && width % 2 == 0 && window_rows >= 0 &&
                  window_rows <= 65536 && source_rows >= 0 &&
                  source_rows <= (int64_t(1) << 31) - 1,
              "KV dimensions/capacity differ from bounded query (width %lld even <= 576)",
              (long long)width);
  DSR_REQUIRE(selected >= 0 && selected <= 65536, "invalid sparse indices/sink shape");
  DSR_REQUIRE(isfinite(scale) && scale > 0.f, "invalid attention scale");
  DSR_REQUIRE((reinterpret_cast<uintptr_t>(window) & 3u) == 0 &&
                  (reinterpret_cast<uintptr_t>(source) & 3u) == 0,
              "window/source rows must be 4-byte aligned");
  const size_t smem = size_t(kAttChunk) * (width / 2 + 1) * 4 + 8 * width * 4 + kAttChunk * 4;
  {
    const int rc = set_max_smem(legacy_sparse_kernel, smem, "sparse_attention");
    if (rc != DSR_OK) return rc;
  }
  legacy_sparse_kernel<<<dim3(unsigned(rows), unsigned((heads + 7) / 8)), 256, smem,
                         as_stream(stream)>>>(q, window, source, ids, sink, out, err, int(heads),
                                              int(width), window_rows, source_rows, selected,
                                              scale);
  return launch_status("sparse_attention launch");
}

extern "C" int dsr_scatter_slots(uint16_t* pool, const int64_t* generations, const int32_t* slots,
                                 const int64_t* expected, const uint16_t* values, int32_t* err,
                                 int64_t rows, int64_t width, int64_t capacity, void* stream) {
  clear_error();
  DSR_REQUIRE(pool && generations && slots && expected && values && err, "scatter_slots: null pointer");
  DSR_REQUIRE(width > 0 && width <= kAttMaxWidth && capacity > 0, "invalid cache/generation pool");
  DSR_REQUIRE(rows > 0 && rows <= 4096, "invalid cache update rows");
  legacy_scatter_kernel<<<unsigned(rows), 256, 0, as_stream(stream)>>>(
      pool, generations, slots, expected, values, err, int(rows), int(width), capacity);
  return launch_status("scatter_slots launch");
}

extern "C" int dsr_engram_decode(const uint8_t* encoded, uint16_t* out, int32_t* err, int64_t rows,
                                 void* stream) {
  clear_error();
  DSR_REQUIRE(encoded && out && err, "engram_decode: null pointer");
  DSR_REQUIRE(rows > 0 && rows <= 1024, "encoded Engram rows must be bounded [rows,264] uint8");
  const int64_t elements = rows * 256;
  legacy_engram_kernel<<<unsigned((elements + 255) / 256), 256, 0, as_stream(stream)>>>(
      encoded, out, err, elements);
  return launch_status("engram_decode launch");
}
