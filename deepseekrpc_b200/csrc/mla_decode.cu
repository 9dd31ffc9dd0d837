// Sparse MLA decode attention over the SWA ring plus the top-k selected rows of a
// paged BF16 KV pool, and the log-sum-exp combine of its partials (sm_100a).
// The per-tile work (reference equation, the two tcgen05 products, the
// softmax) is mla_tile_unit in mla_tile.cuh.
//
// mla_decode_kernel: grid (tiles, batch, head groups); one CTA handles one
// 128-row tile (tile 0 = SWA window, tiles 1.. = consecutive 128 top-k ids).
//   warps 0..3  gather the 128 rows (TMA 4-row gathers, 128-byte swizzle), convert the
//               FP32 query to BF16, softmax of the tile, partial output store
//   warp 4      TMEM allocator + tcgen05.mma issuer
// Partials (m in log2 units, l, unnormalised o in bf16) go to the workspace and
// lse_combine_kernel merges them with the sink.
#include "host_common.h"
#include "mla_tile.cuh"

namespace dsr {
namespace {

template <int HG>
__global__ void __launch_bounds__(kMlaThreads, 1)
    mla_decode_kernel(const __grid_constant__ CUtensorMap kv_map,
                      const __grid_constant__ CUtensorMap swa_map,
                      const float* __restrict__ q, const PoolAddr kv,
                      const int64_t* __restrict__ swa_ring, int64_t swa_rows,
                      const int32_t* __restrict__ visible,
                      const int32_t* __restrict__ topk, int k,
                      const int32_t* __restrict__ swa_len, float scale_log2,
                      uint16_t* __restrict__ part_o, float* __restrict__ part_m,
                      float* __restrict__ part_l, int32_t* err, int heads,
                      const uint16_t* __restrict__ q_img, int64_t id_base, int foreign_ok) {
  extern __shared__ uint8_t smem_raw[];
  // top-k ids and the query image come from the preceding kernel
  mla_tile_unit<HG>(align_smem_1024(smem_raw), &kv_map, &swa_map, q, kv, swa_ring, swa_rows, visible, topk, k,
                    swa_len, scale_log2, part_o, part_m, part_l, err, heads, int(blockIdx.x), int(blockIdx.y),
                    int(blockIdx.z), int(gridDim.x), q_img, id_base, foreign_ok, true, [] { pdl_wait(); });
}

// Persistent form for grids of more than one wave (a batch): one CTA per SM
// walks the items (tile, sequence, head group), tile fastest, with stride
// gridDim.x.  Per item the phases are those of mla_decode_kernel; what changes is
// the overlap: the next item's rows are resolved while this item's score MMA
// runs, and its query image and row gathers are issued as soon as this item's
// O MMA has released the row and query buffers, so they land while this item's
// O^T leaves TMEM.  Every barrier completes once per item (phase parity = item
// count & 1); bar_ofree (128 arrivals) tells the MMA issuer that the previous
// item's O^T has been read before it overwrites those TMEM columns.  The query
// comes from the BF16 image only.  (The issuing stays with the key warps: the
// TMA unit takes the 288 row gathers one at a time, faster from four warps than
// from a dedicated loader warp, and one row buffer serialises gather and compute
// of consecutive items anyway.)
template <int HG>
__global__ void __launch_bounds__(kMlaThreads, 1)
    mla_persistent_kernel(const __grid_constant__ CUtensorMap kv_map,
                          const __grid_constant__ CUtensorMap swa_map, const PoolAddr kv,
                          const int64_t* __restrict__ swa_ring, int64_t swa_rows,
                          const int32_t* __restrict__ visible, const int32_t* __restrict__ topk, int k,
                          const int32_t* __restrict__ swa_len, float scale_log2,
                          uint16_t* __restrict__ part_o, float* __restrict__ part_m,
                          float* __restrict__ part_l, int32_t* err, int heads, int batch, int tiles,
                          const uint16_t* __restrict__ q_img, int64_t id_base, int foreign_ok) {
  using L = MlaLayout<HG>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* bar_s = bars + 0;
  uint64_t* bar_p = bars + 1;
  uint64_t* bar_o = bars + 2;
  uint64_t* bar_q = bars + 3;
  uint64_t* bar_kv = bars + 4;
  uint64_t* bar_ofree = bars + 4 + kMlaBlocks;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + L::kMiscOff + 4);
  int* valid = reinterpret_cast<int*>(smem + L::kValidOff);  // [2][kMlaTile]
  float* red = reinterpret_cast<float*>(smem + L::kRedOff);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int items = tiles * batch * (heads / HG);
  auto item_of = [&](int it, int& tile, int& b, int& hg) {
    tile = it % tiles;
    const int r = it / tiles;
    b = r % batch;
    hg = r / batch;
  };

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&swa_map);
    tma_prefetch_desc(&kv_map);
    for (int c = 0; c < kMlaBlocks; ++c) mbar_init(bar_kv + c, 1);
    mbar_init(bar_s, 1);
    mbar_init(bar_p, 128);
    mbar_init(bar_o, 1);
    mbar_init(bar_q, 1);
    mbar_init(bar_ofree, 128);
    *abort = 0;
    fence_barrier_init();
  }
  if (warp == 4) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tmem_s = tmem_base;
  const uint32_t tmem_o = tmem_base + HG;

  pdl_launch_dependents();  // the combine kernel may start its prologue early
  pdl_wait();               // top-k ids and the query image come from the preceding kernels

  if (warp < 4) {
    const int t = threadIdx.x;  // key slot of this thread == TMEM lane
    int issued = 0;             // items whose query and rows were requested (thread 0's count)
    // query image (thread 0) and row gathers (every warp) of item `it`
    auto issue = [&](int it, int32_t row) {
      int tile, b, hg;
      item_of(it, tile, b, hg);
      if (t == 0) {
        constexpr uint32_t kBytes = kMlaBlocks * HG * 128;
        const int gi = heads < 64 ? heads : 64;
        const int h0 = hg * HG;
        const uint8_t* img = reinterpret_cast<const uint8_t*>(q_img) +
                             ((int64_t(b) * (heads / gi) + h0 / gi) * kMlaBlocks * gi + h0 % gi) * 128;
        mbar_arrive_expect_tx(bar_q, kBytes);
        if (gi == HG) {
          bulk_load(sbase + L::kQOff, img, kBytes, bar_q);
        } else {
#pragma unroll 1
          for (int c = 0; c < kMlaBlocks; ++c)
            bulk_load(sbase + L::kQOff + c * (HG * 128), img + int64_t(c) * gi * 128, HG * 128, bar_q);
        }
        for (int c = 0; c < kMlaBlocks; ++c) mbar_arrive_expect_tx(bar_kv + c, kMlaTile * 128);
        ++issued;
      }
      mla_gather_rows(sbase + L::kKvOff, tile == 0 ? &swa_map : &kv_map, bar_kv, warp, lane, row);
    };
    auto resolve = [&](int it, int slot) -> int32_t {
      int tile, b, hg;
      item_of(it, tile, b, hg);
      const int32_t oob = mla_oob_row(tile, swa_rows, kv);
      const int32_t row = mla_key_row(tile, b, t, oob, kv, swa_ring, swa_rows, visible, topk, k, swa_len, id_base,
                                      foreign_ok, err);
      valid[slot * kMlaTile + t] = row != oob;
      return row;
    };
    if (int(blockIdx.x) < items) issue(blockIdx.x, resolve(blockIdx.x, 0));
    int n = 0;
    for (int it = blockIdx.x; it < items; it += gridDim.x, ++n) {
      const uint32_t par = uint32_t(n) & 1u;
      const int next = it + int(gridDim.x);
      // the next item's rows, while this item's score MMA runs (its valid[] slot was
      // last read by the item before this one; each thread reads only its own entry)
      const int32_t row_next = next < items ? resolve(next, (n + 1) & 1) : 0;
      int tile, b, hg;
      item_of(it, tile, b, hg);
      const int64_t pidx = (int64_t(b) * tiles + tile) * heads + hg * HG;
      const bool ok = mbar_wait(bar_s, par, abort, err);
      mla_softmax<HG>(smem, tmem_s, warp, t, ok, valid + (n & 1) * kMlaTile, scale_log2, bar_p, red, part_m,
                      part_l, pidx, err);
      const bool o_ok = ok && mbar_wait(bar_o, par, abort, err);
      // the O MMA has read the rows and P^T: the next item's query and rows may land
      // (the abort flag is read once per warp: the gathers shuffle across all lanes)
      const bool go = next < items && __shfl_sync(0xffffffffu, *abort == 0 ? 1 : 0, 0) != 0;
      if (go) issue(next, row_next);
      if (o_ok) {
        tc_fence_after();
        mla_store_o<HG>(tmem_o, warp, t, part_o + pidx * kMlaDv);
      }
      tc_fence_before();
      mbar_arrive(bar_ofree);
    }
    if (*abort && t == 0 && issued > 0) {
      // let the last requested query and rows land before exit
      const uint32_t last = uint32_t(issued - 1) & 1u;
      for (int c = 0; c < kMlaBlocks; ++c) mbar_drain(bar_kv + c, last);
      mbar_drain(bar_q, last);
    }
  } else if (warp == 4 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc_s = umma_idesc_bf16(128, HG, false, false);
    constexpr uint32_t idesc_o = umma_idesc_bf16(128, HG, true, false);
    int n = 0, committed_o = 0;
    for (int it = blockIdx.x; it < items; it += gridDim.x, ++n) {
      const uint32_t par = uint32_t(n) & 1u;
      bool ready = mbar_wait(bar_q, par, abort, err);
#pragma unroll 1
      for (int c = 0; c < kMlaBlocks && ready; ++c) {
        ready = mbar_wait(bar_kv + c, par, abort, err);
        if (!ready) break;
        tc_fence_after();
#pragma unroll
        for (int sub = 0; sub < 4; ++sub) {
          const uint64_t ad = umma_desc_sw128(sbase + L::kKvOff + c * 16384 + sub * 32, 16, 1024);
          const uint64_t bd = umma_desc_sw128(sbase + L::kQOff + c * (HG * 128) + sub * 32, 16, 1024);
          umma_bf16(tmem_s, ad, bd, idesc_s, (c | sub) != 0 ? 1u : 0u);
        }
      }
      if (!ready) break;
      umma_commit(bar_s);
      if (!mbar_wait(bar_p, par, abort, err)) break;
      // the previous item's O^T has left TMEM
      if (n > 0 && !mbar_wait(bar_ofree, par ^ 1u, abort, err)) break;
      tc_fence_after();
#pragma unroll 1
      for (int ks = 0; ks < kMlaTile / 16; ++ks) {
#pragma unroll
        for (int c = 0; c < kMlaDv / 128; ++c) {
          const uint64_t ad = umma_desc_sw128(sbase + L::kKvOff + (2 * c) * 16384 + ks * 2048, 16384, 1024);
          const uint64_t bd =
              umma_desc_sw128(sbase + L::kPOff + (ks >> 2) * (HG * 128) + (ks & 3) * 32, 16, 1024);
          umma_bf16(tmem_o + c * HG, ad, bd, idesc_o, ks > 0 ? 1u : 0u);
        }
      }
      umma_commit(bar_o);
      ++committed_o;
    }
    // the last O MMAs retire before TMEM is released
    if (committed_o > 0) mbar_drain(bar_o, uint32_t(committed_o - 1) & 1u);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Combine of per-shard partials in their exchange layout: packed f32
// [world][o (B*H*512) | m (B*H) | l (B*H)], one (b, h) per CTA; the sink enters
// once.  out[b,h,:] = sum_w o_w 2^{m_w-M} / (2^{log2(e) sink_h - M} + sum_w l_w 2^{m_w-M}).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) lse_combine_packed_kernel(
    const float* __restrict__ packed, int world, const float* __restrict__ sink,
    float* __restrict__ out, int32_t* err, int heads) {
  __shared__ float wgt[64];
  __shared__ float stat[2];
  const int b = blockIdx.x, h = blockIdx.y;
  const int64_t bh = int64_t(gridDim.x) * heads, pair = int64_t(b) * heads + h;
  const int64_t span = bh * (kMlaDv + 2);  // floats per shard
  pdl_wait();
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    float sk = sink[h];
    if (!isfinite(sk)) {
      if (lane == 0) flag(err, DSR_ERR_NONFINITE);
      sk = 0.f;
    }
    sk *= kLog2e;
    float M = sk;
    for (int w = lane; w < world; w += 32) M = fmaxf(M, packed[w * span + bh * kMlaDv + pair]);
#pragma unroll
    for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float lsum = 0.f;
    for (int w = lane; w < world; w += 32) {
      const float e = exp2f(packed[w * span + bh * kMlaDv + pair] - M);
      wgt[w] = e;
      lsum += packed[w * span + bh * (kMlaDv + 1) + pair] * e;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
    if (lane == 0) stat[0] = 1.f / (lsum + exp2f(sk - M));
  }
  __syncthreads();
  const float inv = stat[0];
  for (int d = threadIdx.x * 4; d < kMlaDv; d += blockDim.x * 4) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int w = 0; w < world; ++w) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(packed + w * span + pair * kMlaDv + d));
      const float e = wgt[w];
      acc.x = fmaf(v.x, e, acc.x);
      acc.y = fmaf(v.y, e, acc.y);
      acc.z = fmaf(v.z, e, acc.z);
      acc.w = fmaf(v.w, e, acc.w);
    }
    const float4 o = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
    if (!isfinite(o.x) || !isfinite(o.y) || !isfinite(o.z) || !isfinite(o.w)) flag(err, DSR_ERR_NONFINITE);
    *reinterpret_cast<float4*>(out + pair * kMlaDv + d) = o;
  }
}

// ---------------------------------------------------------------------------
// LSE combine.  m in log2 units; with a sink (natural-log units, converted
// here) the output is normalised, otherwise the merged partial is returned.
// ---------------------------------------------------------------------------
// four consecutive partial values as floats: fp32 partials (the public combine)
// or bf16 bits (the tile partials of the MLA kernel)
template <typename T>
struct PartLoad;
template <>
struct PartLoad<float> {
  using Raw = float4;
  static __device__ __forceinline__ Raw load(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
  static __device__ __forceinline__ float4 cvt(Raw r) { return r; }
};
template <>
struct PartLoad<uint16_t> {
  using Raw = uint2;
  static __device__ __forceinline__ Raw load(const uint16_t* p) { return __ldg(reinterpret_cast<const uint2*>(p)); }
  static __device__ __forceinline__ float4 cvt(Raw r) {
    return make_float4(__uint_as_float(r.x << 16), __uint_as_float(r.x & 0xffff0000u),
                       __uint_as_float(r.y << 16), __uint_as_float(r.y & 0xffff0000u));
  }
};

// kInFlight: partials whose columns a thread requests before the weights exist.
// Few CTAs (one sequence): 24, one memory round trip per CTA.  Thousands of CTAs
// (a batch): 8, so that eight CTAs fit an SM and occupancy hides the latency.
template <typename T, int kInFlight>
__global__ void __launch_bounds__(128, kInFlight > 8 ? 1 : 8) lse_combine_kernel(
    const T* __restrict__ part_o, const float* __restrict__ part_m,
    const float* __restrict__ part_l, int parts, const float* __restrict__ sink,
    float* __restrict__ out, float* __restrict__ out_m, float* __restrict__ out_l, int32_t* err,
    int heads, int dv) {
  extern __shared__ float wgt[];  // [parts] weights 2^{m_t - M}
  __shared__ float stat[2];       // M, L
  const int b = blockIdx.x, h = blockIdx.y;
  pdl_wait();
  const int64_t pbase = int64_t(b) * parts * heads + h;  // partial t at pbase + t * heads
  // the columns of the first kInFlight partials are requested before the weights
  // exist, so the statistics and the values arrive in one memory round trip
  const int d0 = threadIdx.x * 4;
  using P = PartLoad<T>;
  typename P::Raw v[kInFlight];
#pragma unroll
  for (int j = 0; j < kInFlight; ++j)
    if (j < parts && d0 < dv) v[j] = P::load(part_o + (pbase + int64_t(j) * heads) * dv + d0);
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    float sk = 0.f, M = -CUDART_INF_F;
    if (sink != nullptr) {
      sk = sink[h];
      if (!isfinite(sk)) {
        if (lane == 0) flag(err, DSR_ERR_NONFINITE);
        sk = 0.f;
      }
      sk *= kLog2e;
      M = sk;
    }
    float mv[4], lv[4];  // up to 128 partials, loaded together
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int t = lane + 32 * j;
      mv[j] = t < parts ? part_m[pbase + int64_t(t) * heads] : -CUDART_INF_F;
      lv[j] = t < parts ? part_l[pbase + int64_t(t) * heads] : 0.f;
    }
    for (int t = lane + 128; t < parts; t += 32) M = fmaxf(M, part_m[pbase + int64_t(t) * heads]);
#pragma unroll
    for (int j = 0; j < 4; ++j) M = fmaxf(M, mv[j]);
#pragma unroll
    for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const float base = M == -CUDART_INF_F ? 0.f : M;
    float lsum = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int t = lane + 32 * j;
      if (t < parts) {
        const float e = exp2f(mv[j] - base);
        wgt[t] = e;
        lsum += lv[j] * e;
      }
    }
    for (int t = lane + 128; t < parts; t += 32) {
      const int64_t i = pbase + int64_t(t) * heads;
      const float e = exp2f(part_m[i] - base);
      wgt[t] = e;
      lsum += part_l[i] * e;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
    if (lane == 0) {
      if (sink != nullptr) lsum += exp2f(sk - base);
      stat[0] = M;
      stat[1] = lsum;
    }
  }
  __syncthreads();
  const float inv = sink != nullptr ? 1.f / stat[1] : 1.f;
  for (int d = d0; d < dv; d += blockDim.x * 4) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (d == d0) {
#pragma unroll
      for (int j = 0; j < kInFlight; ++j)
        if (j < parts) {
          const float w = wgt[j];
          const float4 x = P::cvt(v[j]);
          acc.x = fmaf(x.x, w, acc.x);
          acc.y = fmaf(x.y, w, acc.y);
          acc.z = fmaf(x.z, w, acc.z);
          acc.w = fmaf(x.w, w, acc.w);
        }
    }
    // columns past the first group, and partials past kInFlight, 8 loads at a time
    for (int t0 = d == d0 ? kInFlight : 0; t0 < parts; t0 += 8) {
      typename P::Raw u[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (t0 + j < parts) u[j] = P::load(part_o + (pbase + int64_t(t0 + j) * heads) * dv + d);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (t0 + j < parts) {
          const float w = wgt[t0 + j];
          const float4 x = P::cvt(u[j]);
          acc.x = fmaf(x.x, w, acc.x);
          acc.y = fmaf(x.y, w, acc.y);
          acc.z = fmaf(x.z, w, acc.z);
          acc.w = fmaf(x.w, w, acc.w);
        }
    }
    const float4 o = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
    if (!isfinite(o.x) || !isfinite(o.y) || !isfinite(o.z) || !isfinite(o.w)) flag(err, DSR_ERR_NONFINITE);
    *reinterpret_cast<float4*>(out + (int64_t(b) * heads + h) * dv + d) = o;
  }
  if (sink == nullptr && threadIdx.x == 0) {
    out_m[int64_t(b) * heads + h] = stat[0];
    out_l[int64_t(b) * heads + h] = stat[1];
  }
}

template <int HG>
int launch_mla(const float* q, const uint16_t* kv_pool, const PoolAddr& kv, const int32_t* visible,
               const int32_t* topk, int64_t k, const uint16_t* swa, const int64_t* swa_ring, int64_t swa_rows,
               const int32_t* swa_len,
               float scale, uint16_t* part_o, float* part_m, float* part_l, int32_t* err,
               int64_t batch, int64_t heads, int tiles, cudaStream_t stream, bool pdl,
               const uint16_t* q_img, int64_t id_base, bool foreign_ok) {
  using L = MlaLayout<HG>;
  {
    int rc = set_max_smem(mla_decode_kernel<HG>, L::kAlloc, "mla decode");
    if (rc == DSR_OK) rc = set_max_smem(mla_persistent_kernel<HG>, L::kAlloc, "mla decode");
    if (rc != DSR_OK) return rc;
  }
  // row-gather tensor maps: one-row boxes of 64 columns over the pool and the SWA rows
  CUtensorMap kv_map, swa_map;
  int rc = encode_tmap_bf16_2d(&kv_map, kv_pool, kMlaD, uint64_t(kv.rows), 64, 1);
  if (rc != DSR_OK) return rc;
  rc = encode_tmap_bf16_2d(&swa_map, swa, kMlaD, uint64_t(swa_rows), 64, 1);
  if (rc != DSR_OK) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(tiles), unsigned(batch), unsigned(heads / HG));
  cfg.blockDim = dim3(kMlaThreads, 1, 1);
  cfg.dynamicSmemBytes = L::kAlloc;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  // more items than one wave (a batch): one persistent CTA per SM overlaps each
  // item's output with the next item's loads (the BF16 query image is required)
  const int64_t items = int64_t(tiles) * batch * (heads / HG);
  if (q_img != nullptr && items > sm_count()) {
    cfg.gridDim = dim3(unsigned(sm_count()), 1, 1);
    const cudaError_t e = cudaLaunchKernelEx(&cfg, mla_persistent_kernel<HG>, kv_map, swa_map, kv, swa_ring,
                                             swa_rows, visible, topk, int(k), swa_len,
                                             scale * kLog2e, part_o, part_m, part_l, err, int(heads),
                                             int(batch), tiles, q_img, id_base, int(foreign_ok));
    if (e != cudaSuccess) return fail(DSR_ECUDA, "mla launch: %s", cudaGetErrorString(e));
    return DSR_OK;
  }
  const cudaError_t e = cudaLaunchKernelEx(&cfg, mla_decode_kernel<HG>, kv_map, swa_map, q, kv, swa_ring,
                                           swa_rows, visible, topk, int(k), swa_len, scale * kLog2e, part_o,
                                           part_m, part_l, err,
                                           int(heads), q_img, id_base, int(foreign_ok));
  if (e != cudaSuccess) return fail(DSR_ECUDA, "mla launch: %s", cudaGetErrorString(e));
  return DSR_OK;
}

inline int mla_tiles(int64_t k) { return 1 + int((k + kMlaTile - 1) / kMlaTile); }

}  // namespace

size_t mla_workspace_bytes(int64_t batch, int64_t heads, int64_t k) {
  const size_t parts = size_t(batch) * mla_tiles(k) * heads;
  return parts * kMlaDv * 4 + 2 * parts * 4 + 256;
}

namespace {
template <typename T>
int launch_combine(const T* part_o, const float* part_m, const float* part_l,
                   int64_t parts, const float* sink, float* out, float* out_m, float* out_l,
                   int32_t* err, int64_t batch, int64_t heads, int64_t dv,
                   cudaStream_t stream, bool pdl) {
  DSR_REQUIRE(part_o && part_m && part_l && out && err, "lse_combine: null pointer");
  DSR_REQUIRE(sink != nullptr || (out_m != nullptr && out_l != nullptr),
              "lse_combine: an unnormalised combine needs out_m and out_l");
  DSR_REQUIRE(parts > 0 && parts <= 4096 && batch > 0 && batch <= 65535 && heads > 0 &&
                  heads <= 65535 && dv > 0 && dv <= 4096 && dv % 4 == 0,
              "lse_combine: invalid shape (dv must be a multiple of 4)");
  DSR_REQUIRE(aligned16(part_o) && aligned16(out), "lse_combine: part_o and out must be 16-byte aligned");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(batch), unsigned(heads), 1);
  cfg.blockDim = dim3(128, 1, 1);
  cfg.dynamicSmemBytes = size_t(parts) * 4;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const bool deep = batch * heads <= 2 * int64_t(sm_count());
  const cudaError_t e =
      deep ? cudaLaunchKernelEx(&cfg, lse_combine_kernel<T, 24>, part_o, part_m, part_l, int(parts), sink,
                                out, out_m, out_l, err, int(heads), int(dv))
           : cudaLaunchKernelEx(&cfg, lse_combine_kernel<T, 8>, part_o, part_m, part_l, int(parts), sink,
                                out, out_m, out_l, err, int(heads), int(dv));
  if (e != cudaSuccess) return fail(DSR_ECUDA, "lse_combine launch: %s", cudaGetErrorString(e));
  return DSR_OK;
}
}  // namespace

int launch_lse_combine(const float* part_o, const float* part_m, const float* part_l,
                       int64_t parts, const float* sink, float* out, float* out_m, float* out_l,
                       int32_t* err, int64_t batch, int64_t heads, int64_t dv,
                       cudaStream_t stream, bool pdl) {
  return launch_combine(part_o, part_m, part_l, parts, sink, out, out_m, out_l, err, batch, heads, dv,
                        stream, pdl);
}

namespace {
// The argument checks of a full (sink-normalised) or partial MLA decode; the
// SWA row count of the [batch, 128, 576] ring layout when swa_ring is null.
int mla_check(const float* q, const uint16_t* kv_pool, const int32_t* visible, const int32_t* topk, int64_t k,
              const uint16_t* swa, const int64_t* swa_ring, int64_t& swa_rows, const int32_t* swa_len,
              const float* sink, float scale, float* out, void* workspace, size_t workspace_bytes, int32_t* err,
              int64_t batch, int64_t heads, const uint16_t* q_img, int64_t id_base, bool partial, float* out_m,
              float* out_l) {
  DSR_REQUIRE(q_img == nullptr || aligned16(q_img), "sparse_mla_decode: query image must be 16-byte aligned");
  DSR_REQUIRE(q && kv_pool && visible && topk && swa && swa_len && out && err && workspace,
              "sparse_mla_decode: null pointer");
  DSR_REQUIRE(partial ? (sink == nullptr && out_m != nullptr && out_l != nullptr) : sink != nullptr,
              "sparse_mla_decode: a sink (full) or out_m and out_l (partial) are required");
  DSR_REQUIRE(id_base >= 0 && id_base < (int64_t(1) << 31), "sparse_mla_decode: invalid id base");
  DSR_REQUIRE(heads == 16 || heads == 32 || heads == 64 || heads == 128,
              "sparse_mla_decode: heads %lld not in {16,32,64,128}", (long long)heads);
  DSR_REQUIRE(batch > 0 && batch <= 65535, "sparse_mla_decode: invalid batch");
  DSR_REQUIRE(k >= 0 && k <= 8192, "sparse_mla_decode: k %lld outside [0, 8192]", (long long)k);
  if (swa_ring == nullptr) swa_rows = batch * DSR_SWA_ROWS;  // the [batch, 128, 576] ring layout
  DSR_REQUIRE(swa_rows > 0 && swa_rows < (int64_t(1) << 31), "sparse_mla_decode: invalid SWA rows");
  DSR_REQUIRE(isfinite(scale) && scale > 0.f, "invalid attention scale");
  DSR_REQUIRE(aligned16(q) && aligned16(kv_pool) && aligned16(swa),
              "sparse_mla_decode: q, kv_pool and swa must be 16-byte aligned");
  const size_t need = mla_workspace_bytes(batch, heads, k);
  DSR_REQUIRE(workspace_bytes >= need, "sparse_mla_decode: workspace %zu < %zu bytes",
              workspace_bytes, need);
  return DSR_OK;
}

// heads per CTA: the largest group (<= 64) whose grid still fits one wave of
// CTAs; smaller groups re-gather the same rows (L2 hits) to use more SMs
int mla_head_group(int64_t batch, int64_t heads, int tiles) {
  int hg = heads < 64 ? int(heads) : 64;
  while (hg > 16 && batch * tiles * (heads / (hg / 2)) <= sm_count()) hg /= 2;
  return hg;
}
}  // namespace

int launch_mla_decode(const float* q, const uint16_t* kv_pool, const PoolAddr& kv, const int32_t* visible,
                      const int32_t* topk, int64_t k, const uint16_t* swa, const int64_t* swa_ring,
                      int64_t swa_rows, const int32_t* swa_len, const float* sink, float scale, float* out,
                      void* workspace, size_t workspace_bytes, int32_t* err, int64_t batch,
                      int64_t heads, cudaStream_t stream, bool pdl, const uint16_t* q_img,
                      int64_t id_base, bool partial, float* out_m, float* out_l) {
  int rc = mla_check(q, kv_pool, visible, topk, k, swa, swa_ring, swa_rows, swa_len, sink, scale, out, workspace,
                     workspace_bytes, err, batch, heads, q_img, id_base, partial, out_m, out_l);
  if (rc != DSR_OK) return rc;
  const int tiles = mla_tiles(k);
  const size_t parts = size_t(batch) * tiles * heads;
  uint16_t* part_o = static_cast<uint16_t*>(workspace);  // bf16 tile partials
  float* part_m = reinterpret_cast<float*>(part_o + parts * kMlaDv);
  float* part_l = part_m + parts;
  const int hg = mla_head_group(batch, heads, tiles);
  switch (hg) {
    case 16:
      rc = launch_mla<16>(q, kv_pool, kv, visible, topk, k, swa, swa_ring, swa_rows, swa_len, scale, part_o,
                          part_m, part_l, err, batch, heads, tiles, stream, pdl, q_img, id_base, partial);
      break;
    case 32:
      rc = launch_mla<32>(q, kv_pool, kv, visible, topk, k, swa, swa_ring, swa_rows, swa_len, scale, part_o,
                          part_m, part_l, err, batch, heads, tiles, stream, pdl, q_img, id_base, partial);
      break;
    default:
      rc = launch_mla<64>(q, kv_pool, kv, visible, topk, k, swa, swa_ring, swa_rows, swa_len, scale, part_o,
                          part_m, part_l, err, batch, heads, tiles, stream, pdl, q_img, id_base, partial);
      break;
  }
  if (rc != DSR_OK) return rc;
  return launch_combine(part_o, part_m, part_l, tiles, sink, out, out_m, out_l, err, batch, heads,
                        kMlaDv, stream, pdl);
}

int fused_mla_units(size_t room, int64_t batch, int64_t heads, int64_t k) {
  if (batch <= 0 || k < 0 || k > 8192 || !(heads == 16 || heads == 32 || heads == 64 || heads == 128)) return 0;
  const int tiles = mla_tiles(k);
  const int hg = mla_head_group(batch, heads, tiles);
  const int64_t units = batch * tiles * (heads / hg);
  const size_t need = hg == 16 ? size_t(MlaLayout<16>::kBytes) : size_t(MlaLayout<32>::kBytes);
  return hg > 32 || units > sm_count() || need > room ? 0 : int(units);
}

int plan_fused_mla(MlaFuseLaunch* plan, size_t room, const float* q, const uint16_t* kv_pool, const PoolAddr& kv,
                   const int32_t* visible, const int32_t* topk, const uint16_t* swa, const int64_t* swa_ring,
                   int64_t swa_rows, const int32_t* swa_len, const float* sink, float scale, float* out,
                   void* workspace, size_t workspace_bytes, int32_t* err, int64_t batch, int64_t heads, int64_t k) {
  plan->args = MlaFuse{};
  int rc = mla_check(q, kv_pool, visible, topk, k, swa, swa_ring, swa_rows, swa_len, sink, scale, out, workspace,
                     workspace_bytes, err, batch, heads, nullptr, 0, false, nullptr, nullptr);
  if (rc != DSR_OK) return rc;
  const int tiles = mla_tiles(k);
  const int hg = mla_head_group(batch, heads, tiles);
  const int units = fused_mla_units(room, batch, heads, k);
  if (units == 0) return DSR_OK;  // separate kernels
  rc = encode_tmap_bf16_2d(&plan->kv_map, kv_pool, kMlaD, uint64_t(kv.rows), 64, 1);
  if (rc == DSR_OK) rc = encode_tmap_bf16_2d(&plan->swa_map, swa, kMlaD, uint64_t(swa_rows), 64, 1);
  if (rc != DSR_OK) return rc;
  const size_t parts = size_t(batch) * tiles * heads;
  MlaFuse& a = plan->args;
  a.q = q;
  a.kv_pool = kv_pool;
  a.kv = kv;
  a.swa_ring = swa_ring;
  a.swa_rows = swa_rows;
  a.swa_len = swa_len;
  a.sink = sink;
  a.scale_log2 = scale * kLog2e;
  a.part_o = static_cast<uint16_t*>(workspace);
  a.part_m = reinterpret_cast<float*>(a.part_o + parts * kMlaDv);
  a.part_l = a.part_m + parts;
  a.out = out;
  a.heads = int(heads);
  a.hg = hg;
  a.tiles = tiles;
  a.units = units;
  return DSR_OK;
}

}  // namespace dsr

extern "C" size_t dsr_mla_workspace_bytes(int64_t batch, int64_t heads, int64_t k) {
  return dsr::mla_workspace_bytes(batch, heads, k);
}

extern "C" int dsr_sparse_mla_decode(const float* q, const uint16_t* kv_pool, int64_t pool_blocks,
                                     const int32_t* block_table, int64_t table_stride,
                                     const int32_t* visible, const int32_t* topk, int64_t k,
                                     const uint16_t* swa, const int32_t* swa_len,
                                     const float* sink, float scale, float* out, void* workspace,
                                     size_t workspace_bytes, int32_t* err, int64_t batch,
                                     int64_t heads, void* stream) {
  dsr::clear_error();
  dsr::PoolAddr kv;
  const int rc = dsr::paged_addr(&kv, block_table, table_stride, pool_blocks, "sparse_mla_decode");
  if (rc != DSR_OK) return rc;
  return dsr::launch_mla_decode(q, kv_pool, kv, visible, topk, k, swa, nullptr, 0, swa_len, sink, scale, out,
                                workspace, workspace_bytes, err, batch, heads, dsr::as_stream(stream), false);
}

extern "C" int dsr_sparse_mla_decode_ring(const float* q, const uint16_t* kv_pool, int64_t kv_rows,
                                          const int64_t* kv_ring, const int32_t* visible, const int32_t* topk,
                                          int64_t k, const uint16_t* swa_pool, int64_t swa_rows,
                                          const int64_t* swa_ring, const int32_t* swa_len, const float* sink,
                                          float scale, float* out, void* workspace, size_t workspace_bytes,
                                          int32_t* err, int64_t batch, int64_t heads, void* stream) {
  dsr::clear_error();
  dsr::PoolAddr kv;
  int rc = dsr::ring_addr(&kv, kv_ring, kv_rows, "sparse_mla_decode_ring");
  if (rc != DSR_OK) return rc;
  DSR_REQUIRE(swa_ring != nullptr, "sparse_mla_decode_ring: null SWA ring descriptors");
  return dsr::launch_mla_decode(q, kv_pool, kv, visible, topk, k, swa_pool, swa_ring, swa_rows, swa_len, sink,
                                scale, out, workspace, workspace_bytes, err, batch, heads, dsr::as_stream(stream),
                                false);
}

extern "C" int dsr_sparse_mla_partial(const float* q, const uint16_t* kv_pool, int64_t pool_blocks,
                                      const int32_t* block_table, int64_t table_stride,
                                      const int32_t* visible, const int32_t* topk, int64_t k,
                                      int64_t id_base, const uint16_t* swa, const int32_t* swa_len,
                                      float scale, float* out_o, float* out_m, float* out_l,
                                      void* workspace, size_t workspace_bytes, int32_t* err,
                                      int64_t batch, int64_t heads, void* stream) {
  dsr::clear_error();
  dsr::PoolAddr kv;
  const int rc = dsr::paged_addr(&kv, block_table, table_stride, pool_blocks, "sparse_mla_partial");
  if (rc != DSR_OK) return rc;
  return dsr::launch_mla_decode(q, kv_pool, kv, visible, topk, k, swa, nullptr, 0, swa_len, nullptr, scale, out_o,
                                workspace, workspace_bytes, err, batch, heads, dsr::as_stream(stream), false,
                                nullptr, id_base, true, out_m, out_l);
}

extern "C" int dsr_lse_combine_packed(const float* packed, int64_t world, const float* sink,
                                      float* out, int32_t* err, int64_t batch, int64_t heads,
                                      void* stream) {
  dsr::clear_error();
  DSR_REQUIRE(packed && sink && out && err, "lse_combine_packed: null pointer");
  DSR_REQUIRE(world > 0 && world <= 64 && batch > 0 && batch <= 65535 && heads > 0 && heads <= 1024 &&
                  (batch * heads) % 2 == 0,
              "lse_combine_packed: invalid shape (batch * heads must be even)");
  DSR_REQUIRE(dsr::aligned16(packed) && dsr::aligned16(out),
              "lse_combine_packed: packed and out must be 16-byte aligned");
  dsr::lse_combine_packed_kernel<<<dim3(unsigned(batch), unsigned(heads), 1), 128, 0,
                                   dsr::as_stream(stream)>>>(packed, int(world), sink, out, err,
                                                             int(heads));
  return dsr::launch_status("lse_combine_packed launch");
}

extern "C" int dsr_lse_combine(const float* part_o, const float* part_m, const float* part_l,
                               int64_t parts, const float* sink, float* out, float* out_m,
                               float* out_l, int32_t* err, int64_t batch, int64_t heads,
                               int64_t dv, void* stream) {
  dsr::clear_error();
  return dsr::launch_lse_combine(part_o, part_m, part_l, parts, sink, out, out_m, out_l, err, batch,
                                 heads, dv, dsr::as_stream(stream), false);
}
