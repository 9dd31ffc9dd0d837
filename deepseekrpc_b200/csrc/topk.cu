// Exact per-row top-k selection over fp32 scores.
//
// Semantics follow TiledIndexer._select + merge_ranked
// (src/deepseekrpc/index_selection.py:9-19,119-120): the k largest scores,
// equal scores resolved towards the lower logical id (stable argsort by id,
// then stable descending argsort by score), output sorted ascending and padded
// with -1.
//
// Design: one thread-block cluster of 8 CTAs per row; CTA j owns the j-th
// contiguous eighth of the row (kept in shared memory when it fits).  Scores
// are mapped to order-preserving uint32 keys and the k-th largest key T is
// found by an 11/11/10-bit radix select whose histograms are reduced across
// the cluster through distributed shared memory.  The selected set is
// {key > T} plus the first (in id order) `need` entries with key == T, which
// reproduces the lower-id tie rule.  A warp-ballot ordered compaction then
// writes the ids in ascending order.  No global scratch memory is used.
#include <cooperative_groups.h>

#include "common.cuh"
#include "host_common.h"

#include <math_constants.h>

namespace cg = cooperative_groups;

namespace dsr {
namespace {

constexpr int kTkCluster = 8;
constexpr int kTkThreads = 512;
constexpr int kTkWarps = kTkThreads / 32;
constexpr int kTkBins = 2048;
constexpr int kTkResident = 40960;  // keys per CTA kept in shared memory (160 KiB)

struct TopkShared {
  uint32_t hist[2][kTkBins];
  uint32_t slice[kTkBins / kTkCluster];
  uint32_t slice_tot[kTkCluster];
  uint32_t cta_gt[kTkCluster];
  uint32_t cta_eq[kTkCluster];
  uint32_t warp_take[kTkWarps];
  uint32_t warp_off[kTkWarps];
  uint32_t warp_gt[kTkWarps];
  uint32_t warp_eq[kTkWarps];
  uint32_t bcast[4];
};

struct Select {
  uint32_t bin, above, total;
};

// Key of entry g of a row; 0 marks an absent entry (ids[g] < 0).  NaN sorts
// above +inf as in a torch descending sort.  No finite or infinite score maps
// to 0 (that would need the bit pattern 0xffffffff, a NaN).
__device__ __forceinline__ uint32_t entry_key(const float* srow, const int32_t* irow, int64_t g) {
  if (irow != nullptr && irow[g] < 0) return 0u;
  const float s = srow[g];
  if (isnan(s)) return 0xffffffffu;
  return score_key(s);
}

__device__ __forceinline__ uint32_t warp_sum_u32(uint32_t v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Finds, over the cluster-wide histogram (sum of every CTA's `hist`), the bin b
// such that count(bins > b) < need <= count(bins >= b).  Identical result in
// every CTA.  total = number of keys in the histogram; when total < need the
// result is {0, total, total}.
__device__ Select cluster_select(cg::cluster_group& cluster, TopkShared& sh, uint32_t* hist,
                                 int nbins, uint32_t need, unsigned rank) {
  const int per = nbins / kTkCluster;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  cluster.sync();  // every CTA's histogram is complete
  for (int b = threadIdx.x; b < per; b += blockDim.x) {
    uint32_t s = 0;
#pragma unroll
    for (int c = 0; c < kTkCluster; ++c) s += cluster.map_shared_rank(hist, c)[rank * per + b];
    sh.slice[b] = s;
  }
  __syncthreads();
  if (warp == 0) {
    uint32_t t = 0;
    for (int b = lane; b < per; b += 32) t += sh.slice[b];
    t = warp_sum_u32(t);
    if (lane < kTkCluster) cluster.map_shared_rank(sh.slice_tot, lane)[rank] = t;
  }
  cluster.sync();  // slice totals delivered; remote histogram reads finished
  if (warp == 0) {
    // lane 0 = highest slice
    const uint32_t tot = lane < kTkCluster ? sh.slice_tot[kTkCluster - 1 - lane] : 0u;
    uint32_t incl = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const uint32_t total = __shfl_sync(0xffffffffu, incl, 31);
    Select r{0u, total, total};
    if (total >= need && need > 0) {
      const unsigned hit = __ballot_sync(0xffffffffu, incl >= need);
      const int L = __ffs(hit) - 1;
      const uint32_t above_slice = __shfl_sync(0xffffffffu, incl - tot, L);
      const unsigned s = kTkCluster - 1 - L;
      const uint32_t* rs = cluster.map_shared_rank(sh.slice, s);
      const int bpl = per / 32;  // bins per lane (8 or 4)
      // lane 0 covers the top bpl bins of the slice
      const int top = per - lane * bpl;  // exclusive upper end
      uint32_t mine = 0;
      uint32_t vals[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        vals[i] = i < bpl ? rs[top - 1 - i] : 0u;
        mine += vals[i];
      }
      uint32_t pin = mine;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v = __shfl_up_sync(0xffffffffu, pin, o);
        if (lane >= o) pin += v;
      }
      const unsigned hit2 = __ballot_sync(0xffffffffu, above_slice + pin >= need);
      const int L2 = __ffs(hit2) - 1;
      if (lane == L2) {
        uint32_t cum = above_slice + pin - mine;
        int bin = top - 1;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (i < bpl) {
            if (cum + vals[i] >= need) {
              bin = top - 1 - i;
              break;
            }
            cum += vals[i];
          }
        }
        r.bin = s * per + bin;
        r.above = cum;
        r.total = total;
        sh.bcast[0] = r.bin;
        sh.bcast[1] = r.above;
        sh.bcast[2] = r.total;
      }
    } else if (lane == 0) {
      sh.bcast[0] = 0u;
      sh.bcast[1] = total;
      sh.bcast[2] = total;
    }
  }
  __syncthreads();
  return Select{sh.bcast[0], sh.bcast[1], sh.bcast[2]};
}

__global__ void __cluster_dims__(kTkCluster, 1, 1) __launch_bounds__(kTkThreads, 1)
    topk_kernel(const float* __restrict__ scores, const int32_t* __restrict__ ids,
                const int32_t* __restrict__ lengths, int32_t* __restrict__ out_ids,
                float* __restrict__ out_scores, int32_t* err, int64_t row_stride, int k,
                int64_t id_base, int64_t resident_cap) {
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ TopkShared sh;
  extern __shared__ uint32_t keys[];
  const unsigned rank = cluster.block_rank();
  const int64_t row = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  pdl_wait();  // scores may come from the preceding kernel

  int64_t n = lengths[row];
  if (n < 0 || n > row_stride) {
    if (rank == 0 && tid == 0) flag(err, DSR_ERR_ID);
    n = 0;
  }
  const int64_t chunk = (n + kTkCluster - 1) / kTkCluster;
  const int64_t beg = rank * chunk;
  const int64_t cnt = n > beg ? (n - beg < chunk ? n - beg : chunk) : 0;
  const bool resident = chunk <= resident_cap;  // dynamic smem holds resident_cap keys
  const float* srow = scores + row * row_stride + beg;
  const int32_t* irow = ids != nullptr ? ids + row * row_stride + beg : nullptr;

  auto key_at = [&](int64_t i) -> uint32_t {
    return resident ? keys[i] : entry_key(srow, irow, i);
  };

  for (int i = tid; i < 2 * kTkBins; i += kTkThreads) (&sh.hist[0][0])[i] = 0u;
  __syncthreads();

  // pass 1: top 11 bits (load the chunk into shared memory when it fits)
  for (int64_t i = tid; i < cnt; i += kTkThreads) {
    const uint32_t u = entry_key(srow, irow, i);
    if (resident) keys[i] = u;
    if (u) atomicAdd(&sh.hist[0][u >> 21], 1u);
  }
  const Select s1 = cluster_select(cluster, sh, sh.hist[0], kTkBins, uint32_t(k), rank);
  for (int i = tid; i < kTkBins; i += kTkThreads) sh.hist[0][i] = 0u;
  const uint32_t total = s1.total;

  uint32_t T = 0u, need = 0u;
  if (total > uint32_t(k)) {
    const uint32_t need1 = uint32_t(k) - s1.above;
    const uint32_t p1 = s1.bin;
    // pass 2: next 11 bits among keys whose top 11 bits equal p1
    for (int64_t i = tid; i < cnt; i += kTkThreads) {
      const uint32_t u = key_at(i);
      if (u && (u >> 21) == p1) atomicAdd(&sh.hist[1][(u >> 10) & 2047u], 1u);
    }
    const Select s2 = cluster_select(cluster, sh, sh.hist[1], kTkBins, need1, rank);
    const uint32_t need2 = need1 - s2.above;
    const uint32_t p2 = (p1 << 11) | s2.bin;
    // pass 3: last 10 bits
    for (int64_t i = tid; i < cnt; i += kTkThreads) {
      const uint32_t u = key_at(i);
      if (u && (u >> 10) == p2) atomicAdd(&sh.hist[0][u & 1023u], 1u);
    }
    const Select s3 = cluster_select(cluster, sh, sh.hist[0], 1024, need2, rank);
    need = need2 - s3.above;
    T = (p2 << 10) | s3.bin;
  }

  // pass 4: per-warp counts of keys above T and equal to T (contiguous ranges)
  const int64_t sub = (cnt + kTkWarps - 1) / kTkWarps;
  const int64_t w_beg = warp * sub;
  const int64_t w_end = (w_beg + sub < cnt) ? w_beg + sub : cnt;
  {
    uint32_t gt = 0, eq = 0;
    for (int64_t i = w_beg + lane; i < w_end; i += 32) {
      const uint32_t u = key_at(i);
      gt += (u > T) ? 1u : 0u;
      eq += (u != 0u && u == T) ? 1u : 0u;
    }
    gt = warp_sum_u32(gt);
    eq = warp_sum_u32(eq);
    if (lane == 0) {
      sh.warp_gt[warp] = gt;
      sh.warp_eq[warp] = eq;
    }
  }
  __syncthreads();
  if (tid < kTkCluster) {
    uint32_t gt = 0, eq = 0;
    for (int w = 0; w < kTkWarps; ++w) {
      gt += sh.warp_gt[w];
      eq += sh.warp_eq[w];
    }
    cluster.map_shared_rank(sh.cta_gt, tid)[rank] = gt;
    cluster.map_shared_rank(sh.cta_eq, tid)[rank] = eq;
  }
  cluster.sync();
  if (tid == 0) {
    uint32_t eq_before = 0, off = 0;
    for (unsigned c = 0; c < rank; ++c) {
      const uint32_t left = need > eq_before ? need - eq_before : 0u;
      const uint32_t take = left < sh.cta_eq[c] ? left : sh.cta_eq[c];
      off += sh.cta_gt[c] + take;
      eq_before += sh.cta_eq[c];
    }
    for (int w = 0; w < kTkWarps; ++w) {
      const uint32_t left = need > eq_before ? need - eq_before : 0u;
      const uint32_t take = left < sh.warp_eq[w] ? left : sh.warp_eq[w];
      sh.warp_take[w] = take;
      sh.warp_off[w] = off;
      off += sh.warp_gt[w] + take;
      eq_before += sh.warp_eq[w];
    }
  }
  __syncthreads();

  // pass 5: ordered compaction, one warp per contiguous range
  {
    const uint32_t take = sh.warp_take[warp];
    uint32_t pos = sh.warp_off[warp], eq_seen = 0;
    int32_t* orow = out_ids + row * k;
    float* osrow = out_scores != nullptr ? out_scores + row * k : nullptr;
    const unsigned lt = (1u << lane) - 1u;
    for (int64_t j = w_beg; j < w_end; j += 32) {
      const int64_t i = j + lane;
      const uint32_t u = i < w_end ? key_at(i) : 0u;
      const bool eq = u != 0u && u == T;
      const unsigned eqb = __ballot_sync(0xffffffffu, eq);
      const uint32_t rank_eq = eq_seen + __popc(eqb & lt);
      const bool pick = (u > T) || (eq && rank_eq < take);
      const unsigned pb = __ballot_sync(0xffffffffu, pick);
      if (pick) {
        const uint32_t p = pos + __popc(pb & lt);
        if (p < uint32_t(k)) {
          orow[p] = irow != nullptr ? irow[i] : static_cast<int32_t>(id_base + beg + i);
          if (osrow != nullptr) osrow[p] = srow[i];
        }
      }
      eq_seen += __popc(eqb);
      pos += __popc(pb);
    }
  }
  // padding
  if (rank == 0) {
    const uint32_t chosen = total < uint32_t(k) ? total : uint32_t(k);
    for (int p = int(chosen) + tid; p < k; p += kTkThreads) {
      out_ids[row * k + p] = -1;
      if (out_scores != nullptr) out_scores[row * k + p] = -CUDART_INF_F;
    }
  }
  pdl_launch_dependents();
  cluster.sync();  // keep every CTA's shared memory alive until remote readers are done
}

}  // namespace

int launch_topk(const float* scores, const int32_t* ids, const int32_t* lengths, int32_t* out_ids,
                float* out_scores, int32_t* err, int64_t rows, int64_t row_stride, int64_t k,
                int64_t id_base, cudaStream_t stream, bool pdl) {
  DSR_REQUIRE(scores && lengths && out_ids && err, "topk_select: null pointer");
  DSR_REQUIRE(rows > 0 && rows <= 65535, "topk_select: rows %lld outside [1, 65535]",
              (long long)rows);
  DSR_REQUIRE(k > 0 && k <= 8192, "topk_select: k %lld outside [1, 8192]", (long long)k);
  DSR_REQUIRE(row_stride > 0 && row_stride <= (int64_t(1) << 31) - 1,
              "topk_select: invalid row stride");
  DSR_REQUIRE(id_base >= 0 && id_base + row_stride <= (int64_t(1) << 31),
              "topk_select: ids must fit int32");
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kTkResident * 4);
    configured = true;
  }
  const int64_t chunk = (row_stride + kTkCluster - 1) / kTkCluster;
  const size_t dyn = chunk <= kTkResident ? size_t(chunk) * 4 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kTkCluster, unsigned(rows), 1);
  cfg.blockDim = dim3(kTkThreads, 1, 1);
  cfg.dynamicSmemBytes = dyn;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, topk_kernel, scores, ids, lengths, out_ids,
                                           out_scores, err, row_stride, int(k), id_base,
                                           int64_t(dyn / 4));
  if (e != cudaSuccess) return fail(DSR_ECUDA, "topk launch: %s", cudaGetErrorString(e));
  return DSR_OK;
}

}  // namespace dsr

extern "C" int dsr_topk_select(const float* scores, const int32_t* ids, const int32_t* lengths,
                               int32_t* out_ids, float* out_scores, int32_t* err, int64_t rows,
                               int64_t row_stride, int64_t k, int64_t id_base, void* stream) {
  dsr::clear_error();
  return dsr::launch_topk(scores, ids, lengths, out_ids, out_scores, err, rows, row_stride, k,
                          id_base, dsr::as_stream(stream), false);
}
