// Exact per-row top-k selection over fp32 scores.
//
// Semantics follow TiledIndexer._select + merge_ranked
// (src/deepseekrpc/index_selection.py:9-19,119-120): the k largest scores,
// equal scores resolved towards the lower logical id (stable argsort by id,
// then stable descending argsort by score), output sorted ascending and padded
// with -1.
//
// Every entry gets a unique 63-bit composite key (u << 31) | (0x7fffffff - id),
// u = order-preserving uint32 of the score (-0.0 == +0.0): "larger key" is
// exactly "ranked earlier" under the reference rule, so the selected set is
// {key >= K*} where K* is the k-th largest key.
//
// Design (no grid-wide barrier, no spinning):
//   * a per-row 11-bit histogram of the score keys is built first, either by the
//     indexer epilogue while it produces the scores, or by topk_hist_kernel;
//   * topk_select_kernel spreads each row over many CTAs in 32-entry words.
//     Every CTA finds the threshold bin from the row histogram, writes one
//     bitmap word per 32 entries (bit set = key above the threshold bin) with a
//     warp ballot, and appends its threshold-bin entries to the row's candidate
//     list;
//   * the last CTA to finish a row (atomic ticket after a fence) resolves K*
//     among the candidates with local radix passes over the remaining 52 bits,
//     sets their bits, converts the bitmap into the ascending id list and
//     clears the row's histogram, ticket and candidate count for the next call.
// Candidate-list overflow (heavily tied scores) falls back to the last CTA
// resolving K* by scanning the whole row.  The workspace must be zero before
// its first use; every completed call leaves it zero again.
#include "common.cuh"
#include "host_common.h"

#include <math_constants.h>

namespace dsr {
namespace {

constexpr int kTkThreads = 256;
constexpr int kTkWarps = kTkThreads / 32;
constexpr int kTkBins = 2048;      // level-0 digit: 11 bits
constexpr int kTkCap = 8192;       // candidate entries per row
constexpr int kTkLocalCap = 2048;  // candidate entries one CTA stages in shared memory
constexpr int kTkLevels = 6;
__constant__ int kTkShift[kTkLevels] = {52, 41, 31, 20, 10, 0};
__constant__ int kTkBits[kTkLevels] = {11, 11, 10, 11, 10, 10};

__device__ __forceinline__ uint64_t composite(uint32_t u, uint32_t lo) {
  return (uint64_t(u) << 31) | uint64_t(lo);
}

struct TopkWs {
  size_t hist, done, count, cand_key, cand_idx, bits, total;
  int64_t words;  // bitmap words per row
  __host__ __device__ TopkWs(int64_t rows, int64_t row_stride) {
    words = (row_stride + 31) / 32;
    hist = 0;                                                    // [rows][2048] u32
    done = hist + size_t(rows) * kTkBins * 4;                    // [rows] u32 tickets
    count = done + ((size_t(rows) * 4 + 255) / 256) * 256;       // [rows] u32 candidates
    cand_key = count + ((size_t(rows) * 4 + 255) / 256) * 256;   // [rows][cap] u64 composite
    cand_idx = cand_key + size_t(rows) * kTkCap * 8;             // [rows][cap] u32 entry index
    bits = cand_idx + size_t(rows) * kTkCap * 4;                 // [rows][words] u32
    total = bits + ((size_t(rows) * words * 4 + 255) / 256) * 256;
  }
};

struct TopkShared {
  uint32_t hist[kTkBins];
  uint64_t lkey[kTkLocalCap];
  uint32_t lidx[kTkLocalCap];
  uint32_t scratch[2 * kTkWarps + 8];
  uint32_t nlocal, base, last;
};

struct Select {
  uint32_t bin, above, total;
};

// Score key of entry i of a row; 0 marks an absent entry (ids[i] < 0).  NaN
// sorts above +inf as in a torch descending sort; no score maps to 0.
__device__ __forceinline__ uint32_t entry_key(const float* srow, const int32_t* irow, int64_t i) {
  if (irow != nullptr && irow[i] < 0) return 0u;
  const float s = srow[i];
  if (isnan(s)) return 0xffffffffu;
  return score_key(s);
}

// Whole block: over h[0, nbins) (nbins in {1024, 2048}), the bin b with
// count(bins > b) < need <= count(bins >= b).  Same result in every thread;
// total < need (or need == 0) -> {0, total, total}.
__device__ Select block_find_bin(const uint32_t* h, int nbins, uint32_t need, TopkShared& sh) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bpt = nbins / kTkThreads;  // 8 or 4 bins per thread; thread 0 = top bins
  const int top = nbins - tid * bpt;
  uint32_t v[8], mine = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[i] = i < bpt ? h[top - 1 - i] : 0u;
    mine += v[i];
  }
  uint32_t incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t x = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += x;
  }
  __syncthreads();
  if (lane == 31) sh.scratch[warp] = incl;
  __syncthreads();
  uint32_t off = 0, total = 0;
  for (int w = 0; w < kTkWarps; ++w) {
    const uint32_t x = sh.scratch[w];
    off += w < warp ? x : 0u;
    total += x;
  }
  incl += off;
  const uint32_t excl = incl - mine;
  if (need > 0 && total >= need && excl < need && incl >= need) {
    uint32_t cum = excl;
    int bin = top - 1;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (i < bpt) {
        if (cum + v[i] >= need) {
          bin = top - 1 - i;
          break;
        }
        cum += v[i];
      }
    }
    sh.scratch[kTkWarps] = uint32_t(bin);
    sh.scratch[kTkWarps + 1] = cum;
  }
  __syncthreads();
  if (need == 0 || total < need) return Select{0u, total, total};
  return Select{sh.scratch[kTkWarps], sh.scratch[kTkWarps + 1], total};
}

// Word range [w0, w1) of CTA c over rows * words_per_row bitmap words.
__device__ __forceinline__ void cta_words(int64_t total_words, uint32_t c, uint32_t n, int64_t& w0,
                                          int64_t& w1) {
  w0 = total_words * c / n;
  w1 = total_words * (c + 1) / n;
}
// CTA owning word w (inverse of cta_words).
__device__ __forceinline__ uint32_t word_owner(int64_t w, int64_t total_words, uint32_t n) {
  int64_t c = w * int64_t(n) / total_words;
  while (c + 1 < int64_t(n) && total_words * (c + 1) / n <= w) ++c;
  while (c > 0 && total_words * c / n > w) --c;
  return uint32_t(c);
}

__device__ __forceinline__ int64_t row_length(const int32_t* lengths, int64_t r, int64_t row_stride) {
  const int64_t n = lengths[r];
  return (n < 0 || n > row_stride) ? 0 : n;
}

// ---------------------------------------------------------------------------
// Standalone histogram pass (the decode step gets it from the indexer).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kTkThreads) topk_hist_kernel(
    const float* __restrict__ scores, const int32_t* __restrict__ ids,
    const int32_t* __restrict__ lengths, int64_t rows, int64_t row_stride,
    uint8_t* __restrict__ ws_base) {
  __shared__ uint32_t hist[kTkBins];
  const TopkWs L(rows, row_stride);
  uint32_t* ghist = reinterpret_cast<uint32_t*>(ws_base + L.hist);
  for (int i = threadIdx.x; i < kTkBins; i += kTkThreads) hist[i] = 0u;
  pdl_launch_dependents();
  pdl_wait();
  int64_t w0, w1;
  cta_words(rows * L.words, blockIdx.x, gridDim.x, w0, w1);
  __syncthreads();
  for (int64_t r = w0 / L.words; r < rows && r * L.words < w1; ++r) {
    const int64_t n = row_length(lengths, r, row_stride);
    const int64_t rb = r * L.words;
    const int64_t e0 = (w0 > rb ? w0 - rb : 0) * 32;
    int64_t e1 = ((w1 < rb + L.words ? w1 : rb + L.words) - rb) * 32;
    if (e1 > n) e1 = n;
    const float* srow = scores + r * row_stride;
    const int32_t* irow = ids != nullptr ? ids + r * row_stride : nullptr;
    constexpr int kBatch = 8;
    for (int64_t i0 = e0; i0 < e1; i0 += int64_t(kTkThreads) * kBatch) {
      uint32_t u[kBatch];
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        const int64_t i = i0 + j * kTkThreads + threadIdx.x;
        u[j] = i < e1 ? entry_key(srow, irow, i) : 0u;
      }
#pragma unroll
      for (int j = 0; j < kBatch; ++j)
        if (u[j]) atomicAdd(&hist[u[j] >> 21], 1u);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < kTkBins; i += kTkThreads) {
      const uint32_t v = hist[i];
      if (v) {
        atomicAdd(ghist + r * kTkBins + i, v);
        hist[i] = 0u;
      }
    }
    __syncthreads();
  }
}

// The k-th largest composite among `count` keys whose digits above `level` are
// `prefix` (need = how many of them to take).  Whole block, shared histogram.
template <typename KeyAt>
__device__ uint64_t resolve_kstar(KeyAt key_at, int64_t count, uint64_t prefix, uint32_t need,
                                  TopkShared& sh) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int level = 1;
  for (; level < kTkLevels; ++level) {
    const int nb = 1 << kTkBits[level];
    const int hs = kTkShift[level - 1];  // digits above this one are fixed by `prefix`
    __syncthreads();
    for (int i = tid; i < nb; i += kTkThreads) sh.hist[i] = 0u;
    __syncthreads();
    for (int64_t i = tid; i < count; i += kTkThreads) {
      const uint64_t key = key_at(i);
      if (key && (key >> hs) == (prefix >> hs))
        atomicAdd(&sh.hist[uint32_t(key >> kTkShift[level]) & uint32_t(nb - 1)], 1u);
    }
    __syncthreads();
    const Select r1 = block_find_bin(sh.hist, nb, need, sh);
    need -= r1.above;
    prefix |= uint64_t(r1.bin) << kTkShift[level];
    if (sh.hist[r1.bin] == need) {  // the whole sub-bin is selected
      ++level;
      break;
    }
  }
  // K* = smallest key matching the resolved digits
  const int hs = kTkShift[level - 1];
  uint64_t best = ~uint64_t(0);
  for (int64_t i = tid; i < count; i += kTkThreads) {
    const uint64_t key = key_at(i);
    if (key && (key >> hs) == (prefix >> hs) && key < best) best = key;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const uint64_t other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other < best ? other : best;
  }
  __syncthreads();
  if (lane == 0) {
    sh.scratch[2 * warp] = uint32_t(best);
    sh.scratch[2 * warp + 1] = uint32_t(best >> 32);
  }
  __syncthreads();
  uint64_t kstar = ~uint64_t(0);
  for (int w = 0; w < kTkWarps; ++w) {
    const uint64_t v = (uint64_t(sh.scratch[2 * w + 1]) << 32) | sh.scratch[2 * w];
    kstar = v < kstar ? v : kstar;
  }
  __syncthreads();
  return kstar;
}

// ---------------------------------------------------------------------------
// Selection: bitmap words + candidates per CTA, resolution by the last CTA.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kTkThreads) topk_select_kernel(
    const float* __restrict__ scores, const int32_t* __restrict__ ids,
    const int32_t* __restrict__ lengths, int32_t* __restrict__ out_ids,
    float* __restrict__ out_scores, int32_t* err, int64_t rows, int64_t row_stride, int k,
    int64_t id_base, uint8_t* __restrict__ ws_base) {
  __shared__ __align__(16) TopkShared sh;
  const TopkWs L(rows, row_stride);
  uint32_t* ghist = reinterpret_cast<uint32_t*>(ws_base + L.hist);
  uint32_t* gdone = reinterpret_cast<uint32_t*>(ws_base + L.done);
  uint32_t* gcount = reinterpret_cast<uint32_t*>(ws_base + L.count);
  uint64_t* gkey = reinterpret_cast<uint64_t*>(ws_base + L.cand_key);
  uint32_t* gidx = reinterpret_cast<uint32_t*>(ws_base + L.cand_idx);
  uint32_t* gbits = reinterpret_cast<uint32_t*>(ws_base + L.bits);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t cta = blockIdx.x, nctas = gridDim.x;
  const int64_t total_words = rows * L.words;

  pdl_launch_dependents();  // the consumer may start its prologue; it waits for our completion
  pdl_wait();               // scores and histograms come from the preceding kernel
  int64_t w0, w1;
  cta_words(total_words, cta, nctas, w0, w1);

  for (int64_t r = w0 / L.words; r < rows && r * L.words < w1; ++r) {
    const int64_t rb = r * L.words;
    const int64_t n = row_length(lengths, r, row_stride);
    const int64_t a0 = w0 > rb ? w0 - rb : 0;                         // first word of the row
    const int64_t a1 = (w1 < rb + L.words ? w1 : rb + L.words) - rb;  // end word of the row
    const uint32_t first_cta = word_owner(rb, total_words, nctas);
    const uint32_t touching = word_owner(rb + L.words - 1, total_words, nctas) - first_cta + 1;
    if (cta == first_cta && tid == 0) {
      const int32_t len = lengths[r];
      if (len < 0 || len > row_stride) flag(err, DSR_ERR_ID);
    }
    const float* srow = scores + r * row_stride;
    const int32_t* irow = ids != nullptr ? ids + r * row_stride : nullptr;
    auto id_of = [&](int64_t i) -> int32_t {
      return irow != nullptr ? irow[i] : int32_t(id_base + i);
    };

    // threshold bin of the row
    for (int i = tid; i < kTkBins; i += kTkThreads) sh.hist[i] = ghist[r * kTkBins + i];
    if (tid == 0) sh.nlocal = 0u;
    __syncthreads();
    const Select s0 = block_find_bin(sh.hist, kTkBins, uint32_t(k), sh);
    const bool take_all = s0.total <= uint32_t(k);

    // one warp per bitmap word: ballot of "above the threshold bin"
    for (int64_t wd = a0 + warp; wd < a1; wd += kTkWarps) {
      const int64_t i = wd * 32 + lane;
      const uint32_t u = i < n ? entry_key(srow, irow, i) : 0u;
      const uint32_t d = u >> 21;
      const bool above = u != 0u && (take_all || d > s0.bin);
      const bool cand = !take_all && u != 0u && d == s0.bin;
      const unsigned word = __ballot_sync(0xffffffffu, above);
      if (lane == 0) gbits[r * L.words + wd] = word;
      const unsigned m = __ballot_sync(0xffffffffu, cand);
      if (m) {
        const int leader = __ffs(m) - 1;
        uint32_t slot = 0;
        if (lane == leader) slot = atomicAdd(&sh.nlocal, uint32_t(__popc(m)));
        slot = __shfl_sync(0xffffffffu, slot, leader) + __popc(m & ((1u << lane) - 1u));
        if (cand && slot < uint32_t(kTkLocalCap)) {
          sh.lkey[slot] = composite(u, 0x7fffffffu - uint32_t(id_of(i)));
          sh.lidx[slot] = uint32_t(i);
        }
      }
    }
    __syncthreads();
    const uint32_t nl = sh.nlocal;
    if (tid == 0) {
      // an overflowing CTA forces the whole-row path through an oversized count
      const uint32_t add = nl <= uint32_t(kTkLocalCap) ? nl : uint32_t(kTkCap) + 1u;
      sh.base = add ? atomicAdd(gcount + r, add) : 0u;
    }
    __syncthreads();
    for (uint32_t e = tid; e < nl && e < uint32_t(kTkLocalCap); e += kTkThreads) {
      const uint32_t slot = sh.base + e;
      if (slot < uint32_t(kTkCap)) {
        gkey[r * kTkCap + slot] = sh.lkey[e];
        gidx[r * kTkCap + slot] = sh.lidx[e];
      }
    }
    // ticket: the last CTA of the row finishes it
    __threadfence();
    __syncthreads();
    if (tid == 0) sh.last = atomicAdd(gdone + r, 1u) == touching - 1 ? 1u : 0u;
    __syncthreads();
    if (!sh.last) continue;
    __threadfence();

    // other CTAs' words and candidates are read from L2 (__ldcg), never a stale L1 line
    uint32_t* rbits = gbits + r * L.words;
    const uint32_t count = __ldcg(gcount + r);
    if (!take_all) {
      const uint64_t prefix0 = uint64_t(s0.bin) << kTkShift[0];
      const uint32_t need0 = uint32_t(k) - s0.above;
      const bool whole_bin = sh.hist[s0.bin] == need0;  // every threshold-bin entry is selected
      if (count <= uint32_t(kTkCap)) {
        // ---- radix over the candidates' remaining digits
        const uint64_t* ck = gkey + r * kTkCap;
        const uint64_t kstar =
            whole_bin ? 0ull
                      : resolve_kstar([&](int64_t i) { return __ldcg(ck + i); }, count, prefix0, need0, sh);
        for (uint32_t i = tid; i < count; i += kTkThreads)
          if (__ldcg(ck + i) >= kstar) {
            const uint32_t idx = __ldcg(gidx + r * kTkCap + i);
            atomicOr(rbits + (idx >> 5), 1u << (idx & 31));
          }
      } else {
        // ---- candidate overflow: resolve over the whole row, then mark its bin
        auto row_key = [&](int64_t i) -> uint64_t {
          const uint32_t u = entry_key(srow, irow, i);
          return u ? composite(u, 0x7fffffffu - uint32_t(id_of(i))) : 0ull;
        };
        const uint64_t kstar = whole_bin ? 0ull : resolve_kstar(row_key, n, prefix0, need0, sh);
        for (int64_t i = tid; i < n; i += kTkThreads) {
          const uint32_t u = entry_key(srow, irow, i);
          if (u && (u >> 21) == s0.bin && composite(u, 0x7fffffffu - uint32_t(id_of(i))) >= kstar)
            atomicOr(rbits + (i >> 5), 1u << (i & 31));
        }
      }
      __threadfence();
      __syncthreads();
    }

    // ---- bitmap -> ascending ids (contiguous words per thread, block scan)
    const int64_t nwords = (n + 31) / 32;
    const int64_t per = (nwords + kTkThreads - 1) / kTkThreads;
    const int64_t my0 = tid * per, my1 = my0 + per < nwords ? my0 + per : nwords;
    uint32_t mine = 0;
    for (int64_t wd = my0; wd < my1; ++wd) mine += __popc(__ldcg(rbits + wd));
    uint32_t incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t x = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += x;
    }
    __syncthreads();
    if (lane == 31) sh.scratch[warp] = incl;
    __syncthreads();
    uint32_t pos = incl - mine, total = 0;
    for (int w = 0; w < kTkWarps; ++w) {
      pos += w < warp ? sh.scratch[w] : 0u;
      total += sh.scratch[w];
    }
    int32_t* orow = out_ids + r * k;
    float* osrow = out_scores != nullptr ? out_scores + r * k : nullptr;
    for (int64_t wd = my0; wd < my1; ++wd) {
      uint32_t word = __ldcg(rbits + wd);
      while (word) {
        const int bit = __ffs(word) - 1;
        word &= word - 1;
        const int64_t i = wd * 32 + bit;
        if (pos < uint32_t(k)) {
          orow[pos] = id_of(i);
          if (osrow != nullptr) osrow[pos] = srow[i];
        }
        ++pos;
      }
    }
    const uint32_t chosen = total < uint32_t(k) ? total : uint32_t(k);
    for (int p = int(chosen) + tid; p < k; p += kTkThreads) {
      orow[p] = -1;
      if (osrow != nullptr) osrow[p] = -CUDART_INF_F;
    }
    // every CTA of the row is done with its state: clear it for the next call
    for (int i = tid; i < kTkBins; i += kTkThreads) ghist[r * kTkBins + i] = 0u;
    if (tid == 0) {
      gcount[r] = 0u;
      gdone[r] = 0u;
    }
    __syncthreads();
  }
}

int topk_ctas(int64_t rows, int64_t row_stride) {
  const int64_t words = rows * ((row_stride + 31) / 32);
  int64_t ctas = sm_count();
  if (words < ctas * 4) ctas = (words + 3) / 4;  // at least 4 words (128 entries) per CTA
  return int(ctas < 1 ? 1 : ctas);
}

}  // namespace

size_t topk_workspace_bytes(int64_t rows, int64_t row_stride) {
  return TopkWs(rows, row_stride).total;
}

size_t topk_zeroed_prefix_bytes(int64_t rows, int64_t row_stride) {
  return TopkWs(rows, row_stride).cand_key;
}

// hist_ready: the per-row histograms in the workspace were already built (by the
// indexer); otherwise topk_hist_kernel builds them first.
int launch_topk(const float* scores, const int32_t* ids, const int32_t* lengths, int32_t* out_ids,
                float* out_scores, int32_t* err, int64_t rows, int64_t row_stride, int64_t k,
                int64_t id_base, void* workspace, size_t workspace_bytes, cudaStream_t stream,
                bool pdl, bool hist_ready) {
  DSR_REQUIRE(scores && lengths && out_ids && err && workspace, "topk_select: null pointer");
  DSR_REQUIRE(rows > 0 && rows <= 65535, "topk_select: rows %lld outside [1, 65535]",
              (long long)rows);
  DSR_REQUIRE(k > 0 && k <= 8192, "topk_select: k %lld outside [1, 8192]", (long long)k);
  DSR_REQUIRE(row_stride > 0 && row_stride <= (int64_t(1) << 31) - 1,
              "topk_select: invalid row stride");
  DSR_REQUIRE(id_base >= 0 && id_base + row_stride <= (int64_t(1) << 31),
              "topk_select: ids must fit int32");
  const TopkWs L(rows, row_stride);
  DSR_REQUIRE(workspace_bytes >= L.total, "topk_select: workspace %zu < %zu bytes",
              workspace_bytes, L.total);
  DSR_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255u) == 0,
              "topk_select: workspace must be 256-byte aligned");
  const int ctas = topk_ctas(rows, row_stride);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(ctas), 1, 1);
  cfg.blockDim = dim3(kTkThreads, 1, 1);
  cfg.stream = stream;
  cfg.attrs = attr;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (!hist_ready) {
    cfg.numAttrs = pdl ? 1 : 0;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, topk_hist_kernel, scores, ids, lengths, rows,
                                             row_stride, ws);
    if (e != cudaSuccess) return fail(DSR_ECUDA, "topk histogram launch: %s", cudaGetErrorString(e));
    cfg.numAttrs = 1;
  } else {
    cfg.numAttrs = pdl ? 1 : 0;
  }
  const cudaError_t e = cudaLaunchKernelEx(&cfg, topk_select_kernel, scores, ids, lengths, out_ids,
                                           out_scores, err, rows, row_stride, int(k), id_base, ws);
  if (e != cudaSuccess) return fail(DSR_ECUDA, "topk launch: %s", cudaGetErrorString(e));
  return DSR_OK;
}

}  // namespace dsr

extern "C" size_t dsr_topk_workspace_bytes(int64_t rows, int64_t row_stride) {
  return dsr::topk_workspace_bytes(rows, row_stride);
}

extern "C" int dsr_topk_select(const float* scores, const int32_t* ids, const int32_t* lengths,
                               int32_t* out_ids, float* out_scores, int32_t* err, int64_t rows,
                               int64_t row_stride, int64_t k, int64_t id_base, void* workspace,
                               size_t workspace_bytes, void* stream) {
  dsr::clear_error();
  return dsr::launch_topk(scores, ids, lengths, out_ids, out_scores, err, rows, row_stride, k,
                          id_base, workspace, workspace_bytes, dsr::as_stream(stream), false, false);
}
