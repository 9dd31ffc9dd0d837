// Exact per-row top-k selection fused into the decode indexer (sm_100a).
//
// Semantics: TiledIndexer._select + merge_ranked (src/deepseekrpc/index_selection.py:
// 9-19,79-124): per row the k largest scores, equal scores resolved towards the
// lower id, NaN above +inf, -0.0 == +0.0; ids ascending, -1 padded.  Every entry
// has a unique 63-bit rank key (u << 31) | (0x7fffffff - id), u the
// order-preserving uint32 of its score, so the selection is {key >= K*} with K*
// the k-th largest key.  Digit 0 of a key is u >> 21 (11 bits), digit 1 the next
// 11 bits (key bits 41..51).
//
// The indexer kernel runs this after scoring, in every CTA of its cooperative
// grid (one CTA per SM), on the positions that CTA scored:
//   1. rows of at most k keys take every key (slot = position) before any
//      synchronisation; the epilogue added every score of the other rows to its
//      row's digit-0 histogram, and one grid barrier completes the histograms;
//   2. every CTA finds each of its rows' threshold bin b0, appends its
//      candidates (digit 0 >= b0), in position order, to the row's candidate
//      list as one block (one atomic gives its base and arrival number; a
//      record {base, length, CTA rank} goes under that number), adds the digit 1
//      of its threshold-bin candidates to the row's digit-1 histogram (one
//      thread per candidate), and counts itself done with the row (one 64-bit
//      atomic that also returns the list's length and the number of blocks);
//   3. the row's last CTA to finish step 2 (no waiting: the others have left the
//      row) loads the list, the block records and the digit-1 histogram (one
//      round trip), finds K* (the whole sub-bin of
//      digit 1 selected, or the rank among its few keys), writes the ids (and
//      scores) of the keys >= K* in position order -- blocks follow their CTAs,
//      whose ranks follow positions -- and clears the row's workspace.
// A row whose threshold bin holds more entries than its list has room for
// (massive ties) is resolved by its last CTA from the row's scores.
//
// This code runs once per CTA and launch, so its loops stay rolled: unrolled
// straight-line code would be fetched into the instruction cache once and never
// reused, and instruction fetch would dominate.
#pragma once

#include <math_constants.h>

#include "common.cuh"

namespace dsr {

constexpr int kSelBins = 2048;    // digits 0 and 1: 11 bits each
constexpr int kSelBinCap = 8192;  // threshold-bin entries of a row on the parallel path
constexpr int kSelMaxK = 8192;    // largest k of the fused selection
constexpr int kSelLevels = 6;
__device__ __constant__ int kSelShift[kSelLevels] = {52, 41, 31, 20, 10, 0};
__device__ __constant__ int kSelBits[kSelLevels] = {11, 11, 10, 11, 10, 10};

struct SelectArgs {
  int32_t* out_ids;    // [batch, k]: ids ascending, -1 padded (nullptr: no selection)
  float* out_scores;   // [batch, k]: the selected scores, -inf padded (nullable)
  int k;
  int64_t id_base;     // id of position p = id_base + p
  uint32_t* hist;      // [batch][2048] digit-0 histograms, built by the indexer epilogue
  uint32_t* hist1;     // [batch][2048] digit-1 histograms of each row's threshold-bin candidates
  uint32_t* ctl;       // [64]: [0] barrier arrivals, [1] exits, [2] attention tickets, [3] attention units done
  // [batch]: (CTAs done with the row << 48) | (blocks appended << 32) | candidate-list length
  unsigned long long* row_state;
  uint64_t* list;      // [batch][list_cap] candidate rank keys, one position-ordered block per CTA
  int list_cap;
  uint4* blocks;       // [batch][grid]: the row's i-th appended block {list base, length, CTA rank, -}
  // [batch]: 1 once a row of more than k keys has its top-k written (released by
  // its finisher; read by the fused attention); the grid's last CTA clears it
  uint32_t* ready;
  // [batch][gstride] (nullable): per 32-key group (4 per 128-key tile, tile index
  // within the row) the largest digit 0 of its scores, 0 for an empty group;
  // written by the indexer epilogue for rows of more than k keys, so a CTA with a
  // long range stages only the groups that reach the threshold bin
  uint16_t* gmax;
  int64_t gstride;
};

// Workspace: hist | hist1 | ctl | row_state | ready | list | blocks.  Everything
// before the list must be zero before the first launch; every completed launch
// leaves it zero again (list and blocks need no clearing).
struct SelectLayout {
  size_t hist, hist1, ctl, state, ready, list, blocks, total;
  int64_t cap;
  __host__ __device__ SelectLayout(int64_t batch, int64_t k, int64_t grid) {
    cap = (kSelBinCap + k + 1) & ~int64_t(1);
    hist = 0;
    hist1 = hist + size_t(batch) * kSelBins * 4;
    ctl = hist1 + size_t(batch) * kSelBins * 4;
    state = ctl + 256;
    ready = state + ((size_t(batch) * 8 + 255) / 256) * 256;
    list = ready + ((size_t(batch) * 4 + 255) / 256) * 256;
    blocks = list + size_t(batch) * size_t(cap) * 8;
    total = blocks + size_t(batch) * size_t(grid) * 16;
  }
  // leading bytes that must be zero at launch
  __host__ __device__ size_t zeroed() const { return list; }
};

__device__ __forceinline__ uint32_t sel_rank_u(uint32_t raw) {
  if ((raw & 0x7fffffffu) > 0x7f800000u) return 0xffffffffu;  // NaN ranks above +inf
  return score_key(__uint_as_float(raw));
}
__device__ __forceinline__ uint64_t sel_key(uint32_t u, int64_t id) {
  return (uint64_t(u) << 31) | uint64_t(0x7fffffffu - uint32_t(id));
}
__device__ __forceinline__ int32_t sel_key_id(uint64_t key) {
  return int32_t(0x7fffffffu - (uint32_t(key) & 0x7fffffffu));
}
__device__ __forceinline__ float sel_key_score(uint64_t key) { return key_score(uint32_t(key >> 31)); }

// Atomic add with acquire-release semantics at GPU scope: the CTA's writes
// before it (ordered by a CTA barrier) are visible to whoever observes the new
// value, and whatever the observed old value published is visible after it.
__device__ __forceinline__ unsigned long long atom_add_acq_rel(unsigned long long* p, unsigned long long v) {
  unsigned long long old;
  asm volatile("atom.acq_rel.gpu.global.add.u64 %0, [%1], %2;" : "=l"(old) : "l"(p), "l"(v) : "memory");
  return old;
}

// ---------------------------------------------------------------- grid barrier
// Every CTA of the (cooperative, fully resident) grid arrives once per barrier;
// barrier n completes when the arrival count reaches n * gridDim.x.  A wait that
// exceeds kWaitNs sets DSR_ERR_TIMEOUT and returns false; the CTA then skips its
// remaining work but still arrives at later barriers.
__device__ __forceinline__ bool grid_barrier(uint32_t* arrivals, uint32_t n, int32_t* err) {
  __syncthreads();
  int ok = 1;
  if (threadIdx.x == 0) {
    // release: the CTA's writes before the barrier (ordered by __syncthreads) go with the arrival
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(arrivals) : "memory");
    const uint32_t target = n * gridDim.x;
    const uint64_t start = global_ns();
    for (uint32_t spin = 0;; ++spin) {
      uint32_t v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(arrivals) : "memory");
      if (int32_t(v - target) >= 0) break;
      if ((spin & 15u) == 15u && global_ns() - start > kWaitNs) {
        flag(err, DSR_ERR_TIMEOUT);
        ok = 0;
        break;
      }
    }
  }
  return __syncthreads_and(ok) != 0;
}

// ------------------------------------------------------------- block helpers
template <int kThreads>
__device__ __forceinline__ uint32_t sel_excl_scan(uint32_t v, uint32_t& total, uint32_t* scratch) {
  constexpr int kWarps = kThreads / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t x = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += x;
  }
  __syncthreads();
  if (lane == 31) scratch[warp] = incl;
  __syncthreads();
  uint32_t off = 0;
  total = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    const uint32_t x = scratch[w];
    off += w < warp ? x : 0u;
    total += x;
  }
  return off + incl - v;
}

// The bin b of h[0, nbins) with count(bins > b) < need <= count(bins >= b)
// (1 <= need <= the total); `above` = count(bins > b).  Same in every thread.
template <int kThreads>
__device__ uint32_t sel_find_bin(const uint32_t* h, int nbins, uint32_t need, uint32_t& above,
                                 uint32_t* scratch) {
  const int per = (nbins + kThreads - 1) / kThreads;  // bins per thread, taken from the top
  const int hi = nbins - int(threadIdx.x) * per;
  uint32_t mine = 0;
#pragma unroll 1
  for (int i = 0; i < per; ++i) {
    const int b = hi - 1 - i;
    mine += b >= 0 ? h[b] : 0u;
  }
  uint32_t total;
  const uint32_t excl = sel_excl_scan<kThreads>(mine, total, scratch);
  if (excl < need && excl + mine >= need) {
    uint32_t cum = excl;
#pragma unroll 1
    for (int i = 0; i < per; ++i) {
      const int b = hi - 1 - i;
      if (b < 0) break;
      if (cum + h[b] >= need) {
        scratch[32] = uint32_t(b);
        scratch[33] = cum;
        break;
      }
      cum += h[b];
    }
  }
  __syncthreads();
  above = scratch[33];
  const uint32_t bin = scratch[32];
  __syncthreads();
  return bin;
}

template <int kThreads>
__device__ uint64_t sel_block_min(uint64_t v, uint32_t* scratch) {
  constexpr int kWarps = kThreads / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const uint64_t x = __shfl_xor_sync(0xffffffffu, v, o);
    v = x < v ? x : v;
  }
  __syncthreads();
  if (lane == 0) reinterpret_cast<uint64_t*>(scratch)[warp] = v;
  __syncthreads();
  uint64_t m = ~uint64_t(0);
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    const uint64_t x = reinterpret_cast<uint64_t*>(scratch)[w];
    m = x < m ? x : m;
  }
  __syncthreads();
  return m;
}

// The need-th largest of the n keys key_at(i) whose digits above `level` equal
// `prefix`'s (1 <= need <= their count), resolved digit by digit with a
// shared-memory histogram `hist` (>= 2048 words).
template <int kThreads, typename KeyAt>
__device__ uint64_t sel_kstar(KeyAt key_at, int64_t n, uint64_t prefix, uint32_t need, int level,
                              uint32_t* hist, uint32_t* scratch) {
  int shift = kSelShift[level - 1];
  for (; level < kSelLevels; ++level) {
    const int nb = 1 << kSelBits[level], sh = kSelShift[level], hs = kSelShift[level - 1];
#pragma unroll 1
    for (int i = threadIdx.x; i < nb; i += kThreads) hist[i] = 0u;
    __syncthreads();
#pragma unroll 1
    for (int64_t i = threadIdx.x; i < n; i += kThreads) {
      const uint64_t key = key_at(i);
      if ((key >> hs) == (prefix >> hs)) atomicAdd(&hist[uint32_t(key >> sh) & uint32_t(nb - 1)], 1u);
    }
    __syncthreads();
    uint32_t above;
    const uint32_t bin = sel_find_bin<kThreads>(hist, nb, need, above, scratch);
    need -= above;
    prefix |= uint64_t(bin) << sh;
    shift = sh;
    const bool whole = hist[bin] == need;  // every key of the sub-bin is selected
    __syncthreads();
    if (whole) break;
  }
  uint64_t best = ~uint64_t(0);
#pragma unroll 1
  for (int64_t i = threadIdx.x; i < n; i += kThreads) {
    const uint64_t key = key_at(i);
    if ((key >> shift) == (prefix >> shift) && key < best) best = key;
  }
  return sel_block_min<kThreads>(best, scratch);
}

// Ordered compaction of a run of entries: every thread holds up to kPer entries
// of consecutive groups (entry j of thread t is entry j * kThreads + t), `keep`
// a bitmask; `put(index, j)` receives the kept entries' output indices (base +
// their rank in entry order); returns the count.  `grp` holds kPer * warps words.
template <int kThreads, int kPer, typename Put>
__device__ uint32_t sel_compact(uint32_t keep, uint32_t base, uint32_t* grp, uint32_t* scratch, Put put) {
  constexpr int kWarps = kThreads / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned bal[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    bal[j] = __ballot_sync(0xffffffffu, (keep >> j) & 1u);
    if (lane == 0) grp[j * kWarps + warp] = __popc(bal[j]);
  }
  __syncthreads();
  uint32_t total;
  const uint32_t g = threadIdx.x < kPer * kWarps ? grp[threadIdx.x] : 0u;
  const uint32_t off = sel_excl_scan<kThreads>(g, total, scratch);
  if (threadIdx.x < kPer * kWarps) grp[threadIdx.x] = off;
  __syncthreads();
  const unsigned lt = (1u << lane) - 1u;
#pragma unroll
  for (int j = 0; j < kPer; ++j)
    if ((keep >> j) & 1u) put(base + grp[j * kWarps + warp] + __popc(bal[j] & lt), j);
  __syncthreads();
  return total;
}

}  // namespace dsr
