// Exact per-row top-k selection over fp32 scores.
//
// Semantics follow TiledIndexer._select + merge_ranked
// (src/deepseekrpc/index_selection.py:9-19,119-120): the k largest scores,
// equal scores resolved towards the lower logical id (stable argsort by id,
// then stable descending argsort by score), output sorted ascending and padded
// with -1.
//
// Every entry gets a unique 63-bit rank key (u << 31) | (0x7fffffff - id),
// u = order-preserving uint32 of the score (-0.0 == +0.0, NaN above +inf):
// "larger key" is exactly "ranked earlier" under the reference rule, so the
// selected set is {key >= K*} where K* is the k-th largest key.  Digit 0 of a
// key is u >> 21 (11 bits), digit 1 is the next 11 bits of u.
//
// Design (no grid-wide barrier), one launch:
//   * a per-row histogram of digit 0 is built first, by the indexer epilogue
//     while it produces the scores, or by topk_hist_kernel;
//   * topk_select_kernel spreads each row over the CTAs in 32-entry words.
//     Every CTA streams its range through a ring of bulk copies into shared
//     memory (kTkStages chunks in flight), finds the threshold bin of digit 0
//     from the row histogram, stages its entries at or above that bin
//     (compacted, in entry order, as their rank keys, the count padded to
//     even with a 0 record, which no entry's key equals) in the row's staging
//     area, counts the digit 1 of its threshold-bin entries into a second row
//     histogram, and takes a ticket;
//   * the CTA that takes the last ticket of a row copies all staged records
//     into shared memory at once (warp-wide 16-byte loads for short slots, one
//     bulk copy per long slot), reads the digit-1 histogram, ranks the few
//     entries that share both digits with K* pairwise, selects {key >= K*} with
//     one compare per record, and places the selected ids (and scores) in
//     entry order by two ballot passes around one block scan of per-(pass,
//     warp) counts; then it clears the row's histograms and ticket.
// More than kTkRankCap entries sharing K*'s two digits (massively tied scores)
// are ranked over the whole row; more than kTkRecCap staged records are walked
// from L2 in chunks.  The workspace must be zero before its first use; every
// completed call leaves its zeroed part zero again.  A bounded wait that gives
// up (a copy that never lands) sets DSR_ERR_TIMEOUT; the workspace must then be
// zeroed again.
#include "common.cuh"
#include "host_common.h"

#include <cooperative_groups.h>
#include <math_constants.h>

namespace dsr {
namespace {

constexpr int kTkThreads = 512;   // selection CTA
constexpr int kTkWarps = kTkThreads / 32;
constexpr int kTkBins = 2048;      // digits 0 and 1: 11 bits each
constexpr int kTkMaxCtas = 256;    // CTAs of one launch (one staged-count slot each; fits uint8)
constexpr int kHsThreads = 1024;  // histogram CTA
constexpr int kTkVec = 8;          // 4-entry runs per thread per histogram batch
constexpr int kTkChunk = kHsThreads * 4 * kTkVec;  // entries per histogram batch
// staging chunks: kTkThreads * kPer consecutive entries; kPer = 16 when a CTA
// streams long ranges of implicit-id rows (fixed per-chunk costs amortised),
// else 4 (short ranges, or an id array riding along in the ring)
constexpr int64_t kTkWideRange = 16384;  // entries per CTA from which chunks widen
constexpr int kTkStages = 4;       // staging chunks in flight (bulk copies)
// staged records the last CTA holds in shared memory: a threshold bin spans up to a
// quarter octave of scores, which for normal-like scores of 2^20-entry rows is
// about 11K records above the bin's lower edge
constexpr int kTkRecCap = 31 * kTkThreads;
constexpr int kTkRun = kTkRecCap / kTkThreads;  // records per thread there (at most)
constexpr size_t kTkRingBytes = size_t(kTkStages) * kTkThreads * 16 * 4;  // scores only, 16 per thread
constexpr size_t kTkDynSmem = size_t(kTkRecCap) * 8 > kTkRingBytes ? size_t(kTkRecCap) * 8 : kTkRingBytes;
static_assert(kTkDynSmem >= size_t(kTkStages) * kTkThreads * 4 * 8, "the ring with ids fits too");
static_assert(kTkRun * kTkWarps <= kTkThreads, "one output group per thread");
static_assert(kTkMaxCtas <= kTkThreads, "one thread per slot");
constexpr int kTkRegs = 8;         // staged records per thread per output chunk (strided)
constexpr int kTkSlotBatch = 10;   // slots per warp per batch of record loads (last CTA)
constexpr int kTkRowGroup = 32;    // rows staged before their finishing (one bit each)
constexpr int kTkRankCap = 2048;   // entries ranked in shared memory
constexpr int kTkLevels = 6;
__constant__ int kTkShift[kTkLevels] = {52, 41, 31, 20, 10, 0};
__constant__ int kTkBits[kTkLevels] = {11, 11, 10, 11, 10, 10};

__device__ __forceinline__ uint64_t composite(uint32_t u, uint32_t lo) {
  return (uint64_t(u) << 31) | uint64_t(lo);
}

// Order-preserving key of raw fp32 bits; NaN (any payload) above +inf.
__device__ __forceinline__ uint32_t rank_u(uint32_t raw) {
  if ((raw & 0x7fffffffu) > 0x7f800000u) return 0xffffffffu;
  return score_key(__uint_as_float(raw));
}

struct TopkWs {
  size_t hist, hist1, done, cnt, stage, total;
  int64_t words;    // 32-entry words per row
  int64_t sstride;  // staged records per row (row_stride rounded up to even)
  __host__ __device__ TopkWs(int64_t rows, int64_t row_stride) {
    words = (row_stride + 31) / 32;
    sstride = (row_stride + 1) & ~int64_t(1);
    hist = 0;                                                    // [rows][2048] u32 digit 0
    hist1 = hist + size_t(rows) * kTkBins * 4;                   // [rows][2048] u32 digit 1 of the threshold bin
    done = hist1 + size_t(rows) * kTkBins * 4;                   // [rows] u32 tickets
    cnt = done + ((size_t(rows) * 4 + 255) / 256) * 256;         // [rows][256] u32 staged per CTA
    stage = cnt + size_t(rows) * kTkMaxCtas * 4;                 // [rows][sstride] u64 records
    total = stage + ((size_t(rows) * size_t(sstride) * 8 + 255) / 256) * 256;
  }
};

struct TopkShared {
  uint32_t hist[kTkBins];
  uint64_t rank[kTkRankCap];
  uint32_t pre[kTkThreads + 1];  // exclusive prefix of staged counts per slot
  uint32_t e0s[kTkMaxCtas];      // first entry of each slot's range in the row
  uint32_t tot[2][kTkWarps];      // per-warp staged counts, by chunk parity
  uint32_t grp[kTkThreads];       // last CTA: selected counts, then offsets, of (record pass, warp) groups
  uint4 sink16;                   // target of the stores of lanes with nothing to store
  uint64_t recbar;                // last CTA: the long slots' bulk copies landed
  uint32_t sink4[2];
  uint32_t tot16[kTkRegs][kTkWarps];
  uint8_t map[kTkThreads * kTkRegs];  // chunk position -> slot
  uint32_t scratch[2 * kTkWarps + 8];
  uint64_t full[kTkStages];      // copy ring: chunk landed
  uint64_t kstar;
  uint32_t rbin[kTkRowGroup], rneed[kTkRowGroup], rwhole[kTkRowGroup];  // rows this CTA finishes
  uint32_t rfirst[kTkRowGroup], rtouch[kTkRowGroup], rlen[kTkRowGroup];
  uint32_t nrank, last;
  int abort;
};

struct Select {
  uint32_t bin, above, total;
};

// Score key of entry i of a row; 0 marks an absent entry (ids[i] < 0).
__device__ __forceinline__ uint32_t entry_key(const float* srow, const int32_t* irow, int64_t i) {
  if (irow != nullptr && irow[i] < 0) return 0u;
  return rank_u(__float_as_uint(srow[i]));
}

// Whole block: over h[0, nbins) (nbins in {1024, 2048}), the bin b with
// count(bins > b) < need <= count(bins >= b).  Same result in every thread;
// total < need (or need == 0) -> {0, total, total}.
__device__ Select block_find_bin(const uint32_t* h, int nbins, uint32_t need, TopkShared& sh) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bpt = nbins / kTkThreads;  // 4 or 2 bins per thread; thread 0 = top bins
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
    bool found = false;
#pragma unroll
    for (int i = 0; i < 8; ++i) {  // straight-line: no early exit
      const bool here = !found && i < bpt && cum + v[i] >= need;
      bin = here ? top - 1 - i : bin;
      cum += (!found && !here && i < bpt) ? v[i] : 0u;
      found = found || here;
    }
    sh.scratch[kTkWarps] = uint32_t(bin);
    sh.scratch[kTkWarps + 1] = cum;
  }
  __syncthreads();
  if (need == 0 || total < need) return Select{0u, total, total};
  return Select{sh.scratch[kTkWarps], sh.scratch[kTkWarps + 1], total};
}

// Exclusive block scan of one value per thread; `total` = the block's sum.
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t v, uint32_t& total, TopkShared& sh) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint32_t incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t x = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += x;
  }
  __syncthreads();
  if (lane == 31) sh.scratch[warp] = incl;
  __syncthreads();
  uint32_t off = 0;
  total = 0;
  for (int w = 0; w < kTkWarps; ++w) {
    off += w < warp ? sh.scratch[w] : 0u;
    total += sh.scratch[w];
  }
  return off + incl - v;
}

// CTA c of n takes the words [floor(T c / n), floor(T (c + 1) / n)) of T words
// (T < 2^43, n <= 256).  Divisions are long software routines on the GPU, so the
// host passes m = floor((2^64 - 1) / n) + 1: then floor(a / n) = umulhi(a, m)
// exactly for a < 2^52 (m = 2^64 / n + d with 0 < d <= 1 moves a / n by less
// than 2^-12, while its fraction stays at most 1 - 1/n <= 1 - 2^-8).
struct CtaSplit {
  int64_t total;       // T
  uint32_t n;
  uint64_t inv_n;      // m (unused for n == 1)
  double inv_total;    // 1 / T, for owner estimates
  int64_t words;       // words per row
  uint64_t inv_words;  // floor((2^64 - 1) / words) + 1 (unused for one word)
};
CtaSplit make_split(int64_t total, int64_t n, int64_t words) {
  CtaSplit s;
  s.total = total;
  s.n = uint32_t(n);
  s.inv_n = n > 1 ? ~uint64_t(0) / uint64_t(n) + 1u : 0u;
  s.inv_total = total > 0 ? 1.0 / double(total) : 0.0;
  s.words = words;
  s.inv_words = words > 1 ? ~uint64_t(0) / uint64_t(words) + 1u : 0u;
  return s;
}
// floor(w / words) for w < 2^43: umulhi is off by at most one (the error term
// stays below 1), fixed with one product each way
__device__ __forceinline__ int64_t row_of_word(const CtaSplit& s, int64_t w) {
  if (s.words == 1) return w;
  int64_t q = int64_t(__umul64hi(uint64_t(w), s.inv_words));
  if (q * s.words > w) --q;
  else if ((q + 1) * s.words <= w) ++q;
  return q;
}
__device__ __forceinline__ int64_t split_w0(const CtaSplit& s, int64_t c) {
  const uint64_t a = uint64_t(s.total) * uint64_t(c);
  return s.n == 1u ? int64_t(a) : int64_t(__umul64hi(a, s.inv_n));
}
__device__ __forceinline__ void cta_words(const CtaSplit& s, uint32_t c, int64_t& w0, int64_t& w1) {
  w0 = split_w0(s, c);
  w1 = split_w0(s, int64_t(c) + 1);
}
// CTA owning word w (inverse of cta_words): an estimate, then exact steps.
__device__ __forceinline__ uint32_t word_owner(const CtaSplit& s, int64_t w) {
  int64_t c = int64_t(double(w) * double(s.n) * s.inv_total);
  if (c > int64_t(s.n) - 1) c = int64_t(s.n) - 1;
  if (c < 0) c = 0;
  while (c + 1 < int64_t(s.n) && split_w0(s, c + 1) <= w) ++c;
  while (c > 0 && split_w0(s, c) > w) --c;
  return uint32_t(c);
}

__device__ __forceinline__ int64_t row_length(const int32_t* lengths, int64_t r, int64_t row_stride) {
  const int64_t n = lengths[r];
  return (n < 0 || n > row_stride) ? 0 : n;
}

// ---------------------------------------------------------------------------
// Standalone histogram pass (the decode step gets it from the indexer).
// ---------------------------------------------------------------------------
// Scores cluster in few digit-0 bins, and the lanes of a warp that add to one
// shared word serialise.  On long ranges every bin therefore has kHsCopies
// counters side by side (bin-major: word bin * kHsCopies + lane / 2), so the lanes
// holding one bin hit kHsCopies different banks; a pair of lanes shares a word.
// Short ranges use one counter per bin (less to clear and flush).
constexpr int kHsCopies = 16;
constexpr size_t kTkHistSmem = size_t(kTkBins) * kHsCopies * 4;
constexpr int64_t kTkHistSplit = 16384;  // entries per CTA from which the counters split

template <bool kIds>
__global__ void __launch_bounds__(kHsThreads) topk_hist_kernel(
    const float* __restrict__ scores, const int32_t* __restrict__ ids,
    const int32_t* __restrict__ lengths, int64_t rows, int64_t row_stride,
    uint8_t* __restrict__ ws_base, const CtaSplit split) {
  extern __shared__ uint32_t whist[];  // [kTkBins][copies]
  const TopkWs L(rows, row_stride);
  uint32_t* ghist = reinterpret_cast<uint32_t*>(ws_base + L.hist);
  const int tid = threadIdx.x;
  int64_t w0, w1;
  cta_words(split, blockIdx.x, w0, w1);
  const int copies = (w1 - w0) * 32 >= kTkHistSplit ? kHsCopies : 1;
  const uint32_t my_copy = copies > 1 ? uint32_t((tid & 31) >> 1) : 0u;
  for (int i = tid; i < copies * kTkBins; i += kHsThreads) whist[i] = 0u;
  pdl_launch_dependents();
  pdl_wait();
  __syncthreads();
  for (int64_t r = row_of_word(split, w0); r < rows && r * L.words < w1; ++r) {
    const int64_t n = row_length(lengths, r, row_stride);
    const int64_t rb = r * L.words;
    const int64_t e0 = (w0 > rb ? w0 - rb : 0) * 32;
    int64_t e1 = ((w1 < rb + L.words ? w1 : rb + L.words) - rb) * 32;
    if (e1 > n) e1 = n;
    const float* srow = scores + r * row_stride;
    const int32_t* irow = kIds ? ids + r * row_stride : nullptr;
    const bool vec = (reinterpret_cast<uintptr_t>(srow) & 15u) == 0 &&
                     (!kIds || (reinterpret_cast<uintptr_t>(irow) & 15u) == 0);
    for (int64_t c0 = e0; c0 < e1; c0 += kTkChunk) {
      uint32_t u[4 * kTkVec];
#pragma unroll
      for (int v = 0; v < kTkVec; ++v) {
        const int64_t i = c0 + int64_t(v) * 4 * kHsThreads + 4 * tid;
        if (vec && i + 3 < e1) {
          const uint4 s4 = *reinterpret_cast<const uint4*>(srow + i);
          u[4 * v] = rank_u(s4.x), u[4 * v + 1] = rank_u(s4.y);
          u[4 * v + 2] = rank_u(s4.z), u[4 * v + 3] = rank_u(s4.w);
          if (kIds) {
            const int4 i4 = *reinterpret_cast<const int4*>(irow + i);
            if (i4.x < 0) u[4 * v] = 0u;
            if (i4.y < 0) u[4 * v + 1] = 0u;
            if (i4.z < 0) u[4 * v + 2] = 0u;
            if (i4.w < 0) u[4 * v + 3] = 0u;
          }
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q) u[4 * v + q] = i + q < e1 ? entry_key(srow, irow, i + q) : 0u;
        }
      }
#pragma unroll
      for (int j = 0; j < 4 * kTkVec; ++j)
        if (u[j]) atomicAdd(&whist[(u[j] >> 21) * uint32_t(copies) + my_copy], 1u);
    }
    __syncthreads();
    for (int i = tid; i < kTkBins; i += kHsThreads) {
      uint32_t v = 0;
      for (int c = 0; c < copies; ++c) {
        const int w = i * copies + ((c + i) & (copies - 1));  // rotated: neighbouring bins on other banks
        v += whist[w];
        whist[w] = 0u;
      }
      if (v) atomicAdd(ghist + r * kTkBins + i, v);
    }
    __syncthreads();
  }
}

// The need-th largest rank key among the `count` keys whose digits above
// `level` equal those of `prefix`.  Whole block, shared histogram.
template <typename KeyAt>
__device__ uint64_t resolve_kstar(KeyAt key_at, int64_t count, uint64_t prefix, uint32_t need,
                                  int level, TopkShared& sh) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (; level < kTkLevels; ++level) {
    const int nb = 1 << kTkBits[level];
    const int hs = kTkShift[level - 1];  // digits above this one are fixed by `prefix`
    __syncthreads();
    for (int i = tid; i < nb; i += kTkThreads) sh.hist[i] = 0u;
    __syncthreads();
    for (int64_t i0 = 0; i0 < count; i0 += kTkThreads) {
      const int64_t i = i0 + tid;
      const uint64_t key = i < count ? key_at(i) : 0ull;
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
  for (int64_t i0 = 0; i0 < count; i0 += kTkThreads) {
    const int64_t i = i0 + tid;
    const uint64_t key = i < count ? key_at(i) : 0ull;
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

// Ticket: returns the old value; acq_rel at gpu scope.
__device__ __forceinline__ uint32_t ticket_add(uint32_t* p) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(p) : "memory");
  return old;
}

// A staged record is its entry's rank key; 0 is the pad record.
__device__ __forceinline__ uint64_t record_key(uint64_t rec) { return rec; }
__device__ __forceinline__ int32_t record_id(uint64_t rec) {
  return int32_t(0x7fffffffu - (uint32_t(rec) & 0x7fffffffu));
}
// The score of a staged record (canonical: -0.0 comes back as +0.0, every NaN as
// one NaN pattern, both ranking as the original did).
__device__ __forceinline__ float record_score(uint64_t rec) { return key_score(uint32_t(rec >> 31)); }

// ---------------------------------------------------------------------------
// Selection: staging by every CTA, resolution and output by the row's last CTA.
// ---------------------------------------------------------------------------
template <bool kIds, int kPer>
__global__ void __launch_bounds__(kTkThreads) topk_select_kernel(
    const float* __restrict__ scores, const int32_t* __restrict__ ids,
    const int32_t* __restrict__ lengths, int32_t* __restrict__ out_ids,
    float* __restrict__ out_scores, int32_t* err, int64_t rows, int64_t row_stride, int k,
    int64_t id_base, uint8_t* __restrict__ ws_base, const CtaSplit split) {
  __shared__ __align__(16) TopkShared sh;
  extern __shared__ __align__(128) uint8_t dyn[];  // copy ring, later the row's staged records
  const TopkWs L(rows, row_stride);
  uint32_t* ghist = reinterpret_cast<uint32_t*>(ws_base + L.hist);
  uint32_t* ghist1 = reinterpret_cast<uint32_t*>(ws_base + L.hist1);
  uint32_t* gdone = reinterpret_cast<uint32_t*>(ws_base + L.done);
  uint32_t* gcnt = reinterpret_cast<uint32_t*>(ws_base + L.cnt);
  uint64_t* gstage = reinterpret_cast<uint64_t*>(ws_base + L.stage);
  static_assert(kPer == 4 || (kPer == 16 && !kIds), "chunk width");
  constexpr int kTkPer = kPer;
  constexpr int kTkCh = kTkThreads * kTkPer;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t cta = blockIdx.x;
  if (tid == 0) {
    for (int s = 0; s < kTkStages; ++s) mbar_init(&sh.full[s], 1);
    mbar_init(&sh.recbar, 1);
    sh.abort = 0;
    fence_barrier_init();
  }
  __syncthreads();

  pdl_launch_dependents();  // the consumer may start its prologue; it waits for our completion
  pdl_wait();               // scores and histograms come from the preceding kernel
  int64_t w0, w1;
  cta_words(split, cta, w0, w1);
  uint32_t issued = 0;    // chunks this CTA has put on the copy ring (stage = n % kTkStages)
  uint32_t recphase = 0;  // rows whose long slots this CTA bulk-copied (phase of sh.recbar)

  const int64_t r_first = row_of_word(split, w0);
  const int64_t r_last = row_of_word(split, w1 + L.words - 1);  // ceil(w1 / words)
  const int64_t r_end = r_last < rows ? r_last : rows;
  for (int64_t rg = r_first; rg < r_end; rg += kTkRowGroup) {
    const int64_t rg_end = rg + kTkRowGroup < r_end ? rg + kTkRowGroup : r_end;
    uint32_t won = 0;  // rows of the group whose last ticket this CTA took
    // ---- every row of the group is staged first: finishing one row never
    // delays this CTA's share of the next
    for (int64_t r = rg; r < rg_end; ++r) {
      const int64_t rb = r * L.words;
      const int64_t n = row_length(lengths, r, row_stride);
      const int64_t a0 = w0 > rb ? w0 - rb : 0;                         // first word of the row
      const int64_t a1 = (w1 < rb + L.words ? w1 : rb + L.words) - rb;  // end word of the row
      const int64_t e0 = a0 * 32;
      const int64_t e1 = a1 * 32 < n ? a1 * 32 : n;  // this CTA's entries [e0, e1)
      const uint32_t first_cta = word_owner(split, rb);
      const uint32_t touching = word_owner(split, rb + L.words - 1) - first_cta + 1;
      if (cta == first_cta && tid == 0) {
        const int32_t len = lengths[r];
        if (len < 0 || len > row_stride) flag(err, DSR_ERR_ID);
      }
      const float* srow = scores + r * row_stride;
      const int32_t* irow = kIds ? ids + r * row_stride : nullptr;
      uint32_t* h0row = ghist + r * kTkBins;
      uint32_t* h1row = ghist1 + r * kTkBins;
      uint64_t* srec = gstage + r * L.sstride;

      // ---- chunks of kTkCh entries: thread tid takes the kTkPer consecutive
      // entries c0 + kTkPer * tid + q.  Aligned rows stream through a ring of
      // kTkStages bulk copies into shared memory (one elected thread issues them);
      // others are read with plain loads.
      const bool ring = (row_stride & 3) == 0 && (reinterpret_cast<uintptr_t>(srow) & 15u) == 0 &&
                        (!kIds || (reinterpret_cast<uintptr_t>(irow) & 15u) == 0);
      const int64_t nch = e1 > e0 ? (e1 - e0 + kTkCh - 1) / kTkCh : 0;
      const uint32_t first = issued;
      auto issue = [&](int64_t c) {  // elected thread: chunk c of the row onto its stage
        const uint32_t st = (first + uint32_t(c)) % kTkStages;
        const int64_t c0 = e0 + c * kTkCh;
        const int64_t cnt = ((e1 - c0 < kTkCh ? e1 - c0 : kTkCh) + 3) & ~int64_t(3);  // stays in the row
        const uint32_t bytes = uint32_t(cnt) * 4u;
        mbar_arrive_expect_tx(&sh.full[st], kIds ? 2u * bytes : bytes);
        bulk_load(smem_u32(dyn + size_t(st) * kTkCh * 4), srow + c0, bytes, &sh.full[st]);
        if (kIds)
          bulk_load(smem_u32(dyn + size_t(kTkStages + st) * kTkCh * 4), irow + c0, bytes, &sh.full[st]);
      };
      if (ring && tid == 0) {
        fence_proxy_async_smem();  // the records of a previous row were written through the generic proxy
        for (int64_t c = 0; c < nch && c < kTkStages; ++c) issue(c);
      }
      if (ring) issued += uint32_t(nch);

      // ---- row histogram -> threshold bin of digit 0
      uint32_t hv[kTkBins / kTkThreads];
  #pragma unroll
      for (int j = 0; j < kTkBins / kTkThreads; ++j) hv[j] = h0row[j * kTkThreads + tid];
  #pragma unroll
      for (int j = 0; j < kTkBins / kTkThreads; ++j) sh.hist[j * kTkThreads + tid] = hv[j];
      __syncthreads();
      const Select s0 = block_find_bin(sh.hist, kTkBins, uint32_t(k), sh);
      const bool take_all = s0.total <= uint32_t(k);
      const uint32_t need0 = uint32_t(k) - s0.above;
      const bool whole_bin = take_all || sh.hist[s0.bin] == need0;  // no entry left to rank
      // lowest score of the threshold bin; the edges of bins 0-3 decode to NaN bit
      // patterns and those bins hold nothing above -inf, so every score passes there
      const float thr_f = s0.bin < 4u ? -CUDART_INF_F : key_score(s0.bin << 21);

      // ---- stage entries at or above the threshold bin, compacted in entry order
      uint32_t staged = 0;  // block-uniform running count
      int64_t c = 0;
      bool aborted = false;
      for (; c < nch; ++c) {
        const int64_t i = e0 + c * kTkCh + int64_t(kTkPer) * tid;
        uint32_t raw[kTkPer];
        int32_t idv[kTkPer];
        bool ok = true;
        if (ring) {
          const uint32_t n_ = first + uint32_t(c);
          ok = mbar_wait(&sh.full[n_ % kTkStages], (n_ / kTkStages) & 1u, &sh.abort, err);
          const uint8_t* stage = dyn + size_t(n_ % kTkStages) * kTkCh * 4 + size_t(kTkPer) * 4 * tid;
  #pragma unroll
          for (int v = 0; v < kTkPer / 4; ++v) {
            const uint4 x = reinterpret_cast<const uint4*>(stage)[v];
            raw[4 * v] = x.x, raw[4 * v + 1] = x.y, raw[4 * v + 2] = x.z, raw[4 * v + 3] = x.w;
            if (kIds) {
              const int4 y = reinterpret_cast<const int4*>(stage + size_t(kTkStages) * kTkCh * 4)[v];
              idv[4 * v] = y.x, idv[4 * v + 1] = y.y, idv[4 * v + 2] = y.z, idv[4 * v + 3] = y.w;
            }
          }
        } else {
  #pragma unroll
          for (int q = 0; q < kTkPer; ++q) {
            const bool in = i + q < e1;
            raw[q] = in ? __float_as_uint(srow[i + q]) : 0u;
            if (kIds) idv[q] = in ? irow[i + q] : -1;
          }
        }
        // keep: at or above the threshold bin's lower edge, compared as floats (the
        // key map is monotone; NaN ranks above +inf); kept entries are rare, so
        // their keys, digit-1 counts and records are built in one branch, after
        // the block scan that places them
        uint32_t mask = 0;
        const int64_t room = ok ? e1 - i : 0;  // valid entries of this thread's run
  #pragma unroll
        for (int q = 0; q < kTkPer; ++q) {
          const float sv = __uint_as_float(raw[q]);
          const bool keep = q < room && (!kIds || idv[q] >= 0) && (take_all || sv >= thr_f || sv != sv);
          mask |= uint32_t(keep) << q;
        }
        const uint32_t cnt = __popc(mask);
        uint32_t incl = cnt;
  #pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        if (lane == 31) sh.tot[c & 1][warp] = incl;
        if (__syncthreads_or(!ok)) {  // a copy never landed: every thread leaves together
          aborted = true;
          break;
        }
        if (ring && tid == 0 && c + kTkStages < nch) issue(c + kTkStages);  // this stage is consumed
        uint32_t before = 0, all = 0;
  #pragma unroll
        for (int w = 0; w < kTkWarps; ++w) {
          const uint32_t t = sh.tot[c & 1][w];
          before += w < warp ? t : 0u;
          all += t;
        }
        if (mask != 0u) {
          uint32_t pos = staged + before + incl - cnt;
  #pragma unroll
          for (int q = 0; q < kTkPer; ++q)
            if ((mask >> q) & 1u) {
              const uint32_t u = rank_u(raw[q]);
              if (kIds && idv[q] == 0x7fffffff) flag(err, DSR_ERR_ID);  // reserved for the pad record
              if (!whole_bin && (u >> 21) == s0.bin) atomicAdd(h1row + ((u >> 10) & (kTkBins - 1)), 1u);
              const uint32_t id = kIds ? uint32_t(idv[q]) : uint32_t(id_base + i + q);
              srec[e0 + pos] = composite(u, 0x7fffffffu - id);
              ++pos;
            }
        }
        staged += all;
      }
      if (aborted) {
        // wait (bounded) for the copies still in flight, then leave; the status is set
        if (ring && tid == 0)
          for (int64_t d = c; d < nch && d < c + kTkStages; ++d) {
            const uint32_t n_ = first + uint32_t(d);
            mbar_drain(&sh.full[n_ % kTkStages], (n_ / kTkStages) & 1u);
          }
        return;
      }
      // an even count keeps every CTA's records 16-byte aligned for the last CTA's
      // copies; the pad record is 0, which no entry produces (ids < 2^31 - 1)
      if (staged & 1u) {
        if (tid == 0) srec[e0 + staged] = 0ull;
        ++staged;
      }
      if (tid == 0) gcnt[r * kTkMaxCtas + (cta - first_cta)] = staged;

      // ---- ticket: the last CTA of the row finishes it.  The barrier orders every
      // thread's records and counts before thread 0's acq_rel ticket (cumulative at
      // gpu scope); the last CTA's acquire and barrier order its reads after all.
      __syncthreads();
      if (tid == 0) sh.last = ticket_add(gdone + r) == touching - 1 ? 1u : 0u;
      __syncthreads();
      if (sh.last) {
        won |= 1u << uint32_t(r - rg);
        if (tid == 0) {
          sh.rbin[r - rg] = s0.bin;
          sh.rneed[r - rg] = need0;
          sh.rwhole[r - rg] = whole_bin ? 1u : 0u;
          sh.rfirst[r - rg] = first_cta;
          sh.rtouch[r - rg] = touching;
          sh.rlen[r - rg] = uint32_t(n);
        }
      }
    }
    __syncthreads();
    // ---- then the rows this CTA finishes
    for (uint32_t pend = won; pend; pend &= pend - 1) {
      const int64_t r = rg + (__ffs(pend) - 1);
      const int64_t rb = r * L.words;
      const int64_t n = sh.rlen[r - rg];  // row geometry from the staging pass
      const uint32_t first_cta = sh.rfirst[r - rg];
      const uint32_t touching = sh.rtouch[r - rg];
      const float* srow = scores + r * row_stride;
      const int32_t* irow = kIds ? ids + r * row_stride : nullptr;
      uint32_t* h0row = ghist + r * kTkBins;
      uint32_t* h1row = ghist1 + r * kTkBins;
      uint64_t* srec = gstage + r * L.sstride;
      const uint32_t bin0 = sh.rbin[r - rg], need0 = sh.rneed[r - rg];
      const bool whole_bin = sh.rwhole[r - rg] != 0u;

      // other CTAs' counts, records and digit-1 counts are read from L2 (__ldcg, cp.async.cg)
      uint32_t h1v[kTkBins / kTkThreads];
      if (!whole_bin) {
  #pragma unroll
        for (int j = 0; j < kTkBins / kTkThreads; ++j) h1v[j] = __ldcg(h1row + j * kTkThreads + tid);
      }
      const uint32_t my_cnt = uint32_t(tid) < touching ? __ldcg(gcnt + r * kTkMaxCtas + tid) : 0u;
      if (uint32_t(tid) < touching) {
        int64_t cw0, cw1;
        cta_words(split, first_cta + tid, cw0, cw1);
        sh.e0s[tid] = uint32_t((cw0 > rb ? cw0 - rb : 0) * 32);
      }
      uint32_t total_staged = 0;
      const uint32_t my_pre = block_excl_scan(my_cnt, total_staged, sh);
      sh.pre[tid] = my_pre;
      if (tid == 0) sh.pre[touching] = total_staged;
      // (slots >= touching are never searched: pre[touching] bounds every walk)
      const bool my_long = my_cnt > 64u;  // slot tid holds more than 32 pieces
      const bool long_slots = __syncthreads_or(my_long);

      // ---- up to kTkRecCap records: all of them into shared memory, in slot
      // order, as 16-byte pieces (counts are even).  A slot of up to 32 pieces
      // is copied by one warp's lanes: warp w takes slots w, w + 16, ...,
      // kTkSlotBatch slots per batch of loads (one L2 round trip; the batch lands
      // while digit 1 is resolved).  A longer slot (few CTAs per row, as in
      // prefill rows) is one bulk copy issued by its own thread.  No loop here has
      // a per-lane trip count: on this GPU a loop whose lanes leave at different
      // iterations costs a warp reconvergence of a few hundred cycles.
      const bool in_smem = total_staged <= uint32_t(kTkRecCap);
      uint64_t* recs = reinterpret_cast<uint64_t*>(dyn);
      uint4 piece[kTkSlotBatch];
      auto slot_range = [&](int slot, uint32_t& q0, uint32_t& q1) {
        const bool valid = slot < int(touching);
        q0 = valid ? sh.pre[slot] >> 1 : 0u;
        q1 = valid ? sh.pre[slot + 1] >> 1 : 0u;
      };
      // lanes without a piece store theirs to a sink word: a divergent branch
      // around a store costs more than the store
      auto load_slots = [&](int s0) {
  #pragma unroll
        for (int b = 0; b < kTkSlotBatch; ++b) {
          uint32_t q0, q1;
          slot_range(s0 + b * kTkWarps, q0, q1);
          if (q0 + lane < q1 && q1 - q0 <= 32u)
            piece[b] = __ldcg(reinterpret_cast<const uint4*>(srec + sh.e0s[s0 + b * kTkWarps]) + lane);
        }
      };
      auto store_slots = [&](int s0) {
  #pragma unroll
        for (int b = 0; b < kTkSlotBatch; ++b) {
          uint32_t q0, q1;
          slot_range(s0 + b * kTkWarps, q0, q1);
          uint4* dst = q0 + lane < q1 && q1 - q0 <= 32u ? reinterpret_cast<uint4*>(recs) + q0 + lane : &sh.sink16;
          *dst = piece[b];
        }
      };
      if (in_smem) {
        if (long_slots) {
          // every copying thread announces its bytes before any copy is issued, so
          // the barrier's pending bytes never drop below zero; thread 0 arrives
          fence_proxy_async_smem();  // the area was last written through the generic proxy
          if (my_long) mbar_expect_tx(&sh.recbar, my_cnt * 8u);
          __syncthreads();
          if (my_long) bulk_load(smem_u32(recs + sh.pre[tid]), srec + sh.e0s[tid], my_cnt * 8u, &sh.recbar);
          if (tid == 0) mbar_arrive(&sh.recbar);
        }
        load_slots(warp);
      }

      // digit 1 of K* (while the copies fly)
      uint32_t bin1 = 0, need1 = 0;
      bool sub_all = true;  // every threshold-bin entry with digit 1 == bin1 is selected
      if (!whole_bin) {
  #pragma unroll
        for (int j = 0; j < kTkBins / kTkThreads; ++j) sh.hist[j * kTkThreads + tid] = h1v[j];
        __syncthreads();
        const Select s1 = block_find_bin(sh.hist, kTkBins, need0, sh);
        bin1 = s1.bin;
        need1 = need0 - s1.above;
        sub_all = need1 == sh.hist[s1.bin];
      }
      const uint64_t prefix1 = (uint64_t(bin0) << kTkShift[0]) | (uint64_t(bin1) << kTkShift[1]);
      if (tid == 0) {
        sh.nrank = 0u;
        sh.kstar = prefix1;
      }
      auto shares_two_digits = [&](uint64_t key) { return (key >> kTkShift[1]) == (prefix1 >> kTkShift[1]); };
      auto selected = [&](uint64_t rec, uint64_t kstar) {
        const uint64_t key = record_key(rec);
        return rec != 0ull && (whole_bin || uint32_t(key >> kTkShift[0]) > bin0 || key >= kstar);
      };
      int32_t* orow = out_ids + r * k;
      float* osrow = out_scores != nullptr ? out_scores + r * k : nullptr;
      uint64_t kstar = prefix1;  // with sub_all: every key with those digits qualifies
      uint32_t chosen = 0;

      if (in_smem) {
        store_slots(warp);
        for (int s0 = warp + kTkWarps * kTkSlotBatch; s0 < int(touching); s0 += kTkWarps * kTkSlotBatch) {
          load_slots(s0);
          store_slots(s0);
        }
        if (long_slots) {
          const bool landed = mbar_wait(&sh.recbar, recphase & 1u, &sh.abort, err);
          ++recphase;
          if (__syncthreads_or(!landed)) {
            if (tid == 0) mbar_drain(&sh.recbar, (recphase - 1) & 1u);
            return;  // the status is set
          }
        } else {
          __syncthreads();
        }
        // record f = j * kTkThreads + tid is thread tid's j-th (j < nj, block-
        // uniform): every pass reads consecutive records per warp, and no loop has
        // a per-lane trip count (on this GPU a loop whose lanes leave at
        // different iterations costs a warp reconvergence of a few hundred cycles)
        const uint32_t nj = (total_staged + kTkThreads - 1) / kTkThreads;  // <= kTkRun
        auto rec_at = [&](uint32_t j) -> uint64_t {
          const uint32_t f = j * kTkThreads + uint32_t(tid);
          return f < total_staged ? recs[f] : 0ull;
        };
        if (!sub_all) {
          // ---- K* among the candidates: the records sharing its two digits
          const uint64_t p01 = prefix1 >> 41;  // kTkShift[1]
          for (uint32_t j = 0; j < nj; ++j) {
            const uint64_t rec = rec_at(j);
            if (rec != 0ull && (rec >> 41) == p01) {
              const uint32_t slot = atomicAdd(&sh.nrank, 1u);
              if (slot < uint32_t(kTkRankCap)) sh.rank[slot] = rec;
            }
          }
          __syncthreads();
          const uint32_t nr = sh.nrank;
          if (nr <= uint32_t(kTkThreads)) {
            // keys are unique: exactly one candidate has need1 - 1 candidates above it
            if (uint32_t(tid) < nr) {
              const uint64_t mine = sh.rank[tid];
              uint32_t above = 0;
              for (uint32_t j = 0; j < nr; ++j) above += sh.rank[j] > mine ? 1u : 0u;
              if (above == need1 - 1) sh.kstar = mine;
            }
            __syncthreads();
            kstar = sh.kstar;
          } else if (nr <= uint32_t(kTkRankCap)) {
            kstar = resolve_kstar([&](int64_t j) { return sh.rank[j]; }, nr, prefix1, need1, 2, sh);
          } else {
            auto row_key = [&](int64_t j) -> uint64_t {
              const uint32_t u = entry_key(srow, irow, j);
              const int32_t id = kIds ? irow[j] : int32_t(id_base + j);
              return u ? composite(u, 0x7fffffffu - uint32_t(id)) : 0ull;
            };
            kstar = resolve_kstar(row_key, n, prefix1, need1, 2, sh);
          }
        }
        // ---- ordered output: {key >= K*} (K* >= 1 excludes the pad records).
        // Pass 1 counts each (j, warp) group's selected records; one block scan
        // over the nj * kTkWarps groups (group order = record order) gives their
        // output offsets; pass 2 places each record at its group's offset plus its
        // rank among the group's selected lanes.  The ids (and scores) are
        // gathered in shared memory, then leave in 16-byte stores.
        if (kstar == 0ull) kstar = 1ull;
        const uint32_t lt = (1u << lane) - 1u;
        for (uint32_t j = 0; j < nj; ++j) {
          const unsigned b = __ballot_sync(0xffffffffu, rec_at(j) >= kstar);
          if (lane == 0) sh.grp[j * kTkWarps + warp] = uint32_t(__popc(b));
        }
        __syncthreads();
        uint32_t total_sel = 0;
        const uint32_t goff =
            block_excl_scan(uint32_t(tid) < nj * kTkWarps ? sh.grp[tid] : 0u, total_sel, sh);
        if (uint32_t(tid) < nj * kTkWarps) sh.grp[tid] = goff;  // each thread rewrites only its own entry
        __syncthreads();
        const bool gather = k <= (osrow != nullptr ? kTkRankCap : 2 * kTkRankCap) && (k & 3) == 0 &&
                            (reinterpret_cast<uintptr_t>(orow) & 15u) == 0 &&
                            (reinterpret_cast<uintptr_t>(osrow) & 15u) == 0;
        int32_t* gid = reinterpret_cast<int32_t*>(sh.rank);
        float* gsc = reinterpret_cast<float*>(sh.rank) + k;
        if (gather) {
          // branch-free: unselected lanes store to the sink words
          for (uint32_t j = 0; j < nj; ++j) {
            const uint64_t rec = rec_at(j);
            const bool sel = rec >= kstar;
            const unsigned b = __ballot_sync(0xffffffffu, sel);
            const uint32_t pos = sh.grp[j * kTkWarps + warp] + uint32_t(__popc(b & lt));
            const bool put = sel && pos < uint32_t(k);
            *(put ? gid + pos : reinterpret_cast<int32_t*>(&sh.sink4[0])) = record_id(rec);
            if (osrow != nullptr) *(put ? gsc + pos : reinterpret_cast<float*>(&sh.sink4[1])) = record_score(rec);
          }
        } else {
          for (uint32_t j = 0; j < nj; ++j) {
            const uint64_t rec = rec_at(j);
            const bool sel = rec >= kstar;
            const unsigned b = __ballot_sync(0xffffffffu, sel);
            const uint32_t pos = sh.grp[j * kTkWarps + warp] + uint32_t(__popc(b & lt));
            if (sel && pos < uint32_t(k)) {
              orow[pos] = record_id(rec);
              if (osrow != nullptr) osrow[pos] = record_score(rec);
            }
          }
        }
        if (gather) {
          const uint32_t got = total_sel < uint32_t(k) ? total_sel : uint32_t(k);
          for (uint32_t p0 = 0; p0 < uint32_t(k); p0 += kTkThreads) {
            const uint32_t p = p0 + uint32_t(tid);
            if (p >= got && p < uint32_t(k)) {
              gid[p] = -1;
              if (osrow != nullptr) gsc[p] = -CUDART_INF_F;
            }
          }
          __syncthreads();
          for (int p0 = 0; p0 < k; p0 += 4 * kTkThreads) {
            const int p = p0 + 4 * tid;
            if (p < k) {
              *reinterpret_cast<int4*>(orow + p) = *reinterpret_cast<const int4*>(gid + p);
              if (osrow != nullptr)
                *reinterpret_cast<float4*>(osrow + p) = *reinterpret_cast<const float4*>(gsc + p);
            }
          }
          total_sel = uint32_t(k);  // the padding is written
        }
        chosen = total_sel < uint32_t(k) ? total_sel : uint32_t(k);
      } else {
        // ---- more records than shared memory holds (massively tied scores): walk
        // them from L2 in chunks; a shared map gives every position of a chunk its
        // slot, so consecutive threads load consecutive records
        constexpr uint32_t kChunk = uint32_t(kTkThreads) * kTkRegs;
        uint64_t rec[kTkRegs];
        uint32_t loaded_c0 = 0xffffffffu;  // block-uniform
        auto load_records = [&](uint32_t c0) {
          if (loaded_c0 == c0) return;
          loaded_c0 = c0;
          __syncthreads();  // readers of the previous chunk's map are done
          if (uint32_t(tid) < touching) {
            const uint32_t b = sh.pre[tid], e = sh.pre[tid + 1];
            const uint32_t lo = b > c0 ? b : c0, hi = e < c0 + kChunk ? e : c0 + kChunk;
            for (uint32_t f = lo; f < hi; ++f) sh.map[f - c0] = uint8_t(tid);
          }
          __syncthreads();
  #pragma unroll
          for (int j = 0; j < kTkRegs; ++j) {
            const uint32_t f = c0 + j * kTkThreads + tid;
            if (f < total_staged) {
              const uint32_t slot = sh.map[f - c0];
              rec[j] = __ldcg(srec + sh.e0s[slot] + (f - sh.pre[slot]));
            } else {
              rec[j] = 0ull;
            }
          }
        };
        if (!sub_all) {
          __syncthreads();  // sh.nrank
          for (uint32_t c0 = 0; c0 < total_staged; c0 += kChunk) {
            load_records(c0);
  #pragma unroll
            for (int j = 0; j < kTkRegs; ++j) {
              const uint64_t key = record_key(rec[j]);
              if (rec[j] != 0ull && shares_two_digits(key)) {
                const uint32_t slot = atomicAdd(&sh.nrank, 1u);
                if (slot < uint32_t(kTkRankCap)) sh.rank[slot] = key;
              }
            }
          }
          __syncthreads();
          const uint32_t nr = sh.nrank;
          if (nr <= uint32_t(kTkRankCap)) {
            kstar = resolve_kstar([&](int64_t j) { return sh.rank[j]; }, nr, prefix1, need1, 2, sh);
          } else {
            auto row_key = [&](int64_t j) -> uint64_t {
              const uint32_t u = entry_key(srow, irow, j);
              const int32_t id = kIds ? irow[j] : int32_t(id_base + j);
              return u ? composite(u, 0x7fffffffu - uint32_t(id)) : 0ull;
            };
            kstar = resolve_kstar(row_key, n, prefix1, need1, 2, sh);
          }
        }
        // ---- keep the selected records in entry order and write them out
        uint32_t written = 0;  // block-uniform
        for (uint32_t c0 = 0; c0 < total_staged && written < uint32_t(k); c0 += kChunk) {
          load_records(c0);  // the rank pass already holds a single chunk
          unsigned bal[kTkRegs];
  #pragma unroll
          for (int j = 0; j < kTkRegs; ++j) {
            bal[j] = __ballot_sync(0xffffffffu, selected(rec[j], kstar));
            if (lane == 0) sh.tot16[j][warp] = __popc(bal[j]);
          }
          __syncthreads();
          uint32_t base = written;
  #pragma unroll
          for (int j = 0; j < kTkRegs; ++j) {
            uint32_t before = 0, all = 0;
  #pragma unroll
            for (int w = 0; w < kTkWarps; ++w) {
              const uint32_t t = sh.tot16[j][w];
              before += w < warp ? t : 0u;
              all += t;
            }
            if ((bal[j] >> lane) & 1u) {
              const uint32_t pos = base + before + __popc(bal[j] & ((1u << lane) - 1u));
              if (pos < uint32_t(k)) {
                orow[pos] = record_id(rec[j]);
                if (osrow != nullptr) osrow[pos] = record_score(rec[j]);
              }
            }
            base += all;
          }
          written = base;
          __syncthreads();  // sh.tot16 is reused by the next chunk
        }
        chosen = written < uint32_t(k) ? written : uint32_t(k);
      }
      for (int p0 = int(chosen) & ~(kTkThreads - 1); p0 < k; p0 += kTkThreads) {
        const int p = p0 + tid;
        if (p >= int(chosen) && p < k) {
          orow[p] = -1;
          if (osrow != nullptr) osrow[p] = -CUDART_INF_F;
        }
      }
      // every CTA of the row is done with its state: clear it for the next call
  #pragma unroll
      for (int j = 0; j < kTkBins / kTkThreads; ++j) {
        h0row[j * kTkThreads + tid] = 0u;
        h1row[j * kTkThreads + tid] = 0u;
      }
      if (tid == 0) gdone[r] = 0u;
      __syncthreads();  // the record area and the ring are reused by the next row
    }
  }
}

int topk_ctas(int64_t rows, int64_t row_stride) {
  const int64_t words = rows * ((row_stride + 31) / 32);
  int64_t ctas = sm_count();
  if (ctas > kTkMaxCtas) ctas = kTkMaxCtas;
  if (words < ctas * 4) ctas = (words + 3) / 4;  // at least 4 words (128 entries) per CTA
  return int(ctas < 1 ? 1 : ctas);
}

}  // namespace

size_t topk_workspace_bytes(int64_t rows, int64_t row_stride) {
  return TopkWs(rows, row_stride).total;
}

size_t topk_zeroed_prefix_bytes(int64_t rows, int64_t row_stride) {
  return TopkWs(rows, row_stride).cnt;
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
  DSR_REQUIRE(id_base >= 0 && id_base + row_stride < (int64_t(1) << 31) - 1,
              "topk_select: ids must be below 2^31 - 1");
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
  const CtaSplit split = make_split(rows * ((row_stride + 31) / 32), ctas, (row_stride + 31) / 32);
  if (!hist_ready) {
    int rc = set_max_smem(topk_hist_kernel<true>, kTkHistSmem, "topk histogram");
    if (rc == DSR_OK) rc = set_max_smem(topk_hist_kernel<false>, kTkHistSmem, "topk histogram");
    if (rc != DSR_OK) return rc;
    cfg.numAttrs = pdl ? 1 : 0;
    cfg.dynamicSmemBytes = kTkHistSmem;
    cfg.blockDim = dim3(kHsThreads, 1, 1);
    const cudaError_t e =
        ids != nullptr
            ? cudaLaunchKernelEx(&cfg, topk_hist_kernel<true>, scores, ids, lengths, rows, row_stride, ws, split)
            : cudaLaunchKernelEx(&cfg, topk_hist_kernel<false>, scores, ids, lengths, rows, row_stride, ws,
                                 split);
    cfg.dynamicSmemBytes = 0;
    cfg.blockDim = dim3(kTkThreads, 1, 1);
    if (e != cudaSuccess) return fail(DSR_ECUDA, "topk histogram launch: %s", cudaGetErrorString(e));
    cfg.numAttrs = 1;
  } else {
    cfg.numAttrs = pdl ? 1 : 0;
  }
  {
    int rc = set_max_smem(topk_select_kernel<true, 4>, kTkDynSmem, "topk select");
    if (rc == DSR_OK) rc = set_max_smem(topk_select_kernel<false, 4>, kTkDynSmem, "topk select");
    if (rc == DSR_OK) rc = set_max_smem(topk_select_kernel<false, 16>, kTkDynSmem, "topk select");
    if (rc != DSR_OK) return rc;
  }
  cfg.dynamicSmemBytes = kTkDynSmem;
  const bool wide = rows * ((row_stride + 31) / 32) * 32 / ctas >= kTkWideRange;
  const cudaError_t e =
      ids != nullptr
          ? cudaLaunchKernelEx(&cfg, topk_select_kernel<true, 4>, scores, ids, lengths, out_ids,
                               out_scores, err, rows, row_stride, int(k), id_base, ws, split)
      : wide ? cudaLaunchKernelEx(&cfg, topk_select_kernel<false, 16>, scores, ids, lengths, out_ids,
                                  out_scores, err, rows, row_stride, int(k), id_base, ws, split)
             : cudaLaunchKernelEx(&cfg, topk_select_kernel<false, 4>, scores, ids, lengths, out_ids,
                                  out_scores, err, rows, row_stride, int(k), id_base, ws, split);
  if (e != cudaSuccess) return fail(DSR_ECUDA, "topk launch: %s", cudaGetErrorString(e));
  return DSR_OK;
}

// ---------------------------------------------------------------------------
// Merge of per-shard ranked lists: lists i32[world][2][rows][k] (per shard: the
// scores' bit patterns, then their global ids, -1 padded; a shard's ids increase
// and shard w's ids lie below shard w+1's) -> rows of world*k (score, id) pairs
// in id order, then the exact top-k of each row.
// ---------------------------------------------------------------------------
namespace {
__global__ void __launch_bounds__(256) merge_gather_kernel(const int32_t* __restrict__ lists,
                                                           int world, int rows, int k,
                                                           float* __restrict__ scores,
                                                           int32_t* __restrict__ ids,
                                                           int32_t* __restrict__ lengths) {
  const int64_t total = int64_t(world) * rows * k;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int j = int(i % k);
    const int64_t wr = i / k;
    const int r = int(wr % rows), w = int(wr / rows);
    const int32_t* src = lists + (int64_t(w) * 2 * rows + r) * k + j;
    const int64_t dst = int64_t(r) * world * k + int64_t(w) * k + j;
    scores[dst] = __int_as_float(src[0]);
    ids[dst] = src[int64_t(rows) * k];
  }
  if (blockIdx.x == 0)
    for (int r = threadIdx.x; r < rows; r += blockDim.x) lengths[r] = world * k;
  pdl_launch_dependents();
}

// Rows of at most kMgThreads * kMgMaxPer entries are merged by one CTA each:
// the rank keys stay in registers, a radix select narrows the key range on a
// shared histogram (warp-aggregated counts), and the selected entries leave in
// entry order, which is id order, through one ordered compaction.  No global
// atomics, no staging, one launch.
constexpr int kMgThreads = 1024;
constexpr int kMgWarps = kMgThreads / 32;
constexpr int kMgMaxPer = 16;
constexpr int kMgRankCap = 128;  // bin size ranked directly

// Whole block of kMgThreads: over h[0, nb) (nb in {1024, 2048}) the bin b with
// count(bins > b) < need <= count(bins >= b); returns b, sets `above`.
__device__ uint32_t merge_find_bin(const uint32_t* h, int nb, uint32_t need, uint32_t& above,
                                   uint32_t* wsum, uint32_t* result) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bpt = nb / kMgThreads;  // 1 or 2; thread 0 holds the top bins
  const int top = nb - tid * bpt;
  const uint32_t v0 = h[top - 1], v1 = bpt == 2 ? h[top - 2] : 0u;
  const uint32_t mine = v0 + v1;
  uint32_t incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t x = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += x;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    uint32_t s = wsum[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t x = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += x;
    }
    wsum[lane] = s - wsum[lane];  // exclusive warp offsets
  }
  __syncthreads();
  incl += wsum[warp];
  const uint32_t excl = incl - mine;
  if (excl < need && incl >= need) {
    const bool first = excl + v0 >= need;
    result[0] = uint32_t(first ? top - 1 : top - 2);
    result[1] = first ? excl : excl + v0;
  }
  __syncthreads();
  above = result[1];
  return result[0];
}

template <int E>
__global__ void __launch_bounds__(kMgThreads) merge_select_kernel(const int32_t* __restrict__ lists,
                                                                  int world, int rows, int k,
                                                                  int32_t* __restrict__ out_ids) {
  __shared__ uint32_t hist[kTkBins];
  __shared__ uint32_t wsum[kMgWarps], wmin[kMgWarps], wmax[kMgWarps];
  __shared__ uint32_t cand[kMgRankCap];
  __shared__ uint32_t result[2], ncand, ustar_s, needt_s;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r = blockIdx.x;
  const int n = world * k;
  pdl_launch_dependents();
  pdl_wait();  // the lists come from the preceding exchange

  // thread tid holds the E consecutive entries e0 + j of the row's world * k
  // (entry e is entry e % k of shard e / k, so entry order is id order); every
  // load is issued before any is used
  const int e0 = tid * E;
  uint32_t raw[E];
  int32_t idv[E];
  const bool vec = E >= 4 && k % E == 0 && (reinterpret_cast<uintptr_t>(lists) & 15u) == 0;
  if (vec) {  // the run lies inside one shard and starts on a 16-byte boundary
    const int ec = e0 < n ? e0 : 0;
    const int w = ec / k;
    const int32_t* src = lists + (int64_t(w) * 2 * rows + r) * k + (ec - w * k);
#pragma unroll
    for (int v = 0; v < E / 4; ++v) {
      const int4 a = __ldg(reinterpret_cast<const int4*>(src) + v);
      const int4 b = __ldg(reinterpret_cast<const int4*>(src + int64_t(rows) * k) + v);
      raw[4 * v] = uint32_t(a.x), raw[4 * v + 1] = uint32_t(a.y);
      raw[4 * v + 2] = uint32_t(a.z), raw[4 * v + 3] = uint32_t(a.w);
      idv[4 * v] = b.x, idv[4 * v + 1] = b.y, idv[4 * v + 2] = b.z, idv[4 * v + 3] = b.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < E; ++j) {
      const int e = e0 + j < n ? e0 + j : n - 1;
      const int w = e / k;
      const int32_t* src = lists + (int64_t(w) * 2 * rows + r) * k + (e - w * k);
      raw[j] = uint32_t(__ldg(src));
      idv[j] = __ldg(src + int64_t(rows) * k);
    }
  }
  // score keys (0: absent; present keys are >= 0x007fffff), their count and range
  uint32_t u[E];
  uint32_t mine = 0, umin = 0xffffffffu, umax = 0u;
#pragma unroll
  for (int j = 0; j < E; ++j) {
    const bool present = e0 + j < n && idv[j] >= 0;
    u[j] = present ? rank_u(raw[j]) : 0u;
    mine += present ? 1u : 0u;
    umin = present && u[j] < umin ? u[j] : umin;
    umax = u[j] > umax ? u[j] : umax;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    mine += __shfl_xor_sync(0xffffffffu, mine, o);
    umin = min(umin, __shfl_xor_sync(0xffffffffu, umin, o));
    umax = max(umax, __shfl_xor_sync(0xffffffffu, umax, o));
  }
  if (lane == 0) {
    wsum[warp] = mine;
    wmin[warp] = umin;
    wmax[warp] = umax;
  }
  __syncthreads();
  uint32_t present = wsum[lane];
  umin = wmin[lane];
  umax = wmax[lane];
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    present += __shfl_xor_sync(0xffffffffu, present, o);
    umin = min(umin, __shfl_xor_sync(0xffffffffu, umin, o));
    umax = max(umax, __shfl_xor_sync(0xffffffffu, umax, o));
  }
  __syncthreads();

  // threshold score key u* and how many entries equal to it are taken (need_t):
  // selected = {u > u*} + the first need_t entries with u == u* in entry order,
  // which is the reference's lower-id-first rule for equal scores.  Each radix
  // level bins the remaining range [lo, lo + span] into 2048 equal bins.
  uint32_t ustar = 0u, need_t = 0u;  // take_all: every present entry (u > 0)
  if (present > uint32_t(k)) {
    uint32_t need = uint32_t(k);
    uint32_t lo = umin, span = umax - umin;
    for (int level = 0; level < 4; ++level) {
      const int bits = span ? 32 - __clz(span) : 0;
      const int sh = bits > 11 ? bits - 11 : 0;
      for (int i = tid; i < kTkBins; i += kMgThreads) hist[i] = 0u;
      __syncthreads();
#pragma unroll
      for (int j = 0; j < E; ++j)
        if (u[j] >= lo && u[j] - lo <= span) atomicAdd(&hist[(u[j] - lo) >> sh], 1u);
      __syncthreads();
      uint32_t above;
      const uint32_t b = merge_find_bin(hist, kTkBins, need, above, wsum, result);
      need -= above;
      const uint32_t thr = lo + (b << sh);
      const uint32_t inbin = hist[b];
      if (tid == 0) ncand = 0u;
      __syncthreads();  // hist is cleared by the next level
      if (inbin == need) {  // the whole sub-range is taken
        ustar = thr - 1u;
        break;
      }
      if (sh == 0) {  // one score value: its first `need` entries are taken
        ustar = thr;
        need_t = need;
        break;
      }
      const uint32_t width = (1u << sh) - 1u;
      span = span - (b << sh) < width ? span - (b << sh) : width;
      lo = thr;
      if (inbin <= uint32_t(kMgRankCap)) {
        // few keys in the bin: u* is the one with fewer than `need` keys above it
        // and at least `need` at or above it
#pragma unroll
        for (int j = 0; j < E; ++j)
          if (u[j] >= lo && u[j] - lo <= span) cand[atomicAdd(&ncand, 1u)] = u[j];
        __syncthreads();
        if (uint32_t(tid) < inbin) {
          const uint32_t me = cand[tid];
          uint32_t gt = 0, ge = 0;
          for (uint32_t j = 0; j < inbin; ++j) {
            gt += cand[j] > me ? 1u : 0u;
            ge += cand[j] >= me ? 1u : 0u;
          }
          if (gt < need && need <= ge) {
            ustar_s = me;
            needt_s = need - gt;
          }
        }
        __syncthreads();
        ustar = ustar_s;
        need_t = needt_s;
        break;
      }
    }
  }

  // ordered compaction: one block scan of packed (taken-above << 16 | ties) counts
  uint32_t sure = 0, tie = 0;
#pragma unroll
  for (int j = 0; j < E; ++j) {
    sure |= uint32_t(u[j] != 0u && u[j] > ustar) << j;
    tie |= uint32_t(u[j] != 0u && u[j] == ustar) << j;
  }
  const uint32_t c = (uint32_t(__popc(sure)) << 16) | uint32_t(__popc(tie));
  uint32_t incl = c;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t x = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += x;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  uint32_t wv = wsum[lane], wincl = wv;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t x = __shfl_up_sync(0xffffffffu, wincl, o);
    if (lane >= o) wincl += x;
  }
  const uint32_t tot = __shfl_sync(0xffffffffu, wincl, 31);
  const uint32_t excl = __shfl_sync(0xffffffffu, wincl - wv, warp) + incl - c;
  uint32_t ties_before = excl & 0xffffu;
  uint32_t pos = (excl >> 16) + (ties_before < need_t ? ties_before : need_t);
  const uint32_t total = (tot >> 16) + ((tot & 0xffffu) < need_t ? (tot & 0xffffu) : need_t);
  int32_t* orow = out_ids + int64_t(r) * k;
#pragma unroll
  for (int j = 0; j < E; ++j) {
    bool take = (sure >> j) & 1u;
    if ((tie >> j) & 1u) take = ties_before++ < need_t;
    if (take) {
      if (pos < uint32_t(k)) orow[pos] = idv[j];
      ++pos;
    }
  }
  for (int p = int(total < uint32_t(k) ? total : uint32_t(k)) + tid; p < k; p += kMgThreads) orow[p] = -1;
}

template <int E>
int launch_merge_select(const int32_t* lists, int world, int rows, int k, int32_t* out_ids,
                        cudaStream_t stream) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(rows), 1, 1);
  cfg.blockDim = dim3(kMgThreads, 1, 1);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, merge_select_kernel<E>, lists, world, rows, k, out_ids);
  if (e != cudaSuccess) return fail(DSR_ECUDA, "topk_merge launch: %s", cudaGetErrorString(e));
  return DSR_OK;
}

// Rows of 8193..16384 entries: a cluster of kMcCtas CTAs per row, CTA c holding
// the c-th eighth of the row's entries (in entry order) in registers.  Each radix
// level's histogram is built per CTA; CTA c sums the c-th slice of the bins over
// the cluster through distributed shared memory and every CTA gathers the slices
// (two cluster barriers per level, the per-CTA histograms double-buffered so that
// a level's counts stay readable until every CTA has passed the next level's
// first barrier); every CTA then takes the same threshold decisions.  The
// ordered compaction adds the counts of the lower-ranked CTAs.  Same selection
// and order as merge_select_kernel, spread over eight SMs.
constexpr int kMcCtas = 8;
constexpr int kMcThreads = 256;
constexpr int kMcWarps = kMcThreads / 32;

// merge_find_bin for a block of kMcThreads over h[0, kTkBins).
__device__ uint32_t cluster_find_bin(const uint32_t* h, uint32_t need, uint32_t& above, uint32_t* wsum,
                                     uint32_t* result) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int bpt = kTkBins / kMcThreads;
  const int top = kTkBins - tid * bpt;
  uint32_t mine = 0;
#pragma unroll
  for (int j = 0; j < bpt; ++j) mine += h[top - 1 - j];
  uint32_t incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t x = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += x;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  uint32_t before = 0;
#pragma unroll
  for (int w = 0; w < kMcWarps; ++w) before += w < warp ? wsum[w] : 0u;
  incl += before;
  const uint32_t excl = incl - mine;
  if (excl < need && incl >= need) {  // exactly one thread: its bins from the top
    uint32_t acc = excl;
    for (int j = 0; j < bpt; ++j) {
      const uint32_t v = h[top - 1 - j];
      if (acc + v >= need) {
        result[0] = uint32_t(top - 1 - j);
        result[1] = acc;
        break;
      }
      acc += v;
    }
  }
  __syncthreads();
  above = result[1];
  return result[0];
}

template <int E>
__global__ void __cluster_dims__(kMcCtas, 1, 1) __launch_bounds__(kMcThreads)
    merge_cluster_kernel(const int32_t* __restrict__ lists, int world, int rows, int k,
                         int32_t* __restrict__ out_ids) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ uint32_t hist[2][kTkBins];  // this CTA's counts, by level parity
  __shared__ uint32_t hsum[kTkBins];     // the cluster's counts
  __shared__ uint32_t wsum[kMcWarps], wmin[kMcWarps], wmax[kMcWarps];
  __shared__ uint32_t cand[kMgRankCap], allc[kMgRankCap];
  __shared__ uint32_t pub_a[3], pub_b[1], tot_s[3], base_s[2];
  __shared__ uint32_t result[2], ncand, ustar_s, needt_s;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = int(cluster.block_rank());
  const int r = int(blockIdx.x) / kMcCtas;
  const int n = world * k;
  pdl_launch_dependents();
  pdl_wait();  // the lists come from the preceding exchange

  // thread tid of CTA c holds the E consecutive entries e0 + j (entry e is entry
  // e % k of shard e / k, so entry order is id order)
  const int e0 = (c * kMcThreads + tid) * E;
  uint32_t raw[E];
  int32_t idv[E];
  const bool vec = E >= 4 && k % E == 0 && (reinterpret_cast<uintptr_t>(lists) & 15u) == 0;
  if (vec) {
    const int ec = e0 < n ? e0 : 0;
    const int w = ec / k;
    const int32_t* src = lists + (int64_t(w) * 2 * rows + r) * k + (ec - w * k);
#pragma unroll
    for (int v = 0; v < E / 4; ++v) {
      const int4 a = __ldg(reinterpret_cast<const int4*>(src) + v);
      const int4 b = __ldg(reinterpret_cast<const int4*>(src + int64_t(rows) * k) + v);
      raw[4 * v] = uint32_t(a.x), raw[4 * v + 1] = uint32_t(a.y);
      raw[4 * v + 2] = uint32_t(a.z), raw[4 * v + 3] = uint32_t(a.w);
      idv[4 * v] = b.x, idv[4 * v + 1] = b.y, idv[4 * v + 2] = b.z, idv[4 * v + 3] = b.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < E; ++j) {
      const int e = e0 + j < n ? e0 + j : n - 1;
      const int w = e / k;
      const int32_t* src = lists + (int64_t(w) * 2 * rows + r) * k + (e - w * k);
      raw[j] = uint32_t(__ldg(src));
      idv[j] = __ldg(src + int64_t(rows) * k);
    }
  }
  uint32_t u[E];
  uint32_t mine = 0, umin = 0xffffffffu, umax = 0u;
#pragma unroll
  for (int j = 0; j < E; ++j) {
    const bool present = e0 + j < n && idv[j] >= 0;
    u[j] = present ? rank_u(raw[j]) : 0u;
    mine += present ? 1u : 0u;
    umin = present && u[j] < umin ? u[j] : umin;
    umax = u[j] > umax ? u[j] : umax;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    mine += __shfl_xor_sync(0xffffffffu, mine, o);
    umin = min(umin, __shfl_xor_sync(0xffffffffu, umin, o));
    umax = max(umax, __shfl_xor_sync(0xffffffffu, umax, o));
  }
  if (lane == 0) {
    wsum[warp] = mine;
    wmin[warp] = umin;
    wmax[warp] = umax;
  }
  __syncthreads();
  if (tid == 0) {
    uint32_t p = 0, lo = 0xffffffffu, hi = 0u;
    for (int w = 0; w < kMcWarps; ++w) {
      p += wsum[w];
      lo = min(lo, wmin[w]);
      hi = max(hi, wmax[w]);
    }
    pub_a[0] = p, pub_a[1] = lo, pub_a[2] = hi;
  }
  cluster.sync();
  if (warp == 0) {  // the cluster's count and range, the same in every CTA
    uint32_t p = 0, lo = 0xffffffffu, hi = 0u;
    if (lane < kMcCtas) {
      const uint32_t* rp = cluster.map_shared_rank(pub_a, lane);
      p = rp[0], lo = rp[1], hi = rp[2];
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      p += __shfl_xor_sync(0xffffffffu, p, o);
      lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
      hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    }
    if (lane == 0) tot_s[0] = p, tot_s[1] = lo, tot_s[2] = hi;
  }
  __syncthreads();
  const uint32_t present = tot_s[0];
  umin = tot_s[1];
  umax = tot_s[2];

  // u* and need_t as in merge_select_kernel
  uint32_t ustar = 0u, need_t = 0u;
  if (present > uint32_t(k)) {
    uint32_t need = uint32_t(k);
    uint32_t lo = umin, span = umax - umin;
    for (int level = 0; level < 4; ++level) {
      const int bits = span ? 32 - __clz(span) : 0;
      const int sh = bits > 11 ? bits - 11 : 0;
      uint32_t* h = hist[level & 1];
      for (int i = tid; i < kTkBins; i += kMcThreads) h[i] = 0u;
      if (tid == 0) ncand = 0u;
      __syncthreads();
#pragma unroll
      for (int j = 0; j < E; ++j)
        if (u[j] >= lo && u[j] - lo <= span) atomicAdd(&h[(u[j] - lo) >> sh], 1u);
      cluster.sync();  // every CTA's counts of this level are complete
      {
        // CTA c sums its slice of the bins over the cluster, then every CTA
        // gathers the slices: two rounds of kMcCtas independent remote loads
        constexpr int kSlice = kTkBins / kMcCtas;
        static_assert(kSlice % kMcThreads == 0 || kMcThreads % kSlice == 0, "bin slices");
        for (int i = c * kSlice + tid; i < (c + 1) * kSlice; i += kMcThreads) {
          uint32_t v[kMcCtas];
#pragma unroll
          for (int q = 0; q < kMcCtas; ++q) v[q] = cluster.map_shared_rank(h, q)[i];
          uint32_t t = 0;
#pragma unroll
          for (int q = 0; q < kMcCtas; ++q) t += v[q];
          hsum[i] = t;
        }
        cluster.sync();  // every slice is summed
        for (int i = tid; i < kSlice; i += kMcThreads) {
          uint32_t v[kMcCtas];
#pragma unroll
          for (int q = 0; q < kMcCtas; ++q) v[q] = q == c ? 0u : cluster.map_shared_rank(hsum, q)[q * kSlice + i];
#pragma unroll
          for (int q = 0; q < kMcCtas; ++q)
            if (q != c) hsum[q * kSlice + i] = v[q];
        }
        __syncthreads();
      }
      uint32_t above;
      const uint32_t b = cluster_find_bin(hsum, need, above, wsum, result);
      need -= above;
      const uint32_t thr = lo + (b << sh);
      const uint32_t inbin = hsum[b];
      if (inbin == need) {  // the whole sub-range is taken
        ustar = thr - 1u;
        break;
      }
      if (sh == 0) {  // one score value: its first `need` entries are taken
        ustar = thr;
        need_t = need;
        break;
      }
      const uint32_t width = (1u << sh) - 1u;
      span = span - (b << sh) < width ? span - (b << sh) : width;
      lo = thr;
      if (inbin <= uint32_t(kMgRankCap)) {
        // few keys in the bin: gather them from every CTA, rank them pairwise
#pragma unroll
        for (int j = 0; j < E; ++j)
          if (u[j] >= lo && u[j] - lo <= span) cand[atomicAdd(&ncand, 1u)] = u[j];
        cluster.sync();
        {
          // warp q copies CTA q's candidates after the lower CTAs' ones
          static_assert(kMcWarps == kMcCtas, "one warp per CTA of the cluster");
          const uint32_t nl = lane < kMcCtas ? *cluster.map_shared_rank(&ncand, lane) : 0u;
          uint32_t at = 0;
#pragma unroll
          for (int q = 0; q < kMcCtas; ++q) at += q < warp ? __shfl_sync(0xffffffffu, nl, q) : 0u;
          const uint32_t nq = __shfl_sync(0xffffffffu, nl, warp);
          const uint32_t* cq = cluster.map_shared_rank(cand, warp);
          for (uint32_t i = lane; i < nq; i += 32) allc[at + i] = cq[i];
        }
        __syncthreads();
        if (uint32_t(tid) < inbin) {
          const uint32_t me = allc[tid];
          uint32_t gt = 0, ge = 0;
          for (uint32_t j = 0; j < inbin; ++j) {
            gt += allc[j] > me ? 1u : 0u;
            ge += allc[j] >= me ? 1u : 0u;
          }
          if (gt < need && need <= ge) {
            ustar_s = me;
            needt_s = need - gt;
          }
        }
        __syncthreads();
        ustar = ustar_s;
        need_t = needt_s;
        break;
      }
    }
  }

  // ordered compaction: block scan of packed (taken-above << 16 | ties) counts,
  // then the lower-ranked CTAs' totals
  uint32_t sure = 0, tie = 0;
#pragma unroll
  for (int j = 0; j < E; ++j) {
    sure |= uint32_t(u[j] != 0u && u[j] > ustar) << j;
    tie |= uint32_t(u[j] != 0u && u[j] == ustar) << j;
  }
  const uint32_t cnt = (uint32_t(__popc(sure)) << 16) | uint32_t(__popc(tie));
  uint32_t incl = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t x = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += x;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  uint32_t wbefore = 0, ctot = 0;
#pragma unroll
  for (int w = 0; w < kMcWarps; ++w) {
    wbefore += w < warp ? wsum[w] : 0u;
    ctot += wsum[w];
  }
  if (tid == 0) pub_b[0] = ctot;
  cluster.sync();
  if (tid == 0) {
    uint32_t below = 0, all = 0;
    for (int q = 0; q < kMcCtas; ++q) {
      const uint32_t v = *cluster.map_shared_rank(pub_b, q);
      below += q < c ? v : 0u;
      all += v;
    }
    base_s[0] = below;
    base_s[1] = all;
  }
  __syncthreads();
  const uint32_t excl = base_s[0] + wbefore + incl - cnt;
  const uint32_t tot = base_s[1];
  uint32_t ties_before = excl & 0xffffu;
  uint32_t pos = (excl >> 16) + (ties_before < need_t ? ties_before : need_t);
  const uint32_t total = (tot >> 16) + ((tot & 0xffffu) < need_t ? (tot & 0xffffu) : need_t);
  int32_t* orow = out_ids + int64_t(r) * k;
#pragma unroll
  for (int j = 0; j < E; ++j) {
    bool take = (sure >> j) & 1u;
    if ((tie >> j) & 1u) take = ties_before++ < need_t;
    if (take) {
      if (pos < uint32_t(k)) orow[pos] = idv[j];
      ++pos;
    }
  }
  for (int p = int(total < uint32_t(k) ? total : uint32_t(k)) + c * kMcThreads + tid; p < k;
       p += kMcCtas * kMcThreads)
    orow[p] = -1;
  cluster.sync();  // no CTA leaves while another may still read its shared memory
}

template <int E>
int launch_merge_cluster(const int32_t* lists, int world, int rows, int k, int32_t* out_ids,
                         cudaStream_t stream) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(rows) * kMcCtas, 1, 1);
  cfg.blockDim = dim3(kMcThreads, 1, 1);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, merge_cluster_kernel<E>, lists, world, rows, k, out_ids);
  if (e != cudaSuccess) return fail(DSR_ECUDA, "topk_merge cluster launch: %s", cudaGetErrorString(e));
  return DSR_OK;
}
}  // namespace

size_t topk_merge_workspace_bytes(int64_t rows, int64_t world, int64_t k) {
  const int64_t n = world * k;
  return topk_workspace_bytes(rows, n) + ((size_t(rows) * n * 8 + size_t(rows) * 4 + 255) / 256) * 256;
}

int launch_topk_merge(const int32_t* lists, int64_t world, int64_t rows, int64_t k,
                      int32_t* out_ids, void* workspace, size_t workspace_bytes, int32_t* err,
                      cudaStream_t stream) {
  DSR_REQUIRE(lists && out_ids && err && workspace, "topk_merge: null pointer");
  DSR_REQUIRE(world > 0 && world <= 64 && rows > 0 && rows <= 65535 && k > 0 && k <= 8192,
              "topk_merge: invalid shape");
  DSR_REQUIRE(workspace_bytes >= topk_merge_workspace_bytes(rows, world, k),
              "topk_merge: workspace too small");
  DSR_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255u) == 0,
              "topk_merge: workspace must be 256-byte aligned");
  const int64_t n = world * k;
  if (n > int64_t(kMgThreads) * 8 && n <= int64_t(kMcCtas) * kMcThreads * 8) {
    // 8193..16384 entries (e.g. 8 shards of 2048): a cluster of kMcCtas SMs per
    // row (7.6 against 11.3 us for 4 rows of 8 x 2048 on a B200); at 4096 and
    // 8192 entries the cluster's barriers cost what the spread saves (6.4 against
    // 5.0, 6.7 against 6.8 us), so smaller rows stay on one CTA
    return launch_merge_cluster<8>(lists, int(world), int(rows), int(k), out_ids, stream);
  }
  if (n <= int64_t(kMgThreads) * kMgMaxPer) {
    const int per = int((n + kMgThreads - 1) / kMgThreads);
    if (per <= 1) return launch_merge_select<1>(lists, int(world), int(rows), int(k), out_ids, stream);
    if (per <= 2) return launch_merge_select<2>(lists, int(world), int(rows), int(k), out_ids, stream);
    if (per <= 4) return launch_merge_select<4>(lists, int(world), int(rows), int(k), out_ids, stream);
    if (per <= 8) return launch_merge_select<8>(lists, int(world), int(rows), int(k), out_ids, stream);
    return launch_merge_select<16>(lists, int(world), int(rows), int(k), out_ids, stream);
  }
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const size_t tk = topk_workspace_bytes(rows, n);
  float* scores = reinterpret_cast<float*>(ws + tk);
  int32_t* ids = reinterpret_cast<int32_t*>(scores + rows * n);
  int32_t* lengths = ids + rows * n;
  const int64_t total = rows * n;
  const int blocks = int((total + 255) / 256 < 4 * sm_count() ? (total + 255) / 256 : 4 * sm_count());
  merge_gather_kernel<<<blocks, 256, 0, stream>>>(lists, int(world), int(rows), int(k), scores, ids,
                                                  lengths);
  const int rc = launch_status("topk_merge gather launch");
  if (rc != DSR_OK) return rc;
  return launch_topk(scores, ids, lengths, out_ids, nullptr, err, rows, n, k, 0, ws, tk, stream,
                     true, false);
}

}  // namespace dsr

extern "C" size_t dsr_topk_merge_workspace_bytes(int64_t rows, int64_t world, int64_t k) {
  return dsr::topk_merge_workspace_bytes(rows, world, k);
}

extern "C" int dsr_topk_merge_lists(const int32_t* lists, int64_t world, int64_t rows, int64_t k,
                                    int32_t* out_ids, void* workspace, size_t workspace_bytes,
                                    int32_t* err, void* stream) {
  dsr::clear_error();
  return dsr::launch_topk_merge(lists, world, rows, k, out_ids, workspace, workspace_bytes, err,
                                dsr::as_stream(stream));
}

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
