// Lightning-indexer decode scoring over a paged BF16 index-key pool (sm_100a).
//
// score[b,p] = sum_h w[b,h] * max(q[b,h,:] . K[row(b,p),:], 0)
// (reference equation: native/operations.cu:104-121, reference_attention.py:34-47)
//
// Layout: index_pool bf16 [rows, 128], addressed per sequence either through a
// block table (a logical block j of sequence b, positions 64j..64j+63, lives in
// physical block block_table[b, j]) or as a ring (the reference's row pools:
// position p at row first + (p + offset) % slots).  A ring sequence's visible
// positions occupy at most two contiguous runs of rows -- [first + offset, ...)
// up to the end of its slots, then [first, ...) -- and its tiles follow those
// runs, so every load stays a tiled TMA box at any row.
//
// Kernel: persistent, one CTA per SM, tiles of 128 keys (two 64-row halves).
//   warp 0      TMA producer: two 64x64 boxes per pool block, 128-byte swizzle
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2..9  epilogue, two warpgroups sharing every tile (each reduces half
//               of the heads): Q preparation, TMEM -> registers, ReLU, weighted
//               head reduction, score store, 11-bit score histogram for top-k
// D[key, n] = K[key,:] . B[n,:] with B = [q_hi ; q_lo] (N = 2*heads rows), where
// q_hi = bf16(q) and q_lo = bf16(q - q_hi): the two products summed in FP32
// reproduce the FP32 query to ~2^-17 relative, so scores track the FP32
// reference far inside the 1e-3 tolerance while the contraction runs on the
// tensor cores.  Four TMEM accumulators let the epilogue of tile i overlap the
// MMAs of the next tiles; smem stages are a 4-deep TMA ring.  A BF16-exact
// query (q_lo == 0, the FP8-valued reference query) contracts the q_hi rows only.
#include "common.cuh"
#include "host_common.h"
#include "mla_tile.cuh"
#include "select.cuh"

namespace dsr {
namespace {

constexpr int kIxTile = 128;                 // keys per tile
constexpr int kIxStages = 4;
constexpr int kIxStageBytes = kIxTile * 256; // 128 keys x 128 bf16
constexpr int kIxThreads = 320;              // producer, MMA, 2 epilogue warpgroups
constexpr int kIxMaxBatch = 1024;
constexpr int kIxAcc = 4;                    // TMEM accumulators in flight
constexpr int kIxHistBins = 2048;            // 11-bit score-key histogram for top-k

template <int H>
struct IxLayout {
  static constexpr int N = 2 * H;
  static constexpr int kQSlotBytes = N * 256;  // two 64-column halves of N rows x 128 B
  static constexpr int kStagesOff = 0;
  static constexpr int kQOff = kIxStages * kIxStageBytes;
  static constexpr int kWOff = kQOff + 2 * kQSlotBytes;
  static constexpr int kXchOff = kWOff + 2 * H * 4;            // [2][128] partial scores
  static constexpr int kHistOff = kXchOff + 2 * 128 * 4;       // [2048] u32
  static constexpr int kBarOff = kHistOff + kIxHistBins * 4;
  static constexpr int kNumBars = 2 * kIxStages + 2 * kIxAcc + 4;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;  // tmem slot, abort flag, q_lo flags
  static constexpr int kPrefixOff = kMiscOff + 32;
  static constexpr int kVisOff = kPrefixOff + (kIxMaxBatch + 1) * 4;
  static constexpr int kRunOff = kVisOff + kIxMaxBatch * 4;  // ring rows: positions in the first run
  static constexpr int kBytes = kRunOff + kIxMaxBatch * 4;
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-byte alignment
  static constexpr uint32_t kTmemCols =
      (kIxAcc * N <= 32) ? 32 : (kIxAcc * N <= 64 ? 64 : (kIxAcc * N <= 128 ? 128 : (kIxAcc * N <= 256 ? 256 : 512)));
};

// Tile `tile` (128 keys) of sequence b: its first position, its first pool row
// (ring only; paged tiles take their rows from the block table) and its keys.
// n1 = the sequence's positions in the first ring run.
__device__ __forceinline__ void tile_span(const PoolAddr& pa, int b, int tile, int vis, int n1, int& pos0,
                                          int64_t& row0, int& valid) {
  if (pa.ring == nullptr) {
    pos0 = tile * kIxTile;
    row0 = -1;
  } else {
    const int t1 = (n1 + kIxTile - 1) / kIxTile;
    const int64_t first = pa.ring[3 * int64_t(b)];
    if (tile < t1) {
      pos0 = tile * kIxTile;
      row0 = first + pa.ring[3 * int64_t(b) + 2] + pos0;
    } else {
      pos0 = n1 + (tile - t1) * kIxTile;
      row0 = first + (tile - t1) * kIxTile;
    }
    vis = tile < t1 ? n1 : vis;  // a tile of the first run ends with it
  }
  valid = min(kIxTile, vis - pos0);
}

__device__ __forceinline__ int find_row(const int* prefix, int batch, int t) {
  int lo = 0, hi = batch;  // prefix[lo] <= t < prefix[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (prefix[mid] <= t) lo = mid;
    else hi = mid;
  }
  return lo;
}

// ---------------------------------------------------------------------------
// Exact top-k after the scores (select.cuh): this CTA's rows are those whose
// tiles intersect [t_lo, t_hi); its positions of row b are one contiguous range.
// Every CTA of the grid calls this (it holds the grid barrier).  `work` is the
// shared memory the indexer no longer needs (work_bytes >= list_cap * 8),
// `hist` 2048 words, `scratch` >= 128 words (scans, compaction groups).
// ---------------------------------------------------------------------------
constexpr int kSelThreads = 320;  // the indexer CTA: every warp joins the selection
constexpr int kSelPer = 4;        // entries per thread per compaction chunk
constexpr int kSelScoreLd = 15;   // float4 score groups staged per thread and chunk (at most)
static_assert(4 * kSelScoreLd <= 64, "a thread's candidate mask (4 bits per group) must fit 64 bits");
static_assert(((kSelBinCap + kSelMaxK + 2 + kSelThreads - 1) / kSelThreads | 1) <= 64,
              "a finisher run (list capacity / threads) must fit a 64-bit mask");
constexpr uint32_t kSelPairwise = 256;  // sub-bin keys ranked pairwise (more: one more radix level)

__device__ __forceinline__ void select_range(const PoolAddr& pa, const int* prefix, const int* vis_s,
                                             const int* run_s, int b, int t_lo, int t_hi, int& p_lo, int& p_hi,
                                             bool& first) {
  const int ta = max(t_lo, prefix[b]), tb = min(t_hi, prefix[b + 1]);
  first = ta == prefix[b];
  if (ta >= tb) {
    p_lo = p_hi = 0;
    return;
  }
  int pos0, valid;
  int64_t row0;
  tile_span(pa, b, ta - prefix[b], vis_s[b], run_s[b], pos0, row0, valid);
  p_lo = pos0;
  tile_span(pa, b, tb - 1 - prefix[b], vis_s[b], run_s[b], pos0, row0, valid);
  p_hi = pos0 + valid;
}

// 2048 histogram words of global memory into shared memory by 16-byte async
// copies (complete after cp_async_wait_all + __syncthreads)
__device__ __forceinline__ void async_hist(uint32_t* dst, const uint32_t* src) {
#pragma unroll 1
  for (int i = threadIdx.x; i < kSelBins / 4; i += kSelThreads) cp_async16(smem_u32(dst + 4 * i), src + 4 * i);
}

// keys[0, n) (16-byte aligned ends; an odd n copies one key past the end) of
// global memory into shared memory by 16-byte async copies
__device__ __forceinline__ void async_keys(uint64_t* dst, const uint64_t* src, uint32_t n) {
#pragma unroll 1
  for (uint32_t i = threadIdx.x; 2 * i < n; i += kSelThreads) cp_async16(smem_u32(dst + 2 * i), src + 2 * i);
}

// f(key) for every key of the shared-memory list lst[0, L): every thread takes a
// run of consecutive keys (an odd count: the 8-byte loads of a half warp fall on
// distinct banks), four loads in flight.
template <typename F>
__device__ __forceinline__ void list_runs(const uint64_t* lst, uint32_t L, F f) {
  constexpr uint32_t T = kSelThreads;
  const uint32_t per = ((L + T - 1) / T) | 1u;
  const uint32_t l0 = min(L, threadIdx.x * per), l1 = min(L, l0 + per);
#pragma unroll 1
  for (uint32_t i = l0; i < l1; i += 4) {
    uint64_t kq[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) kq[u] = i + u < l1 ? lst[i + u] : 0ull;
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (i + u < l1) f(kq[u]);
  }
}

// The row's last CTA for a row without overflow (select.cuh, step 3): L keys in
// the row's list, its nblk blocks in arrival order (block s starts at the list
// offset of record s; the offsets ascend), the row held by nctas CTAs.
//   1. records, the list and the row's digit-1 histogram, all in flight (16-byte
//      async copies);
//   2. K*: the sub-bin (b0, b1) holding it from that histogram; its
//      lower edge when the whole sub-bin is selected, otherwise the need1-th
//      largest of its keys (ranked pairwise when few, else by the next
//      digits).  K* does not depend on the order of the list;
//   3. every thread takes a run of consecutive list entries and marks its keys
//      >= K*; one block scan gives the selected keys before each run;
//   4. from these, the selected keys before each block's start, each block's
//      count, their exclusive scan in CTA rank order (ranks follow positions,
//      and every block is in position order) and so each block's first output
//      slot;
//   5. every thread writes its selected ids (and scores): slot = its block's
//      first slot + the selected keys before it in the block.
// The tables of steps 4-5 live in `hist` (free after step 2; 3 * gridDim.x + 1 +
// kSelThreads words <= 2048) and after the list's capacity in `work` (12 bytes
// per thread <= the kSelThreads * 16 bytes the host keeps there).
__device__ void finish_row(const SelectArgs& a, int b, uint32_t L, uint32_t nblk, uint32_t nctas, uint32_t b0,
                           uint32_t above, uint8_t* work, uint32_t* hist, uint32_t* scratch) {
  constexpr int T = kSelThreads;
  const int tid = threadIdx.x;
  __builtin_assume(__isShared(work));
  __builtin_assume(__isShared(hist));
  __builtin_assume(__isShared(scratch));
  uint32_t* ncand = scratch + 42;
  uint64_t* arr = reinterpret_cast<uint64_t*>(work);
  const uint64_t* lrow = a.list + int64_t(b) * a.list_cap;
  const uint32_t k = uint32_t(a.k);
  int32_t* orow = a.out_ids + int64_t(b) * k;
  float* oscore = a.out_scores != nullptr ? a.out_scores + int64_t(b) * k : nullptr;

  // 1. (thread s holds the record of arrival s; nblk <= gridDim.x < kSelThreads)
  uint4 rec = make_uint4(0u, 0u, ~0u, 0u);
  if (uint32_t(tid) < nblk) rec = __ldcg(a.blocks + int64_t(b) * gridDim.x + tid);
  async_keys(arr, lrow, L);
  async_hist(hist, a.hist1 + int64_t(b) * kSelBins);
  cp_async_wait_all();
  __syncthreads();
  // 2.
  const uint32_t need0 = k - above;
  uint32_t above1;
  const uint32_t b1 = sel_find_bin<T>(hist, kSelBins, need0, above1, scratch) & uint32_t(kSelBins - 1);
  const uint32_t need1 = need0 - above1, in_sub = hist[b1];
  const uint64_t sub = (uint64_t(b0) << kSelShift[0]) | (uint64_t(b1) << kSelShift[1]);
  __syncthreads();
  uint64_t kstar = sub;
  if (in_sub != need1) {
    if (in_sub > kSelPairwise) {
      kstar = sel_kstar<T>([&](int64_t i) { return arr[i]; }, L, sub, need1, 2, hist, scratch);
    } else {
      uint64_t* subk = reinterpret_cast<uint64_t*>(hist);
      if (tid == 0) {
        *ncand = 0u;
        scratch[46] = uint32_t(sub);  // K* stays the edge if the ranking finds none
        scratch[47] = uint32_t(sub >> 32);
      }
      __syncthreads();
      list_runs(arr, L, [&](uint64_t key) {
        if ((key >> kSelShift[1]) == (sub >> kSelShift[1])) {
          const uint32_t at = atomicAdd(ncand, 1u);
          if (at < kSelPairwise) subk[at] = key;
        }
      });
      __syncthreads();
      const uint32_t c = min(*ncand, kSelPairwise);
#pragma unroll 1
      for (uint32_t i = tid; i < c; i += T) {
        const uint64_t key = subk[i];
        uint32_t higher = 0;
#pragma unroll 1
        for (uint32_t j = 0; j < c; ++j) higher += subk[j] > key ? 1u : 0u;
        if (higher == need1 - 1) {
          scratch[46] = uint32_t(key);
          scratch[47] = uint32_t(key >> 32);
        }
      }
      __syncthreads();
      kstar = (uint64_t(scratch[47]) << 32) | scratch[46];
      __syncthreads();
    }
  }
  // 3. (an odd run length: the 8-byte loads of a half warp fall on distinct banks)
  const uint32_t per = ((L + T - 1) / T) | 1u;
  const uint32_t l0 = min(L, tid * per), l1 = min(L, l0 + per);
  uint64_t mask = 0;  // bit j: key l0 + j selected
#pragma unroll 1
  for (uint32_t i = l0; i < l1; i += 4) {
    uint64_t kq[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) kq[u] = i + u < l1 ? arr[i + u] : 0ull;
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (i + u < l1 && kq[u] >= kstar) mask |= 1ull << (i + u - l0);
  }
  uint32_t found;
  const uint32_t p0 = sel_excl_scan<T>(uint32_t(__popcll(mask)), found, scratch);
  // 4. tables: per rank, its block's count, then its first slot (rslot); per
  // arrival s, the block's start (abase, abase[nblk] = L) and first slot less
  // the selected keys before it (sbase); per run, the block holding its first
  // entry (first), its selected keys before it (runp) and its mask (runm)
  uint32_t* rslot = hist;
  uint32_t* abase = rslot + gridDim.x;
  uint32_t* sbase = abase + gridDim.x + 1;
  uint32_t* first = sbase + gridDim.x;
  uint64_t* runm = reinterpret_cast<uint64_t*>(work + size_t(a.list_cap) * 8);  // the list's capacity is 16-byte aligned
  uint32_t* runp = reinterpret_cast<uint32_t*>(runm + T);
  runp[tid] = p0;
  runm[tid] = mask;
  first[tid] = 0u;
  if (uint32_t(tid) < nblk) abase[tid] = min(rec.x, L);
  if (tid == 0) abase[nblk] = L;
#pragma unroll 1
  for (uint32_t r = tid; r < nctas; r += T) rslot[r] = 0u;  // ranks that appended nothing
  __syncthreads();
  // thread s (arrival s): the selected keys before its block's start and end,
  // from the runs holding them; its count; the block of every run starting in it
  const auto before = [&](uint32_t x) -> uint32_t {  // selected keys before list entry x
    if (x >= L) return found;
    const uint32_t t = x / per, j = x - t * per;
    return runp[t] + uint32_t(__popcll(runm[t] & ((1ull << j) - 1ull)));
  };
  uint32_t pstart = 0;
  const bool has_rec = uint32_t(tid) < nblk && rec.z < nctas;
  if (uint32_t(tid) < nblk) {
    const uint32_t lo = min(rec.x, L), hi = min(lo + rec.y, L);
    pstart = before(lo);
    if (has_rec) rslot[rec.z] = before(hi) - pstart;
#pragma unroll 1
    for (uint32_t t = (lo + per - 1) / per; t * per < hi; ++t) first[t] = uint32_t(tid);
  }
  __syncthreads();
  uint32_t total;
  const uint32_t cnt = uint32_t(tid) < nctas ? rslot[tid] : 0u;  // each thread reads and rewrites its own rank
  const uint32_t rs = sel_excl_scan<T>(cnt, total, scratch);
  if (uint32_t(tid) < nctas) rslot[tid] = rs;
  __syncthreads();
  if (has_rec) sbase[tid] = rslot[rec.z] - pstart;  // mod 2^32
  __syncthreads();
  // 5. (slots past k only after a CTA gave up: its candidates are missing)
  if (mask != 0ull) {
    uint32_t cur = first[tid], nxt = abase[cur + 1], p = p0, slot = sbase[cur] + p0;
#pragma unroll 1
    for (uint32_t i = l0; i < l1; i += 4) {
      uint64_t kq[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) kq[u] = i + u < l1 && ((mask >> (i + u - l0)) & 1ull) ? arr[i + u] : 0ull;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t x = i + u;
        if (x >= l1) break;
        if (x == nxt && cur + 1 < nblk) {  // the next block starts here (blocks are never empty)
          ++cur;
          nxt = abase[cur + 1];
          slot = sbase[cur] + p;
        }
        if ((mask >> (x - l0)) & 1ull) {
          if (slot < k) {
            orow[slot] = sel_key_id(kq[u]);
            if (oscore != nullptr) oscore[slot] = sel_key_score(kq[u]);
          }
          ++slot;
          ++p;
        }
      }
    }
  }
}

__device__ void select_phase(const SelectArgs& a, const float* __restrict__ scores, int64_t score_stride,
                             int batch, const int* prefix, const int* vis_s, const int* run_s, const PoolAddr& pa,
                             int t_lo, int t_hi, uint8_t* work, size_t work_bytes, uint32_t* hist,
                             uint32_t* scratch, int32_t* err, bool live, const MlaFuse& mla) {
  constexpr int T = kSelThreads;
  const int tid = threadIdx.x;
  const int k = a.k;
  // every pointer into shared memory stays in the shared state space (shared
  // loads, stores and atomics rather than generic ones)
  __builtin_assume(__isShared(work));
  __builtin_assume(__isShared(hist));
  __builtin_assume(__isShared(scratch));
  uint32_t* grp = scratch + 64;
  const int rb0 = t_lo < t_hi ? find_row(prefix, batch, t_lo) : 0;
  const int rb1 = t_lo < t_hi ? find_row(prefix, batch, t_hi - 1) : -1;
  const int total = prefix[batch];

  // ---- before the barrier: rows without keys (one CTA pads them) and rows of
  // at most k keys (every key selected: output slot = position), which need no
  // histogram
  if (live && blockIdx.x == 0)
    for (int b = 0; b < batch; ++b)
      if (vis_s[b] == 0)
#pragma unroll 1
        for (int i = tid; i < k; i += T) {
          a.out_ids[int64_t(b) * k + i] = -1;
          if (a.out_scores != nullptr) a.out_scores[int64_t(b) * k + i] = -CUDART_INF_F;
        }
  for (int b = rb0; b <= rb1 && live; ++b) {
    int p_lo, p_hi;
    bool first;
    select_range(pa, prefix, vis_s, run_s, b, t_lo, t_hi, p_lo, p_hi, first);
    const int v = vis_s[b];
    if (p_lo >= p_hi || v > k) continue;
    const float* srow = scores + int64_t(b) * score_stride;
    int32_t* orow = a.out_ids + int64_t(b) * k;
    float* oscore = a.out_scores != nullptr ? a.out_scores + int64_t(b) * k : nullptr;
#pragma unroll 1
    for (int p = p_lo + tid; p < p_hi; p += T) {
      orow[p] = int32_t(a.id_base + p);
      if (oscore != nullptr) oscore[p] = key_score(sel_rank_u(__float_as_uint(__ldcg(srow + p))));
    }
    if (first)
#pragma unroll 1
      for (int p = v + tid; p < k; p += T) {
        orow[p] = -1;
        if (oscore != nullptr) oscore[p] = -CUDART_INF_F;
      }
  }

  live = grid_barrier(a.ctl, 1, err) && live;  // every row's digit-0 histogram is complete

  // CTAs holding tiles of row b.  CTA c holds tiles [floor(total*c/G), floor(total*(c+1)/G)),
  // so tile t belongs to CTA floor(((t+1)*G - 1) / total); with fewer tiles than
  // CTAs every CTA holds at most one tile, and the row has one CTA per tile
  auto row_ctas = [&](int b) -> uint32_t {
    const int tiles = prefix[b + 1] - prefix[b];
    if (total < int(gridDim.x)) return uint32_t(tiles);
    const uint64_t G = gridDim.x;
    const uint64_t c0 = ((uint64_t(prefix[b]) + 1) * G - 1) / uint64_t(total);
    const uint64_t c1 = (uint64_t(prefix[b + 1]) * G - 1) / uint64_t(total);
    return uint32_t(c1 - c0 + 1);
  };
  unsigned long long* state = a.row_state;

  // ---- per row of more than k keys: threshold bin b0, this CTA's candidates
  // (digit 0 >= b0) appended to the row's list in one block; then the CTA
  // counts itself done with the row, and the row's last CTA finishes it.
  // Shared memory: the candidate buffer (list_cap keys), then the staging of
  // the scores (16-byte async copies, read back by rolled loops)
  uint64_t* buf = reinterpret_cast<uint64_t*>(work);
  float4* stage = reinterpret_cast<float4*>(work + size_t(a.list_cap) * 8);
  const int nld = int(min(size_t(kSelScoreLd), (work_bytes - size_t(a.list_cap) * 8) / (T * 16)));  // >= 1 (host check)
  for (int b = rb0; b <= rb1; ++b) {
    int p_lo, p_hi;
    bool first;
    select_range(pa, prefix, vis_s, run_s, b, t_lo, t_hi, p_lo, p_hi, first);
    const int v = vis_s[b];
    if (p_lo >= p_hi || v <= k) continue;
    const uint32_t nctas = row_ctas(b);
    const float* srow = scores + int64_t(b) * score_stride;
    uint32_t b0 = 0, above = 0, nkept = 0;  // nkept: this CTA's candidates in buf
    bool overflow = false;
    // this CTA's rank among the row's CTAs (with fewer tiles than CTAs, one tile each)
    const uint32_t rank = total < int(gridDim.x)
                              ? uint32_t(t_lo - prefix[b])
                              : uint32_t(blockIdx.x) -
                                    uint32_t(((uint64_t(prefix[b]) + 1) * gridDim.x - 1) / uint64_t(total));
    if (live) {
      // The range's scores in staged slots of 16 bytes.  Full mode: slot q is the
      // float4 at a0 + 4q of the aligned groups covering [p_lo, p_hi) (the row's
      // stride is a multiple of 64 floats); it is issued before the threshold is
      // known, with the histogram.  Group mode (a range of more than one staging
      // chunk, with the epilogue's group maxima): windows of the range's 32-key
      // groups; slot q holds float4 q % 9 of the window's (q / 9)-th group whose
      // largest digit 0 reaches the threshold bin, groups in position order.
      const int a0 = p_lo & ~3;
      const int n4 = (((p_hi + 3) & ~3) - a0) >> 2;
      const size_t used = size_t(a.list_cap) * 8 + size_t(nld) * T * 16;
      const int win = a.gmax == nullptr || work_bytes < used
                          ? 0
                          : int(min(size_t(2048), (work_bytes - used) / 8) / T * T);
      const bool groups = win >= T && n4 > T * nld;
      uint32_t* gtab = reinterpret_cast<uint32_t*>(work + used);  // [win] group starts, [win] ends
      auto slot_base = [&](int q) -> int { return groups ? (int(gtab[q / 9]) & ~3) + 4 * (q % 9) : a0 + 4 * q; };
      auto slot_lo = [&](int q) -> int { return groups ? int(gtab[q / 9]) : p_lo; };
      auto slot_hi = [&](int q) -> int { return groups ? int(gtab[win + q / 9]) : p_hi; };
      auto stage_chunk = [&](int i0, int ns) {  // staged slot q - i0 = j * T + tid
#pragma unroll 1
        for (int j = 0; j < nld; ++j) {
          const int q = i0 + j * T + tid;
          if (q < ns) {
            const int base = slot_base(q);
            if (base < slot_hi(q)) cp_async16(smem_u32(stage + j * T + tid), srow + base);
          }
        }
      };
      if (!groups) stage_chunk(0, n4);
      async_hist(hist, a.hist + int64_t(b) * kSelBins);
      cp_async_wait_all();
      __syncthreads();
      b0 = sel_find_bin<T>(hist, kSelBins, uint32_t(k), above, scratch) & uint32_t(kSelBins - 1);
      // massive ties: more threshold-bin entries than the list has room for; the
      // row's last CTA resolves the row from its scores
      overflow = hist[b0] > uint32_t(a.list_cap - k);
      if (!overflow) {
        // digit 0 >= b0 <=> score >= the lowest score of bin b0 (the key map is
        // monotone; NaN ranks above +inf); bins 0-3 decode to NaN patterns and
        // hold nothing above -inf, so with b0 < 4 every score passes
        const float thr = b0 < 4u ? -CUDART_INF_F : key_score(b0 << 21);
        // per staged chunk: every thread tests a run of consecutive slots (an odd
        // count: conflict-free 16-byte reads), one block scan places its
        // candidates, so the block comes out in position order
        uint32_t nbuf = 0;
        const int ta = max(t_lo, prefix[b]) - prefix[b], tb = min(t_hi, prefix[b + 1]) - prefix[b];
        const int g_end = groups ? 4 * tb : 1;
#pragma unroll 1
        for (int g0 = groups ? 4 * ta : 0; g0 < g_end; g0 += groups ? win : 1) {
          int ns = n4;
          if (groups) {
            // this window's groups that reach the threshold bin: thread tid tests r
            // consecutive groups, one block scan places them in position order
            const int g1 = min(g_end, g0 + win), r = (g1 - g0 + T - 1) / T;  // r <= 2048 / T
            const uint16_t* grow = a.gmax + int64_t(b) * a.gstride;
            uint32_t pick = 0;
#pragma unroll 1
            for (int i = 0; i < r; ++i) {
              const int g = g0 + r * tid + i;
              if (g < g1 && uint32_t(__ldcg(grow + g)) >= b0) pick |= 1u << i;
            }
            uint32_t nsel;
            uint32_t slot = sel_excl_scan<T>(uint32_t(__popc(pick)), nsel, scratch);
#pragma unroll 1
            for (int i = 0; i < r; ++i)
              if ((pick >> i) & 1u) {
                const int g = g0 + r * tid + i;
                int pos0, valid;
                int64_t row0;
                tile_span(pa, b, g >> 2, vis_s[b], run_s[b], pos0, row0, valid);
                const int gs = pos0 + 32 * (g & 3);
                gtab[slot] = uint32_t(gs);
                gtab[win + slot] = uint32_t(max(gs, min(pos0 + valid, gs + 32)));
                ++slot;
              }
            __syncthreads();
            ns = 9 * int(nsel);
          }
#pragma unroll 1
          for (int i0 = 0; i0 < ns; i0 += T * nld) {
            const int cn4 = min(T * nld, ns - i0);
            if (groups || i0 > 0) {
              stage_chunk(i0, ns);
              cp_async_wait_all();
            }
            __syncthreads();
            const int m = ((cn4 + T - 1) / T) | 1;
            const int q0 = min(cn4, tid * m), q1 = min(cn4, q0 + m);
            uint64_t take = 0;
            // four slots in flight; most slots have all four scores below the
            // threshold (NaN compares false and is kept) and need nothing more
#pragma unroll 1
            for (int qa = q0; qa < q1; qa += 4) {
              float4 x4[4];
#pragma unroll
              for (int u = 0; u < 4; ++u) x4[u] = stage[min(qa + u, q1 - 1)];
              uint32_t pass = 0;
#pragma unroll
              for (int u = 0; u < 4; ++u)
                if (qa + u < q1 && !(x4[u].x < thr && x4[u].y < thr && x4[u].z < thr && x4[u].w < thr))
                  pass |= 1u << u;
#pragma unroll 1
              while (pass != 0u) {
                const int u = __ffs(pass) - 1;
                pass &= pass - 1u;
                const float4 g = u == 0 ? x4[0] : (u == 1 ? x4[1] : (u == 2 ? x4[2] : x4[3]));
                const int qi = qa + u;
                const float xs[4] = {g.x, g.y, g.z, g.w};
                const int base = slot_base(i0 + qi), lo = slot_lo(i0 + qi), hi = slot_hi(i0 + qi);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const int p = base + e;  // slots past a group's end were not copied: p >= hi
                  if (!(xs[e] >= thr || xs[e] != xs[e]) || p < lo || p >= hi) continue;
                  const uint32_t uk = sel_rank_u(__float_as_uint(xs[e]));
                  if ((uk >> 21) < b0) continue;
                  take |= 1ull << ((qi - q0) * 4 + e);
                }
              }
            }
            uint32_t tot;
            uint32_t o = nbuf + sel_excl_scan<T>(uint32_t(__popcll(take)), tot, scratch);
#pragma unroll 1
            while (take != 0ull) {
              const int bit = __ffsll(take) - 1;
              take &= take - 1ull;
              const int qi = q0 + (bit >> 2), e = bit & 3;
              const float x = reinterpret_cast<const float*>(stage + qi)[e];
              if (o < uint32_t(a.list_cap))
                buf[o] = sel_key(sel_rank_u(__float_as_uint(x)), a.id_base + slot_base(i0 + qi) + e);
              ++o;
            }
            nbuf += tot;
            __syncthreads();  // the chunk is read before the next one is staged
          }
        }
        // the block: one atomic gives its base and arrival number, its record goes under that number
        const uint32_t n = min(nbuf, uint32_t(a.list_cap));
        nkept = n;
        // digit 1 of the block's threshold-bin candidates into the row's digit-1
        // histogram before this CTA counts in: one thread per candidate, so a
        // thread issues one or two atomics, none of them inside a scan loop
        uint32_t* h1row = a.hist1 + int64_t(b) * kSelBins;
#pragma unroll 1
        for (uint32_t i = tid; i < n; i += T) {
          const uint64_t key = buf[i];
          if (uint32_t(key >> kSelShift[0]) == b0) atomicAdd(h1row + ((key >> kSelShift[1]) & uint64_t(kSelBins - 1)), 1u);
        }
        if (tid == 0 && n != 0u) {
          const unsigned long long old = atomicAdd(state + b, (1ull << 32) | n);
          scratch[40] = uint32_t(old);
          scratch[41] = uint32_t(old >> 32) & 0xffffu;
        }
        __syncthreads();
        if (n != 0u) {
          const uint32_t base = scratch[40], seq = scratch[41];
          uint64_t* lrow = a.list + int64_t(b) * a.list_cap;
#pragma unroll 1
          for (uint32_t i = tid; i < n; i += T)
            if (base + i < uint32_t(a.list_cap)) lrow[base + i] = buf[i];
          if (tid == 0 && seq < gridDim.x) a.blocks[int64_t(b) * gridDim.x + seq] = make_uint4(base, n, rank, 0u);
        }
      }
    }
    // count in (live or not): the last CTA of the row sees every other CTA's
    // blocks and histogram reads complete, the list's length and the number of
    // blocks
    __syncthreads();
    if (tid == 0) {
      const unsigned long long old = atom_add_acq_rel(state + b, 1ull << 48);
      scratch[43] = uint32_t(old >> 48) == nctas - 1 ? 1u : 0u;
      scratch[40] = uint32_t(old);
      scratch[41] = uint32_t(old >> 32) & 0xffffu;
    }
    __syncthreads();
    if (scratch[43] == 0u) {
      // not the row's finisher: with the attention in this launch, this CTA's
      // candidates' KV rows go toward L2 while the finisher runs (the top-k is
      // among them)
      if (mla.units > 0 && live && !overflow)
#pragma unroll 1
        for (uint32_t i = tid; i < nkept; i += T) {
          const int64_t r = addr_row(mla.kv, b, int64_t(sel_key_id(buf[i])) - a.id_base);
          if (r >= 0 && r < mla.kv.rows) bulk_prefetch_l2(mla.kv_pool + r * kMlaD, kMlaD * 2);
        }
      continue;
    }
    const uint32_t L = min(scratch[40], uint32_t(a.list_cap));
    const uint32_t nblk = min(scratch[41], uint32_t(gridDim.x));
    __syncthreads();

    if (live && overflow) {
      // massive ties: K* over the whole row's scores, then the row in position order
      int32_t* orow = a.out_ids + int64_t(b) * k;
      float* oscore = a.out_scores != nullptr ? a.out_scores + int64_t(b) * k : nullptr;
      const int64_t id0 = a.id_base;
      auto row_key = [&](int64_t i) -> uint64_t {
        return sel_key(sel_rank_u(__float_as_uint(__ldcg(srow + i))), id0 + i);
      };
      const uint64_t ks =
          sel_kstar<T>(row_key, v, uint64_t(b0) << kSelShift[0], uint32_t(k) - above, 1, hist, scratch);
      uint32_t written = 0;
#pragma unroll 1
      for (int c0 = 0; c0 < v && written < uint32_t(k); c0 += T * kSelPer) {
        uint32_t keep = 0;
        uint64_t keys[kSelPer];
#pragma unroll
        for (int j = 0; j < kSelPer; ++j) {
          const int i = c0 + j * T + tid;
          keys[j] = i < v ? row_key(i) : 0ull;
          keep |= uint32_t(i < v && keys[j] >= ks) << j;
        }
        written += sel_compact<T, kSelPer>(keep, written, grp, scratch, [&](uint32_t slot, int j) {
          if (slot >= uint32_t(k)) return;
          orow[slot] = sel_key_id(keys[j]);
          if (oscore != nullptr) oscore[slot] = sel_key_score(keys[j]);
        });
      }
    } else if (live) {
      finish_row(a, b, L, nblk, nctas, b0, above, work, hist, scratch);
    }
    // the row's ids are written (every thread's stores precede the barrier)
    __syncthreads();
    if (tid == 0) asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(a.ready + b), "r"(1u) : "memory");
    // the row's workspace back to zero for the next launch
#pragma unroll 1
    for (int i = tid; i < kSelBins; i += T) {
      a.hist[int64_t(b) * kSelBins + i] = 0u;
      a.hist1[int64_t(b) * kSelBins + i] = 0u;
    }
    if (tid == 0) state[b] = 0ull;
    __syncthreads();
  }
}

// After the selection (and the fused attention): the last CTA to leave resets
// the counters and the rows' ready flags (every other CTA has passed the barrier
// and read them).
__device__ void select_exit(const SelectArgs& a, int batch, uint32_t* scratch) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t done = atomicAdd(a.ctl + 1, 1u);
    scratch[0] = done == gridDim.x - 1 ? 1u : 0u;
    if (done == gridDim.x - 1) {
      a.ctl[0] = 0u;
      a.ctl[1] = 0u;
      a.ctl[2] = 0u;
      a.ctl[3] = 0u;
    }
  }
  __syncthreads();
  if (scratch[0] != 0u)
#pragma unroll 1
    for (int b = threadIdx.x; b < batch; b += blockDim.x) a.ready[b] = 0u;
}

// ---------------------------------------------------------------------------
// The decode step's sparse attention and LSE combine in the same launch
// (MlaFuse, after the selection).  Every CTA takes one ticket; ticket u < units
// is the tile unit (tile, sequence, head group) = (u % tiles, (u / tiles) %
// batch, u / (tiles * batch)) of mla_tile_unit.  A unit of tile >= 1 reads its
// sequence's top-k ids once they are complete: rows of at most k keys at the
// grid barrier, the others when their finisher has released ready[b].  Every
// unit counts itself done; once all are, every CTA combines a share of the
// outputs, a warp per 128 output columns of one (sequence, head).
// ---------------------------------------------------------------------------
// Waits (thread-scalar, bounded) until *p >= target with acquire semantics.
__device__ __forceinline__ bool wait_count(const uint32_t* p, uint32_t target, int32_t* err) {
  const uint64_t start = global_ns();
  for (uint32_t spin = 0;; ++spin) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    if (int32_t(v - target) >= 0) return true;
    if ((spin & 15u) == 15u && global_ns() - start > kWaitNs) {
      flag(err, DSR_ERR_TIMEOUT);
      return false;
    }
  }
}

template <int H, int HG>
__device__ void attention_unit(const SelectArgs& sel, const MlaFuse& m, const CUtensorMap* kv_map,
                               const CUtensorMap* swa_map, const int32_t* visible, const int* vis_s, int batch,
                               uint8_t* smem, uint32_t u, int32_t* err) {
  // the tile's shared memory lies below the weights, histogram and tables of
  // the indexer CTA (the host plans only tiles that fit)
  if constexpr (MlaLayout<HG>::kBytes <= IxLayout<H>::kWOff) {
    const int tile = int(u % uint32_t(m.tiles));
    const int r = int(u / uint32_t(m.tiles));
    const int b = r % batch, hg = r / batch;
    const bool wait = vis_s[b] > sel.k;
    mla_tile_unit<HG>(smem, kv_map, swa_map, m.q, m.kv, m.swa_ring, m.swa_rows, visible, sel.out_ids, sel.k,
                      m.swa_len, m.scale_log2, m.part_o, m.part_m, m.part_l, err, m.heads, tile, b, hg, m.tiles,
                      nullptr, sel.id_base, 0, false, [&] {
                        if (!wait) return;
                        if (threadIdx.x == 0) wait_count(sel.ready + b, 1u, err);
                        asm volatile("bar.sync 1, 128;" ::: "memory");  // the 128 key threads
                      });
  }
}

// Output columns [128 q, 128 q + 128) of (sequence b, head h), q = item & 3,
// (b, h) = item >> 2, by one warp: out = sum_t o_t 2^{m_t - M} / (2^{log2(e)
// sink_h - M} + sum_t l_t 2^{m_t - M}) over the tile partials t (the equation
// of lse_combine_kernel).  The statistics and the columns of the first kPre
// partials are requested together (one memory round trip); `w` holds the
// warp's tile weights.
__device__ void combine_item(const MlaFuse& m, int item, float* w, int32_t* err) {
  constexpr int kPre = 24;
  const int lane = threadIdx.x & 31;
  const int pair = item >> 2, quarter = item & 3;
  const int h = pair % m.heads, tiles = m.tiles;
  const int64_t pbase = int64_t(pair / m.heads) * tiles * m.heads + h;  // tile t at pbase + t * heads
  const int d = quarter * 128 + lane * 4;
  auto col = [&](int t) { return reinterpret_cast<const uint2*>(m.part_o + (pbase + int64_t(t) * m.heads) * kMlaDv + d); };
  uint2 raw[kPre];
#pragma unroll
  for (int j = 0; j < kPre; ++j)
    if (j < tiles) raw[j] = __ldcg(col(j));
  float mv[3], lv[3];  // tiles lane, lane + 32, lane + 64 (tiles <= 65: k <= 8192)
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int t = lane + 32 * j;
    mv[j] = t < tiles ? __ldcg(m.part_m + pbase + int64_t(t) * m.heads) : -CUDART_INF_F;
    lv[j] = t < tiles ? __ldcg(m.part_l + pbase + int64_t(t) * m.heads) : 0.f;
  }
  float sk = m.sink[h];
  if (!isfinite(sk)) {
    if (lane == 0) flag(err, DSR_ERR_NONFINITE);
    sk = 0.f;
  }
  sk *= kLog2e;
  float M = fmaxf(sk, fmaxf(mv[0], fmaxf(mv[1], mv[2])));
#pragma unroll
  for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  const float base = M == -CUDART_INF_F ? 0.f : M;
  float lsum = 0.f;
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int t = lane + 32 * j;
    if (t < tiles) {
      const float e = exp2f(mv[j] - base);
      w[t] = e;
      lsum += lv[j] * e;
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
  lsum += exp2f(sk - base);
  const float inv = 1.f / lsum;
  __syncwarp();
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  auto fma4 = [&](uint2 r, float e) {
    acc.x = fmaf(__uint_as_float(r.x << 16), e, acc.x);
    acc.y = fmaf(__uint_as_float(r.x & 0xffff0000u), e, acc.y);
    acc.z = fmaf(__uint_as_float(r.y << 16), e, acc.z);
    acc.w = fmaf(__uint_as_float(r.y & 0xffff0000u), e, acc.w);
  };
#pragma unroll
  for (int j = 0; j < kPre; ++j)
    if (j < tiles) fma4(raw[j], w[j]);
#pragma unroll 1
  for (int t0 = kPre; t0 < tiles; t0 += 8) {  // partials past kPre, 8 loads at a time
    uint2 r8[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (t0 + j < tiles) r8[j] = __ldcg(col(t0 + j));
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (t0 + j < tiles) fma4(r8[j], w[t0 + j]);
  }
  const float4 o = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
  if (!isfinite(o.x) || !isfinite(o.y) || !isfinite(o.z) || !isfinite(o.w)) flag(err, DSR_ERR_NONFINITE);
  *reinterpret_cast<float4*>(m.out + int64_t(pair) * kMlaDv + d) = o;
  __syncwarp();  // w is rewritten by the warp's next item
}

// `weights`: kIxThreads / 32 * 128 floats of shared memory outside the tile's
// (tiles <= 128: k <= 8192).
template <int H>
__device__ void attention_phase(const SelectArgs& sel, const MlaFuse& m, const CUtensorMap* kv_map,
                                const CUtensorMap* swa_map, const int32_t* visible, const int* vis_s, int batch,
                                uint8_t* smem, float* weights, uint32_t* scratch, int32_t* err) {
  // the selection's generic writes to this shared memory precede the tile's
  // async-proxy writes (row gathers) and reads (MMA operands)
  fence_proxy_async_smem();
  __syncthreads();
  if (threadIdx.x == 0) scratch[0] = atomicAdd(sel.ctl + 2, 1u);
  __syncthreads();
  const uint32_t u = scratch[0];
  if (u < uint32_t(m.units)) {
    if (m.hg == 16)
      attention_unit<H, 16>(sel, m, kv_map, swa_map, visible, vis_s, batch, smem, u, err);
    else
      attention_unit<H, 32>(sel, m, kv_map, swa_map, visible, vis_s, batch, smem, u, err);
    __syncthreads();  // the unit's partial stores precede its count (release)
    if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(sel.ctl + 3) : "memory");
  }
  if (threadIdx.x == 0) scratch[1] = wait_count(sel.ctl + 3, uint32_t(m.units), err) ? 1u : 0u;
  __syncthreads();
  if (scratch[1] == 0u) return;
  // items spread over the CTAs first (warp w of CTA c: items c + G (w + 10 j))
  constexpr int kWarps = kIxThreads / 32;
  const int items = batch * m.heads * (kMlaDv / 128);
  float* w = weights + (threadIdx.x >> 5) * 128;
#pragma unroll 1
  for (int i = int(blockIdx.x) + int(gridDim.x) * int(threadIdx.x >> 5); i < items; i += int(gridDim.x) * kWarps)
    combine_item(m, i, w, err);
}

// 32 lanes x 8 consecutive 32-bit TMEM columns
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
template <int C>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t* r) {
  if constexpr (C == 8) {
    tmem_ld8(taddr, r);
  } else {
#pragma unroll
    for (int j = 0; j < C; j += 16) tmem_ld16(taddr + j, *reinterpret_cast<uint32_t(*)[16]>(r + j));
  }
}

template <int H>
__global__ void __launch_bounds__(kIxThreads, 1)
    indexer_decode_kernel(const __grid_constant__ CUtensorMap kmap, const float* __restrict__ q,
                          const float* __restrict__ weights, const PoolAddr pa,
                          const int32_t* __restrict__ visible, float* __restrict__ scores, int64_t score_stride,
                          int32_t* err, int batch, const float* __restrict__ mla_q,
                          uint16_t* __restrict__ mla_img, int mla_heads, uint32_t* __restrict__ hist,
                          const SelectArgs sel, const __grid_constant__ CUtensorMap kv_map,
                          const __grid_constant__ CUtensorMap swa_map, const MlaFuse mla) {
  using L = IxLayout<H>;
  constexpr int N = L::N;
  constexpr int HH = H / 2;  // heads per epilogue warpgroup
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* full = bars;
  uint64_t* empty = bars + kIxStages;
  uint64_t* tfull = bars + 2 * kIxStages;
  uint64_t* tempty = tfull + kIxAcc;
  uint64_t* qfull = tempty + kIxAcc;
  uint64_t* qempty = qfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + L::kMiscOff + 4);
  int* qlonz = reinterpret_cast<int*>(smem + L::kMiscOff + 8);  // [2] q_lo != 0 per slot
  int* prefix = reinterpret_cast<int*>(smem + L::kPrefixOff);
  int* vis_s = reinterpret_cast<int*>(smem + L::kVisOff);  // validated visible counts
  int* run_s = reinterpret_cast<int*>(smem + L::kRunOff);  // ring: positions in the first run
  float* wsm = reinterpret_cast<float*>(smem + L::kWOff);
  float* xch = reinterpret_cast<float*>(smem + L::kXchOff);
  uint32_t* hsm = reinterpret_cast<uint32_t*>(smem + L::kHistOff);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // Start-up: the producer warp goes first to memory (visibility, tile prefix,
  // then block-table entries and the first tiles) and only arrives at the
  // start-up barrier; the MMA warp allocates TMEM, the epilogue clears the
  // histogram, and both wait there for the prefix.
  if (warp == 0) {
    if (lane == 0) {
      for (int i = 0; i < kIxStages; ++i) {
        mbar_init(&full[i], 1);
        mbar_init(&empty[i], 1);
      }
      for (int i = 0; i < kIxAcc; ++i) {
        mbar_init(&tfull[i], 1);
        mbar_init(&tempty[i], 256);
      }
      for (int i = 0; i < 2; ++i) {
        mbar_init(&qfull[i], 256);
        mbar_init(&qempty[i], 1);
      }
      *abort = 0;
      fence_barrier_init();
      tma_prefetch_desc(&kmap);
    }
    pdl_wait();  // pool rows / visibility may come from the preceding append kernel
    // validated visible counts, tiles per row and their prefix
    const int per_lane = (batch + 31) / 32;
    const int b0 = lane * per_lane;
    int local = 0;
    for (int b = b0; b < b0 + per_lane && b < batch; ++b) {
      int v = visible[b];
      if (v < 0 || int64_t(v) > addr_capacity(pa, b) || int64_t(v) > score_stride) {
        flag(err, DSR_ERR_ID);
        v = 0;
      }
      // a ring sequence: the positions before the wrap, then the rest from the region's first row
      const int n1 = pa.ring == nullptr ? v : int(min(int64_t(v), pa.ring[3 * int64_t(b) + 1] - pa.ring[3 * int64_t(b) + 2]));
      vis_s[b] = v;
      run_s[b] = n1;
      local += (n1 + kIxTile - 1) / kIxTile + (v - n1 + kIxTile - 1) / kIxTile;
    }
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int x = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += x;
    }
    int run = incl - local;
    for (int b = b0; b < b0 + per_lane && b < batch; ++b) {
      prefix[b] = run;
      run += (run_s[b] + kIxTile - 1) / kIxTile + (vis_s[b] - run_s[b] + kIxTile - 1) / kIxTile;
    }
    if (lane == 31) prefix[batch] = incl;
    __syncwarp();
    asm volatile("bar.arrive 1, %0;" ::"n"(kIxThreads) : "memory");
  } else {
    if (warp == 1) {
      tmem_alloc(tmem_slot, L::kTmemCols);
      if (mla.units == 0) tmem_relinquish();  // a fused attention tile allocates again
    } else {
      for (int i = threadIdx.x - 64; i < kIxHistBins; i += kIxThreads - 64) hsm[i] = 0u;
    }
    tc_fence_before();
    pdl_wait();
    asm volatile("bar.sync 1, %0;" ::"n"(kIxThreads) : "memory");
    tc_fence_after();
  }
  const uint32_t tmem_base = warp == 0 ? 0u : *tmem_slot;  // the producer never reads TMEM

  const int total = prefix[batch];
  const int t_lo = int((int64_t(total) * blockIdx.x) / gridDim.x);
  const int t_hi = int((int64_t(total) * (blockIdx.x + 1)) / gridDim.x);

  if (t_lo >= t_hi && warp >= 2 && mla_q != nullptr)
    mla_query_image(mla_q, mla_img, batch, mla_heads, threadIdx.x - 64, 256);
  if (t_lo < t_hi) {
    if (warp == 0) {
      // ------------------------------------------------------------ producer
      // The first pool rows of the 64-row halves of 16 tiles (block-table
      // entries, or ring runs) are resolved by the 32 lanes at once (one load
      // latency per 16 tiles); lane 0 then issues the TMA boxes.  Every key is
      // read once: its lines go first when L2 evicts, so the scores, the
      // selection's state and this kernel's code stay cached.
      const uint64_t stream_policy = l2_evict_first_policy();
      for (int g0 = t_lo, s0 = 0; g0 < t_hi; g0 += 16, s0 += 16) {
        const int t = g0 + (lane >> 1), blk = lane & 1;
        int32_t hrow = -1;  // -1: a half beyond the tile's keys, not loaded
        if (t < t_hi) {
          const int b = find_row(prefix, batch, t);
          int pos0, valid;
          int64_t row0;
          tile_span(pa, b, t - prefix[b], vis_s[b], run_s[b], pos0, row0, valid);
          if (blk * 64 < valid) {
            int64_t r = row0 >= 0 ? row0 + blk * 64 : addr_row(pa, b, pos0 + blk * 64);
            if (r < 0 || r >= pa.rows) {
              flag(err, DSR_ERR_ID);
              r = 0;
            }
            hrow = int32_t(r);
          }
        }
        bool ok = true;
        for (int j = 0; j < 16 && g0 + j < t_hi; ++j) {
          const int32_t r0 = __shfl_sync(0xffffffffu, hrow, 2 * j);
          const int32_t r1 = __shfl_sync(0xffffffffu, hrow, 2 * j + 1);
          if (lane == 0) {
            const int s = s0 + j;
            const int stage = s % kIxStages;
            ok = mbar_wait(&empty[stage], ((s / kIxStages) & 1) ^ 1, abort, err);
            if (ok) {
              const int nblk = r1 >= 0 ? 2 : 1;
              mbar_arrive_expect_tx(&full[stage], uint32_t(nblk) * 2u * 8192u);
              const uint32_t dst = sbase + L::kStagesOff + stage * kIxStageBytes;
#pragma unroll
              for (int kh = 0; kh < 2; ++kh) {
                tma_load_2d_hint(dst + kh * 16384, &kmap, &full[stage], kh * 64, r0, stream_policy);
                if (nblk == 2)
                  tma_load_2d_hint(dst + kh * 16384 + 8192, &kmap, &full[stage], kh * 64, r1, stream_policy);
              }
            }
          }
          if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
        }
        if (*abort) break;
      }
    } else if (warp == 1) {
      // ----------------------------------------------------------- MMA issuer
      if (lane == 0) {
        uint32_t idesc = umma_idesc_bf16(128, N, false, false);
        int b = find_row(prefix, batch, t_lo);
        int rowseq = 0;
        for (int t = t_lo, s = 0; t < t_hi; ++t, ++s) {
          if (t >= prefix[b + 1]) {  // next non-empty row
            while (t >= prefix[b + 1]) ++b;
            ++rowseq;
          }
          const bool row_first = (t == t_lo) || (t == prefix[b]);
          const bool row_last = (t + 1 == t_hi) || (t + 1 == prefix[b + 1]);
          const int slot = rowseq & 1;
          if (row_first) {
            if (!mbar_wait(&qfull[slot], (rowseq >> 1) & 1, abort, err)) break;
            // a BF16-exact query has q_lo == 0: contract only the q_hi rows
            idesc = umma_idesc_bf16(128, qlonz[slot] ? N : H, false, false);
          }
          const int stage = s % kIxStages;
          if (!mbar_wait(&full[stage], (s / kIxStages) & 1, abort, err)) break;
          const int acc = s % kIxAcc;
          if (!mbar_wait(&tempty[acc], ((s / kIxAcc) & 1) ^ 1, abort, err)) break;
          tc_fence_after();
          const uint32_t a0 = sbase + L::kStagesOff + stage * kIxStageBytes;
          const uint32_t b0 = sbase + L::kQOff + slot * L::kQSlotBytes;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t ad = umma_desc_sw128(a0 + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = umma_desc_sw128(b0 + (kk >> 2) * (N * 128) + (kk & 3) * 32, 16, 1024);
            umma_bf16(tmem_base + acc * N, ad, bd, idesc, kk > 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          umma_commit(&tfull[acc]);
          if (row_last) umma_commit(&qempty[slot]);
        }
      }
      __syncwarp();
    } else {
      // ------------------------------------------------------------- epilogue
      // Two warpgroups share every tile: warpgroup g reduces heads [g*H/2, (g+1)*H/2).
      const int et = threadIdx.x - 64;  // 0..255
      const int wg = et >> 7;
      const int row_in_tile = (warp & 3) * 32 + lane;  // TMEM lane of this thread
      int b = find_row(prefix, batch, t_lo);
      int rowseq = 0;
      uint32_t lonz0 = 1, lonz1 = 1;  // q_lo != 0 for the row in slot 0 / 1
      // prepares Q (hi/lo bf16, 128-byte swizzled K-major) and weights of row rb into slot
      auto prepare = [&](int rb, int seq) -> bool {
        const int slot = seq & 1;
        // every epilogue thread reaches the barrier reduction below, aborted or not
        const bool live = !*abort && mbar_wait(&qempty[slot], ((seq >> 1) & 1) ^ 1, abort, err);
        uint8_t* qs = smem + L::kQOff + slot * L::kQSlotBytes;
        const float4* src = reinterpret_cast<const float4*>(q + int64_t(rb) * H * 128);
        constexpr int kPer = H * 32 / 256;  // float4 per thread, all loads in flight at once
        float4 xv[kPer];
        uint32_t lo_any = 0;
#pragma unroll
        for (int j = 0; j < kPer; ++j) xv[j] = __ldg(src + et + j * 256);
#pragma unroll
        for (int j = 0; j < kPer && live; ++j) {
          const int i = et + j * 256;
          const int h = i >> 5, d = (i & 31) * 4;
          const float xs[4] = {xv[j].x, xv[j].y, xv[j].z, xv[j].w};
          uint16_t hi[4], lo[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const __nv_bfloat16 hb = __float2bfloat16_rn(xs[e]);
            hi[e] = __bfloat16_as_ushort(hb);
            lo[e] = __bfloat16_as_ushort(__float2bfloat16_rn(xs[e] - __bfloat162float(hb)));
          }
          const int half = d >> 6, col = d & 63;
          uint8_t* base = qs + half * (N * 128);
          *reinterpret_cast<uint2*>(base + sw128_offset(h, col)) =
              make_uint2(hi[0] | (uint32_t(hi[1]) << 16), hi[2] | (uint32_t(hi[3]) << 16));
          *reinterpret_cast<uint2*>(base + sw128_offset(H + h, col)) =
              make_uint2(lo[0] | (uint32_t(lo[1]) << 16), lo[2] | (uint32_t(lo[3]) << 16));
          lo_any |= (lo[0] | lo[1] | lo[2] | lo[3]) & 0x7fffu;
        }
        for (int h = et; h < H; h += 256) wsm[slot * H + h] = weights[int64_t(rb) * H + h];
        uint32_t any;
        asm volatile(
            "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
            "bar.red.or.pred q, 2, 256, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
            : "=r"(any)
            : "r"(lo_any));
        if (et == 0) qlonz[slot] = int(any);  // read by the MMA issuer after qfull
        (slot ? lonz1 : lonz0) = any;
        fence_proxy_async_smem();
        mbar_arrive(&qfull[slot]);
        return live;
      };
      // flushes the CTA's score histogram of row rb into the row's global histogram
      auto flush = [&](int rb) {
        asm volatile("bar.sync 3, 256;" ::: "memory");
        // (the fused selection takes every key of a row of at most k keys: no histogram)
        const bool add = hist != nullptr && (sel.out_ids == nullptr || vis_s[rb] > sel.k);
        if (hist != nullptr)
          for (int i = et; i < kIxHistBins; i += 256) {
            const uint32_t v = hsm[i];
            if (v) {
              if (add) atomicAdd(hist + int64_t(rb) * kIxHistBins + i, v);
              hsm[i] = 0u;
            }
          }
        asm volatile("bar.sync 3, 256;" ::: "memory");
      };
      // Every epilogue thread walks every tile and reaches every named barrier;
      // after an aborted wait it only skips the work (no early exit).
      bool live = prepare(b, 0);
      // this CTA's share of the MLA query image, after the first row's query
      if (mla_q != nullptr) mla_query_image(mla_q, mla_img, batch, mla_heads, et, 256);
      for (int t = t_lo, s = 0; t < t_hi; ++t, ++s) {
        if (t >= prefix[b + 1]) {  // next non-empty row
          flush(b);
          while (t >= prefix[b + 1]) ++b;
          ++rowseq;
        }
        // prepare the next row's query before waiting on this tile
        if (t + 1 < t_hi && t + 1 == prefix[b + 1]) {
          int nb = b + 1;
          while (t + 1 >= prefix[nb + 1]) ++nb;
          live = prepare(nb, rowseq + 1) && live;
        }
        const int acc = s % kIxAcc;
        live = live && !*abort && mbar_wait(&tfull[acc], (s / kIxAcc) & 1, abort, err);
        float score = 0.f, check = 0.f;
        if (live) {
          tc_fence_after();
          const float* w = wsm + (rowseq & 1) * H + wg * HH;
          const uint32_t taddr = tmem_base + acc * N + wg * HH + (uint32_t((warp & 3) * 32) << 16);
          if ((rowseq & 1) ? lonz1 : lonz0) {
            uint32_t hi[HH], lo[HH];
            tmem_ld_cols<HH>(taddr, hi);
            tmem_ld_cols<HH>(taddr + H, lo);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < HH; ++j) {
              const float d = __uint_as_float(hi[j]) + __uint_as_float(lo[j]);
              check += d;
              score = fmaf(fmaxf(d, 0.f), w[j], score);
            }
          } else {
            uint32_t hi[HH];
            tmem_ld_cols<HH>(taddr, hi);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < HH; ++j) {
              const float d = __uint_as_float(hi[j]);
              check += d;
              score = fmaf(fmaxf(d, 0.f), w[j], score);
            }
          }
          tc_fence_before();
          mbar_arrive(&tempty[acc]);
        }
        if (wg == 1) xch[(s & 1) * 128 + row_in_tile] = score;
        int pos0, valid;
        int64_t row0;
        tile_span(pa, b, t - prefix[b], vis_s[b], run_s[b], pos0, row0, valid);
        const int p = pos0 + row_in_tile;
        const bool mine = row_in_tile < valid;
        if (live && mine && !isfinite(check)) flag(err, DSR_ERR_NONFINITE);
        asm volatile("bar.sync 3, 256;" ::: "memory");
        if (wg == 0) {  // warp-uniform
          uint32_t digit = 0;  // digit 0 of the score's rank key; 0: no key here
          if (live && mine) {
            score += xch[(s & 1) * 128 + row_in_tile];
            if (!isfinite(score)) flag(err, DSR_ERR_NONFINITE);
            scores[int64_t(b) * score_stride + p] = score;
            // NaN ranks above +inf, as in the top-k kernel's key mapping
            digit = isnan(score) ? kIxHistBins - 1 : score_key(score) >> 21;
            atomicAdd(&hsm[digit], 1u);
          }
          // the warp's 32 keys are group (tile, warp & 3) of the row: its largest digit 0
          if (sel.gmax != nullptr && vis_s[b] > sel.k) {
            const uint32_t top = __reduce_max_sync(0xffffffffu, digit);
            if (lane == 0) sel.gmax[int64_t(b) * sel.gstride + int64_t(t - prefix[b]) * 4 + (warp & 3)] = uint16_t(top);
          }
        }
      }
      flush(b);
    }
  }
  pdl_launch_dependents();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
  // exact top-k of the scores (cooperative launches only: the phase holds grid barriers)
  if (sel.out_ids != nullptr) {
    const bool live = *abort == 0;
    __syncthreads();
    select_phase(sel, scores, score_stride, batch, prefix, vis_s, run_s, pa, t_lo, t_hi, smem + L::kStagesOff,
                 size_t(L::kWOff - L::kStagesOff), hsm, reinterpret_cast<uint32_t*>(xch), err, live, mla);
    if (mla.units > 0)
      attention_phase<H>(sel, mla, &kv_map, &swa_map, visible, vis_s, batch, smem, reinterpret_cast<float*>(hsm),
                         reinterpret_cast<uint32_t*>(xch), err);
    select_exit(sel, batch, reinterpret_cast<uint32_t*>(xch));
  }
}

template <int H>
int launch_ix(const CUtensorMap& map, const float* q, const float* weights, const PoolAddr& pa,
              const int32_t* visible, float* scores, int64_t score_stride, int32_t* err, int batch,
              const float* mla_q, uint16_t* mla_img, int mla_heads, uint32_t* hist,
              cudaStream_t stream, bool pdl, const SelectArgs& sel, const MlaFuseLaunch& fuse) {
  using L = IxLayout<H>;
  {
    const int rc = set_max_smem(indexer_decode_kernel<H>, L::kAlloc, "indexer decode");
    if (rc != DSR_OK) return rc;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(sm_count()), 1, 1);
  cfg.blockDim = dim3(kIxThreads, 1, 1);
  cfg.dynamicSmemBytes = L::kAlloc;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  DSR_REQUIRE(sel.out_ids == nullptr ||
                  size_t(L::kWOff - L::kStagesOff) >= size_t(sel.list_cap) * 8 + size_t(kSelThreads) * 16,
              "indexer decode: k %d leaves no shared memory for the selection", sel.k);
  DSR_REQUIRE(sel.out_ids == nullptr || sm_count() < kSelThreads,
              "indexer decode: %d SMs: the selection takes one CTA per SM and at most %d", sm_count(),
              kSelThreads - 1);
  DSR_REQUIRE(fuse.args.units == 0 || (sel.out_ids != nullptr && fuse.args.units <= sm_count() &&
                                       (fuse.args.hg == 16 || fuse.args.hg == 32) && fuse.args.tiles <= 128),
              "indexer decode: invalid fused attention plan");
  // with the selection: cooperative (its grid barriers need every CTA resident
  // at once) and, like the plain form, free to start while the preceding kernel
  // ends: every thread waits (griddepcontrol.wait) before it reads anything a
  // preceding kernel writes, so only the launch itself overlaps
  int n = 0;
  if (sel.out_ids != nullptr) {
    attr[n].id = cudaLaunchAttributeCooperative;
    attr[n++].val.cooperative = 1;
  }
  if (pdl || sel.out_ids != nullptr) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n++].val.programmaticStreamSerializationAllowed = 1;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  const cudaError_t e =
      cudaLaunchKernelEx(&cfg, indexer_decode_kernel<H>, map, q, weights, pa, visible, scores, score_stride,
                         err, batch, mla_q, mla_img, mla_heads, sel.out_ids != nullptr ? sel.hist : hist, sel,
                         fuse.kv_map, fuse.swa_map, fuse.args);
  if (e != cudaSuccess) return fail(DSR_ECUDA, "indexer launch: %s", cudaGetErrorString(e));
  return DSR_OK;
}

}  // namespace

int launch_indexer_decode(const float* q, const float* weights, const uint16_t* index_pool,
                          const PoolAddr& pa, const int32_t* visible, float* scores, int64_t score_stride,
                          int32_t* err, int64_t batch, int64_t heads, cudaStream_t stream,
                          bool pdl, const float* mla_q, uint16_t* mla_img, int64_t mla_heads,
                          uint32_t* hist, const SelectArgs* sel, const MlaFuseLaunch* fuse) {
  const SelectArgs none{};
  static const MlaFuseLaunch no_fuse{};  // units == 0: the maps are never read
  const SelectArgs& sa = sel != nullptr ? *sel : none;
  DSR_REQUIRE(mla_q == nullptr || (mla_img != nullptr && aligned16(mla_q) && aligned16(mla_img) &&
                                   (mla_heads == 16 || mla_heads == 32 || mla_heads == 64 ||
                                    mla_heads == 128)),
              "indexer_decode: invalid MLA query image job");
  DSR_REQUIRE(q && weights && index_pool && visible && scores && err, "indexer_decode: null pointer");
  DSR_REQUIRE(heads == 16 || heads == 32 || heads == 64,
              "indexer_decode: heads %lld not in {16,32,64}", (long long)heads);
  DSR_REQUIRE(batch > 0 && batch <= kIxMaxBatch, "indexer_decode: batch %lld outside [1,%d]",
              (long long)batch, kIxMaxBatch);
  DSR_REQUIRE(score_stride > 0 && score_stride <= (int64_t(1) << 31) - 1,
              "indexer_decode: invalid score stride");
  DSR_REQUIRE(aligned16(index_pool) && aligned16(q), "indexer_decode: pool and q must be 16-byte aligned");
  CUtensorMap map;
  const int rc = encode_tmap_bf16_2d(&map, index_pool, 128, uint64_t(pa.rows), 64, 64);
  if (rc != DSR_OK) return rc;
  switch (heads) {
    case 16:
      return launch_ix<16>(map, q, weights, pa, visible, scores, score_stride, err, int(batch), mla_q, mla_img,
                           int(mla_heads), hist, stream, pdl, sa, fuse != nullptr ? *fuse : no_fuse);
    case 32:
      return launch_ix<32>(map, q, weights, pa, visible, scores, score_stride, err, int(batch), mla_q, mla_img,
                           int(mla_heads), hist, stream, pdl, sa, fuse != nullptr ? *fuse : no_fuse);
    default:
      return launch_ix<64>(map, q, weights, pa, visible, scores, score_stride, err, int(batch), mla_q, mla_img,
                           int(mla_heads), hist, stream, pdl, sa, fuse != nullptr ? *fuse : no_fuse);
  }
}

size_t indexer_attention_room(int64_t idx_heads) {
  return idx_heads == 16 ? size_t(IxLayout<16>::kWOff)
                         : (idx_heads == 32 ? size_t(IxLayout<32>::kWOff) : size_t(IxLayout<64>::kWOff));
}

size_t select_workspace_bytes(int64_t batch, int64_t k) { return SelectLayout(batch, k, sm_count()).total; }

int select_args(SelectArgs* a, void* workspace, int64_t batch, int64_t k, int64_t id_base, int32_t* out_ids,
                float* out_scores) {
  DSR_REQUIRE(workspace != nullptr && out_ids != nullptr, "select: null workspace or output");
  DSR_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255u) == 0, "select: workspace must be 256-byte aligned");
  DSR_REQUIRE(k > 0 && k <= kSelMaxK, "select: k %lld outside [1, %d]", (long long)k, kSelMaxK);
  const SelectLayout L(batch, k, sm_count());
  uint8_t* base = static_cast<uint8_t*>(workspace);
  a->out_ids = out_ids;
  a->out_scores = out_scores;
  a->k = int(k);
  a->id_base = id_base;
  a->hist = reinterpret_cast<uint32_t*>(base + L.hist);
  a->hist1 = reinterpret_cast<uint32_t*>(base + L.hist1);
  a->ctl = reinterpret_cast<uint32_t*>(base + L.ctl);
  a->row_state = reinterpret_cast<unsigned long long*>(base + L.state);
  a->blocks = reinterpret_cast<uint4*>(base + L.blocks);
  a->ready = reinterpret_cast<uint32_t*>(base + L.ready);
  a->gmax = nullptr;  // bound by callers that reserve select_group_bytes()
  a->gstride = 0;
  a->list = reinterpret_cast<uint64_t*>(base + L.list);
  a->list_cap = int(L.cap);
  return DSR_OK;
}

}  // namespace dsr

extern "C" int dsr_indexer_decode(const float* q, const float* weights, const uint16_t* index_pool,
                                  int64_t pool_blocks, const int32_t* block_table,
                                  int64_t table_stride, const int32_t* visible, float* scores,
                                  int64_t score_stride, int32_t* err, int64_t batch, int64_t heads,
                                  void* stream) {
  dsr::clear_error();
  dsr::PoolAddr pa;
  const int rc = dsr::paged_addr(&pa, block_table, table_stride, pool_blocks, "indexer_decode");
  if (rc != DSR_OK) return rc;
  return dsr::launch_indexer_decode(q, weights, index_pool, pa, visible, scores, score_stride, err, batch, heads,
                                    dsr::as_stream(stream), false, nullptr, nullptr, 0, nullptr);
}

extern "C" int dsr_indexer_decode_ring(const float* q, const float* weights, const uint16_t* index_pool,
                                       int64_t pool_rows, const int64_t* ring, const int32_t* visible,
                                       float* scores, int64_t score_stride, int32_t* err, int64_t batch,
                                       int64_t heads, void* stream) {
  dsr::clear_error();
  dsr::PoolAddr pa;
  const int rc = dsr::ring_addr(&pa, ring, pool_rows, "indexer_decode_ring");
  if (rc != DSR_OK) return rc;
  return dsr::launch_indexer_decode(q, weights, index_pool, pa, visible, scores, score_stride, err, batch, heads,
                                    dsr::as_stream(stream), false, nullptr, nullptr, 0, nullptr);
}
