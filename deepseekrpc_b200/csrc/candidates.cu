// Candidate-block mode of the lightning indexer (TiledIndexer,
// index_selection.py:62-90,108-123).
//
// Production: the scores of a dense source indexer are max-reduced over blocks
// of 8 consecutive positions (-inf past the visible keys, NaN propagates), the
// block holding the newest position (visible - 1) is pinned to +inf, and the
// `keep` best blocks (ties: lower block id) come back ascending, -1 padded --
// the reference's merge_ranked over reduced tiles, done as one exact top-k.
// Restriction: a later indexer scores only the positions of those blocks
// (below its visible count) and keeps its top-k of them.  The candidate lists
// are validated as the reference validates them: strictly increasing block ids,
// -1 padding only at the end, every block below ceil(visible / 8), and at least
// one block for a nonempty query; a violating row sets status 1 and scores
// nothing.
#include "common.cuh"
#include "host_common.h"

#include <math_constants.h>

namespace dsr {
namespace {

inline int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

// NaN-propagating maximum, as torch.amax.
__device__ __forceinline__ float max_nan(float a, float b) {
  return (isnan(a) || isnan(b)) ? CUDART_NAN_F : fmaxf(a, b);
}

// Block scores: bscores[r][j] = max(scores[r][8j .. 8j+7] below visible), the
// newest block pinned to +inf; blens[r] = ceil(visible / 8).
__global__ void __launch_bounds__(256) block_scores_kernel(
    const float* __restrict__ scores, const int32_t* __restrict__ visible, int rows,
    int64_t score_stride, float* __restrict__ bscores, int64_t bstride,
    int32_t* __restrict__ blens, int32_t* err) {
  const int64_t total = int64_t(rows) * bstride;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int r = int(i / bstride);
    const int64_t j = i - int64_t(r) * bstride;
    int64_t vis = visible[r];
    if (vis < 0 || vis > score_stride) {
      if (j == 0) flag(err, DSR_ERR_ID);
      vis = 0;
    }
    if (j == 0) blens[r] = int32_t((vis + 7) / 8);
    if (j * 8 >= vis) continue;
    const float* s = scores + int64_t(r) * score_stride + j * 8;
    float m = -CUDART_INF_F;
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (j * 8 + e < vis) m = max_nan(m, s[e]);
    if (j == (vis - 1) / 8) m = CUDART_INF_F;
    bscores[i] = m;
  }
  pdl_launch_dependents();
}

// Candidate expansion: per row, positions[r][8i+e] = blocks[r][i]*8 + e (or -1
// past the visible keys / for padding), phys[...] its pool row, count = C*8;
// cap[r] = pool rows (every pool row is a valid key for the scorer).
__global__ void __launch_bounds__(256) expand_kernel(
    const int32_t* __restrict__ blocks, int ncand, const int32_t* __restrict__ visible,
    const int32_t* __restrict__ block_table, int64_t table_stride, int64_t pool_blocks,
    int32_t* __restrict__ positions, int32_t* __restrict__ phys, int32_t* __restrict__ counts,
    int32_t* __restrict__ caps, int32_t* err) {
  __shared__ int bad;
  const int r = blockIdx.x;
  const int32_t* brow = blocks + int64_t(r) * ncand;
  int64_t vis = visible[r];
  if (threadIdx.x == 0) bad = (vis < 0 || vis > table_stride * 64) ? 1 : 0;
  __syncthreads();
  if (bad) vis = 0;
  const int64_t nblk = (vis + 7) / 8;
  int any = 0;
  for (int i = threadIdx.x; i < ncand; i += blockDim.x) {
    const int32_t b = brow[i];
    const int32_t prev = i > 0 ? brow[i - 1] : -2;
    if (b != -1) {
      any = 1;
      // strictly after the previous entry, which must itself be a block
      if (b < 0 || int64_t(b) >= nblk || (i > 0 && (prev == -1 || prev >= b))) bad = 1;
    }
  }
  any = __syncthreads_or(any);
  if (threadIdx.x == 0 && vis > 0 && !any) bad = 1;
  __syncthreads();
  if (bad) {
    if (threadIdx.x == 0) flag(err, DSR_ERR_ID);
  }
  for (int64_t i = threadIdx.x; i < int64_t(ncand) * 8; i += blockDim.x) {
    const int32_t b = bad ? -1 : brow[i >> 3];
    const int64_t p = int64_t(b) * 8 + (i & 7);
    int32_t pos = -1, row = -1;
    if (b >= 0 && p < vis) {
      const int64_t blk = block_table[int64_t(r) * table_stride + (p >> 6)];
      if (blk < 0 || blk >= pool_blocks) {
        flag(err, DSR_ERR_ID);
      } else {
        pos = int32_t(p);
        row = int32_t(blk * 64 + (p & 63));
      }
    }
    positions[int64_t(r) * ncand * 8 + i] = pos;
    phys[int64_t(r) * ncand * 8 + i] = row;
  }
  if (threadIdx.x == 0) {
    counts[r] = ncand * 8;
    caps[r] = int32_t(pool_blocks * 64);
  }
}

struct CandWs {
  size_t bscores, blens, topk, total;
  CandWs(int64_t rows, int64_t score_stride) {
    const int64_t bstride = (score_stride + 7) / 8;
    bscores = 0;
    blens = round_up(int64_t(rows) * bstride * 4, 256);
    topk = blens + round_up(rows * 4, 256);
    total = topk + topk_workspace_bytes(rows, bstride);
  }
};

struct SelWs {
  size_t positions, phys, scores, counts, caps, topk, total;
  SelWs(int64_t rows, int64_t ncand) {
    const int64_t n = ncand * 8;
    positions = 0;
    phys = round_up(rows * n * 4, 256);
    scores = phys + round_up(rows * n * 4, 256);
    counts = scores + round_up(rows * n * 4, 256);
    caps = counts + round_up(rows * 4, 256);
    topk = caps + round_up(rows * 4, 256);
    total = topk + topk_workspace_bytes(rows, n);
  }
};

}  // namespace
}  // namespace dsr

using namespace dsr;

extern "C" size_t dsr_candidate_blocks_workspace_bytes(int64_t rows, int64_t score_stride,
                                                       int64_t keep) {
  (void)keep;  // the block top-k's scratch does not depend on it
  return CandWs(rows, score_stride).total;
}

extern "C" int dsr_candidate_blocks(const float* scores, const int32_t* visible, int64_t rows,
                                    int64_t score_stride, int64_t keep, int32_t* out_blocks,
                                    void* workspace, size_t workspace_bytes, int32_t* err,
                                    void* stream) {
  clear_error();
  DSR_REQUIRE(scores && visible && out_blocks && err && workspace, "candidate_blocks: null pointer");
  DSR_REQUIRE(rows > 0 && rows <= 65535 && keep > 0 && keep <= 8192 && score_stride > 0 &&
                  score_stride <= (int64_t(1) << 31) - 1,
              "candidate_blocks: invalid shape");
  const CandWs L(rows, score_stride);
  DSR_REQUIRE(workspace_bytes >= L.total, "candidate_blocks: workspace %zu < %zu bytes",
              workspace_bytes, L.total);
  DSR_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255u) == 0,
              "candidate_blocks: workspace must be 256-byte aligned");
  const int64_t bstride = (score_stride + 7) / 8;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* bscores = reinterpret_cast<float*>(ws + L.bscores);
  int32_t* blens = reinterpret_cast<int32_t*>(ws + L.blens);
  const cudaStream_t s = as_stream(stream);
  const int64_t total = rows * bstride;
  const int grid = int((total + 255) / 256 < 8 * sm_count() ? (total + 255) / 256 : 8 * sm_count());
  block_scores_kernel<<<grid, 256, 0, s>>>(scores, visible, int(rows), score_stride, bscores, bstride,
                                           blens, err);
  const int rc = launch_status("candidate block scores launch");
  if (rc != DSR_OK) return rc;
  return launch_topk(bscores, nullptr, blens, out_blocks, nullptr, err, rows, bstride, keep, 0,
                     ws + L.topk, L.total - L.topk, s, true, false);
}

extern "C" size_t dsr_candidate_select_workspace_bytes(int64_t rows, int64_t ncand) {
  return SelWs(rows, ncand).total;
}

extern "C" int dsr_candidate_select(const float* idx_q, const float* idx_w, int64_t idx_heads,
                                    const uint16_t* index_pool, int64_t pool_blocks,
                                    const int32_t* block_table, int64_t table_stride,
                                    const int32_t* visible, const int32_t* candidate_blocks,
                                    int64_t ncand, int64_t k, int32_t* out_ids, void* workspace,
                                    size_t workspace_bytes, int32_t* err, int64_t rows,
                                    void* stream) {
  clear_error();
  DSR_REQUIRE(idx_q && idx_w && index_pool && block_table && visible && candidate_blocks &&
                  out_ids && err && workspace,
              "candidate_select: null pointer");
  DSR_REQUIRE(rows > 0 && rows <= 65535 && ncand > 0 && ncand * 8 <= 65536 && k > 0 && k <= 8192,
              "candidate_select: invalid shape");
  DSR_REQUIRE(pool_blocks > 0 && pool_blocks * 64 <= (int64_t(1) << 31) - 1 && table_stride > 0,
              "candidate_select: invalid pool or block table");
  const SelWs L(rows, ncand);
  DSR_REQUIRE(workspace_bytes >= L.total, "candidate_select: workspace %zu < %zu bytes",
              workspace_bytes, L.total);
  DSR_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255u) == 0,
              "candidate_select: workspace must be 256-byte aligned");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int32_t* positions = reinterpret_cast<int32_t*>(ws + L.positions);
  int32_t* phys = reinterpret_cast<int32_t*>(ws + L.phys);
  float* scores = reinterpret_cast<float*>(ws + L.scores);
  int32_t* counts = reinterpret_cast<int32_t*>(ws + L.counts);
  int32_t* caps = reinterpret_cast<int32_t*>(ws + L.caps);
  const cudaStream_t s = as_stream(stream);
  expand_kernel<<<unsigned(rows), 256, 0, s>>>(candidate_blocks, int(ncand), visible, block_table,
                                               table_stride, pool_blocks, positions, phys, counts,
                                               caps, err);
  int rc = launch_status("candidate expansion launch");
  if (rc != DSR_OK) return rc;
  // candidate keys scored where they lie in the pool (no gathered copy)
  rc = dsr_index_scores(idx_q, index_pool, idx_w, phys, caps, scores, err, rows, idx_heads,
                        ncand * 8, pool_blocks * 64, stream);
  if (rc != DSR_OK) return rc;
  return launch_topk(scores, positions, counts, out_ids, nullptr, err, rows, ncand * 8, k, 0,
                     ws + L.topk, L.total - L.topk, s, false, false);
}
