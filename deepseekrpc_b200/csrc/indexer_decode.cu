// Lightning-indexer decode scoring over a paged BF16 index-key pool (sm_100a).
//
// score[b,p] = sum_h w[b,h] * max(q[b,h,:] . K[row(b,p),:], 0)
// (reference equation: native/operations.cu:104-121, reference_attention.py:34-47)
//
// Layout: index_pool bf16 [pool_blocks*64, 128]; a logical block j of sequence b
// (positions 64j..64j+63) lives in physical block block_table[b, j].
//
// Kernel: persistent, one CTA per SM, tiles of 128 keys (two pool blocks).
//   warp 0      TMA producer: two 64x64 boxes per pool block, 128-byte swizzle
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2..5  epilogue: Q preparation, TMEM -> registers, ReLU, weighted
//               head reduction, score store
// D[key, n] = K[key,:] . B[n,:] with B = [q_hi ; q_lo] (N = 2*heads rows), where
// q_hi = bf16(q) and q_lo = bf16(q - q_hi): the two products summed in FP32
// reproduce the FP32 query to ~2^-17 relative, so scores track the FP32
// reference far inside the 1e-3 tolerance while the contraction runs on the
// tensor cores.  Accumulators are double-buffered in TMEM so the epilogue of
// tile i overlaps the MMA of tile i+1; smem stages are a 4-deep TMA ring.
#include "common.cuh"
#include "host_common.h"

namespace dsr {
namespace {

constexpr int kIxTile = 128;                 // keys per tile
constexpr int kIxStages = 4;
constexpr int kIxStageBytes = kIxTile * 256; // 128 keys x 128 bf16
constexpr int kIxThreads = 192;
constexpr int kIxMaxBatch = 1024;

template <int H>
struct IxLayout {
  static constexpr int N = 2 * H;
  static constexpr int kQSlotBytes = N * 256;  // two 64-column halves of N rows x 128 B
  static constexpr int kStagesOff = 0;
  static constexpr int kQOff = kIxStages * kIxStageBytes;
  static constexpr int kWOff = kQOff + 2 * kQSlotBytes;
  static constexpr int kBarOff = kWOff + 2 * H * 4;
  static constexpr int kNumBars = 2 * kIxStages + 8;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;  // tmem slot, abort flag
  static constexpr int kPrefixOff = kMiscOff + 16;
  static constexpr int kBytes = kPrefixOff + (kIxMaxBatch + 1) * 4;
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-byte alignment
  static constexpr uint32_t kTmemCols = (2 * N <= 32) ? 32 : (2 * N <= 64 ? 64 : (2 * N <= 128 ? 128 : 256));
};

__device__ __forceinline__ int find_row(const int* prefix, int batch, int t) {
  int lo = 0, hi = batch;  // prefix[lo] <= t < prefix[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (prefix[mid] <= t) lo = mid;
    else hi = mid;
  }
  return lo;
}

template <int H>
__global__ void __launch_bounds__(kIxThreads, 1)
    indexer_decode_kernel(const __grid_constant__ CUtensorMap kmap, const float* __restrict__ q,
                          const float* __restrict__ weights, const int32_t* __restrict__ block_table,
                          int64_t table_stride, const int32_t* __restrict__ visible,
                          int64_t pool_blocks, float* __restrict__ scores, int64_t score_stride,
                          int32_t* err, int batch) {
  using L = IxLayout<H>;
  constexpr int N = L::N;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* full = bars;
  uint64_t* empty = bars + kIxStages;
  uint64_t* tfull = bars + 2 * kIxStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* qfull = tfull + 4;
  uint64_t* qempty = tfull + 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + L::kMiscOff + 4);
  int* prefix = reinterpret_cast<int*>(smem + L::kPrefixOff);
  float* wsm = reinterpret_cast<float*>(smem + L::kWOff);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kIxStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
      mbar_init(&qfull[i], 128);
      mbar_init(&qempty[i], 1);
    }
    *abort = 0;
    fence_barrier_init();
    tma_prefetch_desc(&kmap);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  pdl_wait();  // pool rows / visibility may come from the preceding append kernel

  // tiles per row and their prefix (warp 0)
  if (warp == 0) {
    const int per_lane = (batch + 31) / 32;
    const int b0 = lane * per_lane;
    int local = 0;
    for (int b = b0; b < b0 + per_lane && b < batch; ++b) {
      int v = visible[b];
      if (v < 0 || int64_t(v) > table_stride * 64 || int64_t(v) > score_stride) {
        flag(err, DSR_ERR_ID);
        v = 0;
      }
      local += (v + kIxTile - 1) / kIxTile;
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
      int v = visible[b];
      if (v < 0 || int64_t(v) > table_stride * 64 || int64_t(v) > score_stride) v = 0;
      run += (v + kIxTile - 1) / kIxTile;
    }
    if (lane == 31) prefix[batch] = incl;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total = prefix[batch];
  const int t_lo = int((int64_t(total) * blockIdx.x) / gridDim.x);
  const int t_hi = int((int64_t(total) * (blockIdx.x + 1)) / gridDim.x);

  if (t_lo < t_hi) {
    if (warp == 0) {
      // ------------------------------------------------------------ producer
      if (lane == 0) {
        int b = find_row(prefix, batch, t_lo);
        for (int t = t_lo, s = 0; t < t_hi; ++t, ++s) {
          while (t >= prefix[b + 1]) ++b;
          const int tile = t - prefix[b];
          const int vis = visible[b];  // validated by the prefix pass (row has tiles)
          const int stage = s % kIxStages;
          if (!mbar_wait(&empty[stage], ((s / kIxStages) & 1) ^ 1, abort, err)) break;
          const int first = tile * kIxTile;
          const int nblk = (vis - first) > 64 ? 2 : 1;
          mbar_arrive_expect_tx(&full[stage], uint32_t(nblk) * 2u * 8192u);
          const uint32_t dst = sbase + L::kStagesOff + stage * kIxStageBytes;
          for (int blk = 0; blk < nblk; ++blk) {
            int64_t pb = block_table[int64_t(b) * table_stride + tile * 2 + blk];
            if (pb < 0 || pb >= pool_blocks) {
              flag(err, DSR_ERR_ID);
              pb = 0;
            }
            for (int kh = 0; kh < 2; ++kh)
              tma_load_2d(dst + kh * 16384 + blk * 8192, &kmap, &full[stage], kh * 64,
                          int32_t(pb * 64));
          }
        }
      }
    } else if (warp == 1) {
      // ----------------------------------------------------------- MMA issuer
      if (lane == 0) {
        constexpr uint32_t idesc = umma_idesc_bf16(128, N, false, false);
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
          if (row_first && !mbar_wait(&qfull[slot], (rowseq >> 1) & 1, abort, err)) break;
          const int stage = s % kIxStages;
          if (!mbar_wait(&full[stage], (s / kIxStages) & 1, abort, err)) break;
          const int acc = s & 1;
          if (!mbar_wait(&tempty[acc], ((s >> 1) & 1) ^ 1, abort, err)) break;
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
      const int et = threadIdx.x - 64;  // 0..127
      const int sp = warp & 3;          // TMEM sub-partition of this warp
      int b = find_row(prefix, batch, t_lo);
      int rowseq = 0;
      // prepares Q (hi/lo bf16, 128-byte swizzled K-major) and weights of row rb into slot
      auto prepare = [&](int rb, int seq) -> bool {
        const int slot = seq & 1;
        if (!mbar_wait(&qempty[slot], ((seq >> 1) & 1) ^ 1, abort, err)) return false;
        uint8_t* qs = smem + L::kQOff + slot * L::kQSlotBytes;
        const float4* src = reinterpret_cast<const float4*>(q + int64_t(rb) * H * 128);
        for (int i = et; i < H * 32; i += 128) {  // float4 index
          const int h = i >> 5, d = (i & 31) * 4;
          const float4 x = src[i];
          const float xs[4] = {x.x, x.y, x.z, x.w};
          uint16_t hi[4], lo[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const __nv_bfloat16 hb = __float2bfloat16_rn(xs[j]);
            hi[j] = __bfloat16_as_ushort(hb);
            lo[j] = __bfloat16_as_ushort(__float2bfloat16_rn(xs[j] - __bfloat162float(hb)));
          }
          const int half = d >> 6, col = d & 63;
          uint8_t* base = qs + half * (N * 128);
          *reinterpret_cast<uint2*>(base + sw128_offset(h, col)) =
              make_uint2(hi[0] | (uint32_t(hi[1]) << 16), hi[2] | (uint32_t(hi[3]) << 16));
          *reinterpret_cast<uint2*>(base + sw128_offset(H + h, col)) =
              make_uint2(lo[0] | (uint32_t(lo[1]) << 16), lo[2] | (uint32_t(lo[3]) << 16));
        }
        for (int h = et; h < H; h += 128) wsm[slot * H + h] = weights[int64_t(rb) * H + h];
        fence_proxy_async_smem();
        mbar_arrive(&qfull[slot]);
        return true;
      };
      bool ok = prepare(b, 0);
      for (int t = t_lo, s = 0; ok && t < t_hi; ++t, ++s) {
        if (t >= prefix[b + 1]) {  // next non-empty row
          while (t >= prefix[b + 1]) ++b;
          ++rowseq;
        }
        // prepare the next row's query before waiting on this tile
        if (t + 1 < t_hi && t + 1 == prefix[b + 1]) {
          int nb = b + 1;
          while (t + 1 >= prefix[nb + 1]) ++nb;
          if (!prepare(nb, rowseq + 1)) break;
        }
        const int acc = s & 1;
        if (!mbar_wait(&tfull[acc], (s >> 1) & 1, abort, err)) break;
        tc_fence_after();
        const float* w = wsm + (rowseq & 1) * H;
        const uint32_t taddr = tmem_base + acc * N + (uint32_t(sp * 32) << 16);
        float score = 0.f, check = 0.f;
#pragma unroll
        for (int c = 0; c < H; c += 16) {
          uint32_t hi[16], lo[16];
          tmem_ld16(taddr + c, hi);
          tmem_ld16(taddr + H + c, lo);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float d = __uint_as_float(hi[j]) + __uint_as_float(lo[j]);
            check += d;
            score = fmaf(fmaxf(d, 0.f), w[c + j], score);
          }
        }
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
        const int tile = t - prefix[b];
        const int p = tile * kIxTile + sp * 32 + lane;
        if (p < visible[b] && p < score_stride) {
          if (!isfinite(score) || !isfinite(check)) flag(err, DSR_ERR_NONFINITE);
          scores[int64_t(b) * score_stride + p] = score;
        }
      }
    }
  }
  pdl_launch_dependents();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

template <int H>
int launch_ix(const CUtensorMap& map, const float* q, const float* weights,
              const int32_t* block_table, int64_t table_stride, const int32_t* visible,
              int64_t pool_blocks, float* scores, int64_t score_stride, int32_t* err, int batch,
              cudaStream_t stream, bool pdl) {
  using L = IxLayout<H>;
  static bool configured = false;
  if (!configured) {
    const cudaError_t e = cudaFuncSetAttribute(
        indexer_decode_kernel<H>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
    if (e != cudaSuccess) return fail(DSR_ECUDA, "indexer smem attribute: %s", cudaGetErrorString(e));
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(sm_count()), 1, 1);
  cfg.blockDim = dim3(kIxThreads, 1, 1);
  cfg.dynamicSmemBytes = L::kAlloc;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e =
      cudaLaunchKernelEx(&cfg, indexer_decode_kernel<H>, map, q, weights, block_table, table_stride,
                         visible, pool_blocks, scores, score_stride, err, batch);
  if (e != cudaSuccess) return fail(DSR_ECUDA, "indexer launch: %s", cudaGetErrorString(e));
  return DSR_OK;
}

}  // namespace

int launch_indexer_decode(const float* q, const float* weights, const uint16_t* index_pool,
                          int64_t pool_blocks, const int32_t* block_table, int64_t table_stride,
                          const int32_t* visible, float* scores, int64_t score_stride,
                          int32_t* err, int64_t batch, int64_t heads, cudaStream_t stream,
                          bool pdl) {
  DSR_REQUIRE(q && weights && index_pool && block_table && visible && scores && err,
              "indexer_decode: null pointer");
  DSR_REQUIRE(heads == 16 || heads == 32 || heads == 64,
              "indexer_decode: heads %lld not in {16,32,64}", (long long)heads);
  DSR_REQUIRE(batch > 0 && batch <= kIxMaxBatch, "indexer_decode: batch %lld outside [1,%d]",
              (long long)batch, kIxMaxBatch);
  DSR_REQUIRE(pool_blocks > 0 && pool_blocks * 64 <= (int64_t(1) << 31) - 1,
              "indexer_decode: pool_blocks %lld outside [1, 2^25)", (long long)pool_blocks);
  DSR_REQUIRE(table_stride > 0 && table_stride * 64 <= (int64_t(1) << 31) - 1,
              "indexer_decode: invalid block-table stride");
  DSR_REQUIRE(score_stride > 0 && score_stride <= (int64_t(1) << 31) - 1,
              "indexer_decode: invalid score stride");
  DSR_REQUIRE(aligned16(index_pool) && aligned16(q), "indexer_decode: pool and q must be 16-byte aligned");
  CUtensorMap map;
  const int rc = encode_tmap_bf16_2d(&map, index_pool, 128, uint64_t(pool_blocks) * 64, 64, 64);
  if (rc != DSR_OK) return rc;
  switch (heads) {
    case 16:
      return launch_ix<16>(map, q, weights, block_table, table_stride, visible, pool_blocks, scores,
                           score_stride, err, int(batch), stream, pdl);
    case 32:
      return launch_ix<32>(map, q, weights, block_table, table_stride, visible, pool_blocks, scores,
                           score_stride, err, int(batch), stream, pdl);
    default:
      return launch_ix<64>(map, q, weights, block_table, table_stride, visible, pool_blocks, scores,
                           score_stride, err, int(batch), stream, pdl);
  }
}

}  // namespace dsr

extern "C" int dsr_indexer_decode(const float* q, const float* weights, const uint16_t* index_pool,
                                  int64_t pool_blocks, const int32_t* block_table,
                                  int64_t table_stride, const int32_t* visible, float* scores,
                                  int64_t score_stride, int32_t* err, int64_t batch, int64_t heads,
                                  void* stream) {
  dsr::clear_error();
  return dsr::launch_indexer_decode(q, weights, index_pool, pool_blocks, block_table, table_stride,
                                    visible, scores, score_stride, err, batch, heads,
                                    dsr::as_stream(stream), false);
}
