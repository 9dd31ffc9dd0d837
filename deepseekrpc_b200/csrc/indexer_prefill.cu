// Lightning-indexer scores of a chunk of prefill queries against one sequence's
// paged BF16 index-key pool (sm_100a tensor cores).
//
// score[t,p] = sum_h w[t,h] * max(q[t,h,:] . K[row(p),:], 0)   for p < visible[t]
// (reference equation: native/operations.cu:104-121, reference_attention.py:34-47;
// the reference scores prefill queries one row at a time through TiledIndexer,
// index_selection.py:79-107).  With causal visibility, visible[t] = position + 1.
//
// This is a dense contraction: every key tile is shared by all queries that see
// it, so a CTA contracts one 128-key tile against a GROUP of 256/H queries at
// once (N = 256 query-head rows), the GEMM shape the decode kernel cannot use.
// N = 256 is the widest single-CTA MMA: per K step it reads 4 KB of keys and
// 8 KB of queries from shared memory for 128x256x16 products, a third less
// shared-memory traffic per FLOP than N = 128, and half the key-tile loads
// (config 4 on a B200: 24.5 ms at N = 128, 19.5 ms at N = 256).
//   warp 0      TMA producer: 128-key tiles (two 64-key pool blocks, 128-byte swizzle)
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2..9  epilogue: two warpgroups, each owning half of the group's queries:
//               TMEM -> registers, ReLU, weighted head reduction, causal mask,
//               score store
// Work items are (query group, key tile) pairs split evenly over one persistent
// CTA per SM; a group's tiles run in order, so its query operand is staged once.
// An FP32 query that is not BF16-exact (q - bf16(q) != 0) is contracted as
// bf16(q) plus the residual bf16(q - bf16(q)), accumulated in the same TMEM
// columns by a second set of MMAs.
#include "common.cuh"
#include "host_common.h"

namespace dsr {
namespace {

constexpr int kPfTile = 128;                  // keys per tile
constexpr int kPfStages = 3;
constexpr int kPfStageBytes = kPfTile * 256;  // 128 keys x 128 bf16
constexpr int kPfThreads = 320;
constexpr int kPfAcc = 2;                     // TMEM accumulators in flight (2 x 256 columns)
constexpr int kPfN = 256;                     // query-head rows per group (the MMA's N)
constexpr int kPfMaxGroups = 96;              // per launch (the group tables share the last KB of smem)

template <int H>
struct PfLayout {
  static constexpr int QB = kPfN / H;                    // queries per group
  static constexpr int kStagesOff = 0;
  static constexpr int kQOff = kPfStages * kPfStageBytes;  // [2 halves][2 * kPfN rows: hi, lo][128 B]
  static constexpr int kQBytes = 2 * 2 * kPfN * 128;
  static constexpr int kWOff = kQOff + kQBytes;            // weights [kPfN] f32
  static constexpr int kBarOff = kWOff + kPfN * 4;
  static constexpr int kNumBars = 2 * kPfStages + 2 * kPfAcc + 2;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;  // tmem slot, abort, lo flag
  static constexpr int kPrefixOff = kMiscOff + 32;
  static constexpr int kGVisOff = kPrefixOff + (kPfMaxGroups + 1) * 4;
  static constexpr int kBytes = kGVisOff + kPfMaxGroups * 4;
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-byte alignment
  static constexpr uint32_t kTmemCols = kPfAcc * kPfN;  // 512
  static_assert(kAlloc <= 232448, "prefill CTA exceeds 227 KB of shared memory");
  static_assert(kTmemCols <= 512, "prefill accumulators exceed TMEM");
};

__device__ __forceinline__ int find_group(const int* prefix, int groups, int t) {
  int lo = 0, hi = groups;  // prefix[lo] <= t < prefix[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (prefix[mid] <= t) lo = mid;
    else hi = mid;
  }
  return lo;
}

template <int H>
__global__ void __launch_bounds__(kPfThreads, 1)
    indexer_prefill_kernel(const __grid_constant__ CUtensorMap kmap, const float* __restrict__ q,
                           const float* __restrict__ weights, const int32_t* __restrict__ block_table,
                           int64_t table_stride, const int32_t* __restrict__ visible,
                           int64_t pool_blocks, float* __restrict__ scores, int64_t score_stride,
                           int32_t* err, int queries) {
  using L = PfLayout<H>;
  constexpr int QB = L::QB;
  constexpr int QH = QB / 2;  // queries per epilogue warpgroup
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* full = bars;
  uint64_t* empty = bars + kPfStages;
  uint64_t* tfull = bars + 2 * kPfStages;
  uint64_t* tempty = tfull + kPfAcc;
  uint64_t* qfull = tempty + kPfAcc;
  uint64_t* qempty = qfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + L::kMiscOff + 4);
  int* qlonz = reinterpret_cast<int*>(smem + L::kMiscOff + 8);
  int* prefix = reinterpret_cast<int*>(smem + L::kPrefixOff);
  int* gvis = reinterpret_cast<int*>(smem + L::kGVisOff);  // keys the group's last query sees
  float* wsm = reinterpret_cast<float*>(smem + L::kWOff);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = (queries + QB - 1) / QB;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kPfStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < kPfAcc; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 256);
    }
    mbar_init(qfull, 256);
    mbar_init(qempty, 1);
    *abort = 0;
    fence_barrier_init();
    tma_prefetch_desc(&kmap);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  pdl_wait();

  // per group: the most keys any of its queries sees (validated), tiles, prefix (warp 0)
  if (warp == 0) {
    const int per_lane = (groups + 31) / 32;
    const int g0 = lane * per_lane;
    int local = 0;
    for (int g = g0; g < g0 + per_lane && g < groups; ++g) {
      int v = 0;
      for (int j = 0; j < QB; ++j) {
        const int t = g * QB + j;
        if (t < queries) {
          const int vt = visible[t];
          if (vt < 0 || int64_t(vt) > table_stride * 64 || int64_t(vt) > score_stride) flag(err, DSR_ERR_ID);
          else v = vt > v ? vt : v;
        }
      }
      gvis[g] = v;
      local += (v + kPfTile - 1) / kPfTile;
    }
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int x = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += x;
    }
    int run = incl - local;
    for (int g = g0; g < g0 + per_lane && g < groups; ++g) {
      prefix[g] = run;
      run += (gvis[g] + kPfTile - 1) / kPfTile;
    }
    if (lane == 31) prefix[groups] = incl;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total = prefix[groups];
  const int t_lo = int((int64_t(total) * blockIdx.x) / gridDim.x);
  const int t_hi = int((int64_t(total) * (blockIdx.x + 1)) / gridDim.x);

  if (t_lo < t_hi) {
    if (warp == 0) {
      // ------------------------------------------------------------ producer
      for (int g0 = t_lo, s0 = 0; g0 < t_hi; g0 += 16, s0 += 16) {
        const int t = g0 + (lane >> 1), blk = lane & 1;
        int64_t pb = -1;  // -1: block beyond the group's visible keys, not loaded
        if (t < t_hi) {
          const int g = find_group(prefix, groups, t);
          const int tile = t - prefix[g];
          if (tile * kPfTile + blk * 64 < gvis[g]) {
            pb = block_table[tile * 2 + blk];
            if (pb < 0 || pb >= pool_blocks) {
              flag(err, DSR_ERR_ID);
              pb = 0;
            }
          }
        }
        bool ok = true;
        for (int j = 0; j < 16 && g0 + j < t_hi; ++j) {
          const int64_t pb0 = __shfl_sync(0xffffffffu, pb, 2 * j);
          const int64_t pb1 = __shfl_sync(0xffffffffu, pb, 2 * j + 1);
          if (lane == 0) {
            const int s = s0 + j;
            const int stage = s % kPfStages;
            ok = mbar_wait(&empty[stage], ((s / kPfStages) & 1) ^ 1, abort, err);
            if (ok) {
              const int nblk = pb1 >= 0 ? 2 : 1;
              mbar_arrive_expect_tx(&full[stage], uint32_t(nblk) * 2u * 8192u);
              const uint32_t dst = sbase + L::kStagesOff + stage * kPfStageBytes;
#pragma unroll
              for (int kh = 0; kh < 2; ++kh) {
                tma_load_2d(dst + kh * 16384, &kmap, &full[stage], kh * 64, int32_t(pb0 * 64));
                if (nblk == 2)
                  tma_load_2d(dst + kh * 16384 + 8192, &kmap, &full[stage], kh * 64, int32_t(pb1 * 64));
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
        constexpr uint32_t idesc = umma_idesc_bf16(128, kPfN, false, false);
        int g = find_group(prefix, groups, t_lo);
        int gseq = 0;
        bool lonz = false;
        for (int t = t_lo, s = 0; t < t_hi; ++t, ++s) {
          if (t >= prefix[g + 1]) {  // next non-empty group
            while (t >= prefix[g + 1]) ++g;
            ++gseq;
          }
          const bool first = (t == t_lo) || (t == prefix[g]);
          const bool last = (t + 1 == t_hi) || (t + 1 == prefix[g + 1]);
          if (first) {
            if (!mbar_wait(qfull, gseq & 1, abort, err)) break;
            lonz = *qlonz != 0;
          }
          const int stage = s % kPfStages;
          if (!mbar_wait(&full[stage], (s / kPfStages) & 1, abort, err)) break;
          const int acc = s % kPfAcc;
          if (!mbar_wait(&tempty[acc], ((s / kPfAcc) & 1) ^ 1, abort, err)) break;
          tc_fence_after();
          const uint32_t a0 = sbase + L::kStagesOff + stage * kPfStageBytes;
          const uint32_t b0 = sbase + L::kQOff;
          // bf16(q) rows, then (for an inexact FP32 q) the residual rows into the same columns
          for (int part = 0; part < (lonz ? 2 : 1); ++part) {
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              const uint64_t ad = umma_desc_sw128(a0 + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
              const uint64_t bd = umma_desc_sw128(
                  b0 + (kk >> 2) * (2 * kPfN * 128) + part * (kPfN * 128) + (kk & 3) * 32, 16, 1024);
              umma_bf16(tmem_base + acc * kPfN, ad, bd, idesc, (kk > 0 || part > 0) ? 1u : 0u);
            }
          }
          umma_commit(&empty[stage]);
          umma_commit(&tfull[acc]);
          if (last) umma_commit(qempty);
        }
      }
      __syncwarp();
    } else {
      // ------------------------------------------------------------- epilogue
      const int et = threadIdx.x - 64;  // 0..255
      const int wg = et >> 7;           // owns queries [wg*QH, wg*QH + QH) of the group
      const int row_in_tile = (warp & 3) * 32 + lane;  // TMEM lane of this thread
      int g = find_group(prefix, groups, t_lo);
      int gseq = 0;
      int qvis[QH];  // visible keys of this warpgroup's queries in the current group
      // stages the group's queries (bf16 and residual, swizzled K-major) and weights
      auto prepare = [&](int gg, int seq) -> bool {
        // every epilogue thread reaches the barrier reduction below, aborted or not
        const bool live = !*abort && mbar_wait(qempty, (seq & 1) ^ 1, abort, err);
        uint8_t* qs = smem + L::kQOff;
        const int t0 = gg * QB;
        constexpr int kPer = kPfN * 32 / 256;  // float4 per thread
        constexpr int kBatch = 16;             // loads in flight per thread
        static_assert(kPer % kBatch == 0, "query staging batches");
        uint32_t lo_any = 0;
#pragma unroll 1
        for (int j0 = 0; j0 < kPer; j0 += kBatch) {
        float4 xv[kBatch];
#pragma unroll
        for (int jj = 0; jj < kBatch; ++jj) {
          const int i = et + (j0 + jj) * 256;   // float4 index in the group's [QB*H][128]
          const int t = t0 + (i >> 5) / H;      // query of this float4
          xv[jj] = t < queries ? __ldg(reinterpret_cast<const float4*>(q + int64_t(t0) * H * 128) + i)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int jj = 0; jj < kBatch && live; ++jj) {
          const int j = j0 + jj;
          const int i = et + j * 256;
          const int n = i >> 5, d = (i & 31) * 4;  // query-head row, column
          const float xs[4] = {xv[jj].x, xv[jj].y, xv[jj].z, xv[jj].w};
          uint16_t hi[4], lo[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const __nv_bfloat16 hb = __float2bfloat16_rn(xs[e]);
            hi[e] = __bfloat16_as_ushort(hb);
            lo[e] = __bfloat16_as_ushort(__float2bfloat16_rn(xs[e] - __bfloat162float(hb)));
          }
          uint8_t* base = qs + (d >> 6) * (2 * kPfN * 128);
          *reinterpret_cast<uint2*>(base + sw128_offset(n, d & 63)) =
              make_uint2(hi[0] | (uint32_t(hi[1]) << 16), hi[2] | (uint32_t(hi[3]) << 16));
          *reinterpret_cast<uint2*>(base + sw128_offset(kPfN + n, d & 63)) =
              make_uint2(lo[0] | (uint32_t(lo[1]) << 16), lo[2] | (uint32_t(lo[3]) << 16));
          lo_any |= (lo[0] | lo[1] | lo[2] | lo[3]) & 0x7fffu;
        }
        }
        if (et < kPfN) {
          const int t = t0 + et / H;
          wsm[et] = t < queries ? weights[int64_t(t0) * H + et] : 0.f;
        }
        uint32_t any;
        asm volatile(
            "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
            "bar.red.or.pred q, 2, 256, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
            : "=r"(any)
            : "r"(lo_any));
        if (et == 0) *qlonz = int(any);  // read by the MMA issuer after qfull
#pragma unroll
        for (int j = 0; j < QH; ++j) {
          const int t = t0 + wg * QH + j;
          qvis[j] = t < queries ? visible[t] : 0;
        }
        fence_proxy_async_smem();
        mbar_arrive(qfull);
        return live;
      };
      bool live = prepare(g, 0);
      for (int t = t_lo, s = 0; t < t_hi; ++t, ++s) {
        if (t >= prefix[g + 1]) {  // next non-empty group (staged at the previous tile)
          while (t >= prefix[g + 1]) ++g;
          ++gseq;
        }
        const int acc = s % kPfAcc;
        live = live && !*abort && mbar_wait(&tfull[acc], (s / kPfAcc) & 1, abort, err);
        float score[QH], check = 0.f;
#pragma unroll
        for (int j = 0; j < QH; ++j) score[j] = 0.f;
        if (live) {
          tc_fence_after();
          const uint32_t taddr = tmem_base + acc * kPfN + wg * (kPfN / 2) + (uint32_t((warp & 3) * 32) << 16);
          uint32_t v[kPfN / 2];
#pragma unroll
          for (int c = 0; c < kPfN / 2; c += 16) tmem_ld16(taddr + c, *reinterpret_cast<uint32_t(*)[16]>(v + c));
          tmem_wait_ld();
          tc_fence_before();
          mbar_arrive(&tempty[acc]);
          const float* w = wsm + wg * (kPfN / 2);
#pragma unroll
          for (int j = 0; j < QH; ++j)
#pragma unroll
            for (int h = 0; h < H; ++h) {
              const float d = __uint_as_float(v[j * H + h]);
              check += d;
              score[j] = fmaf(fmaxf(d, 0.f), w[j * H + h], score[j]);
            }
        }
        const int tile = t - prefix[g];
        const int p = tile * kPfTile + row_in_tile;
        const int tq0 = g * QB + wg * QH;
        if (live) {
          bool seen = false;
#pragma unroll
          for (int j = 0; j < QH; ++j) {
            if (p < qvis[j]) {
              seen = true;
              if (!isfinite(score[j])) flag(err, DSR_ERR_NONFINITE);
              scores[int64_t(tq0 + j) * score_stride + p] = score[j];
            }
          }
          if (seen && !isfinite(check)) flag(err, DSR_ERR_NONFINITE);
        }
        // stage the next group's queries once this group's MMAs are all issued
        if (t + 1 < t_hi && t + 1 == prefix[g + 1]) {
          int ng = g + 1;
          while (t + 1 >= prefix[ng + 1]) ++ng;
          live = prepare(ng, gseq + 1) && live;
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
int launch_pf(const CUtensorMap& map, const float* q, const float* weights,
              const int32_t* block_table, int64_t table_stride, const int32_t* visible,
              int64_t pool_blocks, float* scores, int64_t score_stride, int32_t* err, int queries,
              cudaStream_t stream) {
  using L = PfLayout<H>;
  {
    const int rc = set_max_smem(indexer_prefill_kernel<H>, L::kAlloc, "prefill indexer");
    if (rc != DSR_OK) return rc;
  }
  indexer_prefill_kernel<H><<<sm_count(), kPfThreads, L::kAlloc, stream>>>(
      map, q, weights, block_table, table_stride, visible, pool_blocks, scores, score_stride, err,
      queries);
  return launch_status("prefill indexer launch");
}

}  // namespace

int launch_indexer_prefill(const float* q, const float* weights, const uint16_t* index_pool,
                           int64_t pool_blocks, const int32_t* block_table, int64_t table_stride,
                           const int32_t* visible, float* scores, int64_t score_stride, int32_t* err,
                           int64_t queries, int64_t heads, cudaStream_t stream) {
  DSR_REQUIRE(q && weights && index_pool && block_table && visible && scores && err,
              "indexer_prefill: null pointer");
  DSR_REQUIRE(heads == 32 || heads == 64, "indexer_prefill: heads %lld not in {32,64}",
              (long long)heads);
  DSR_REQUIRE(queries > 0 && queries <= (int64_t(1) << 24), "indexer_prefill: invalid query count");
  DSR_REQUIRE(pool_blocks > 0 && pool_blocks * 64 <= (int64_t(1) << 31) - 1,
              "indexer_prefill: pool_blocks %lld outside [1, 2^25)", (long long)pool_blocks);
  DSR_REQUIRE(table_stride > 0 && table_stride * 64 <= (int64_t(1) << 31) - 1,
              "indexer_prefill: invalid block-table length");
  DSR_REQUIRE(score_stride > 0 && score_stride <= (int64_t(1) << 31) - 1,
              "indexer_prefill: invalid score stride");
  DSR_REQUIRE(aligned16(index_pool) && aligned16(q), "indexer_prefill: pool and q must be 16-byte aligned");
  CUtensorMap map;
  int rc = encode_tmap_bf16_2d(&map, index_pool, 128, uint64_t(pool_blocks) * 64, 64, 64);
  if (rc != DSR_OK) return rc;
  // launches of at most kPfMaxGroups query groups each
  const int64_t per_launch = int64_t(kPfMaxGroups) * (kPfN / heads);
  for (int64_t t0 = 0; t0 < queries; t0 += per_launch) {
    const int n = int(queries - t0 < per_launch ? queries - t0 : per_launch);
    const float* qc = q + t0 * heads * 128;
    const float* wc = weights + t0 * heads;
    float* sc = scores + t0 * score_stride;
    rc = heads == 32 ? launch_pf<32>(map, qc, wc, block_table, table_stride, visible + t0, pool_blocks,
                                     sc, score_stride, err, n, stream)
                     : launch_pf<64>(map, qc, wc, block_table, table_stride, visible + t0, pool_blocks,
                                     sc, score_stride, err, n, stream);
    if (rc != DSR_OK) return rc;
  }
  return DSR_OK;
}

}  // namespace dsr

extern "C" int dsr_indexer_prefill(const float* q, const float* weights, const uint16_t* index_pool,
                                   int64_t pool_blocks, const int32_t* block_table,
                                   int64_t table_len, const int32_t* visible, float* scores,
                                   int64_t score_stride, int32_t* err, int64_t queries,
                                   int64_t heads, void* stream) {
  dsr::clear_error();
  return dsr::launch_indexer_prefill(q, weights, index_pool, pool_blocks, block_table, table_len,
                                     visible, scores, score_stride, err, queries, heads,
                                     dsr::as_stream(stream));
}
