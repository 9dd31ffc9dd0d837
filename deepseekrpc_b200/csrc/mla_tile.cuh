// Sparse MLA decode attention over one 128-row tile (sm_100a): the device code
// shared by the MLA kernels of mla_decode.cu and the fused decode step of
// indexer_decode.cu.
//
// Reference equation (native/operations.cu:30-82, reference_attention.py:13-31):
//   out[b,h] = sum_i e^{s_i} v_i / (e^{sink_h} + sum_i e^{s_i}),  s_i = scale * q[b,h].k_i
// over the selected rows i (duplicates count, -1 skipped), with v_i = k_i.  The
// MLA value is the leading 512 latent columns of the 576-wide row.  One tile:
//   S^T[key, h]  = K[key,:576] . Q[h,:576]          (M=128 keys, N=HG heads)
//   O^T[d, h]    = sum_key V[key,d] P[h,key]         (M=128 dims x 4, N=HG heads)
// The KV tile in shared memory serves both products: K-major A operand for S^T
// and MN-major A operand (V^T) for O^T, so each selected row is read once.
// Partials: m in log2 units, l, unnormalised o in bf16.
#pragma once

#include <math_constants.h>

#include "common.cuh"

namespace dsr {
namespace {

constexpr int kMlaTile = 128;
constexpr int kMlaD = DSR_KV_DIM;   // 576
constexpr int kMlaDv = DSR_V_DIM;   // 512
constexpr int kMlaBlocks = kMlaD / 64;  // 9 column blocks of 64
constexpr int kMlaThreads = 160;
constexpr float kLog2e = 1.4426950408889634f;

template <int HG>
struct MlaLayout {
  static constexpr int kKvOff = 0;                         // 9 x 16 KiB
  static constexpr int kQOff = kMlaBlocks * 16384;         // 9 x HG x 128 B
  static constexpr int kQBytes = kMlaBlocks * HG * 128;
  static constexpr int kSPitch = kMlaTile + 1;             // transposed scores, words
  static constexpr int kPOff = kQOff + ((HG * kSPitch * 4 + 1023) / 1024) * 1024;  // P^T
  static constexpr int kRedOff = kQOff + kQBytes;
  static constexpr int kTpk = kMlaTile / HG;               // threads per head
  static constexpr int kRedBytes = 2 * kTpk * HG * 4;
  static constexpr int kValidOff = kRedOff + kRedBytes;       // [2][kMlaTile] (two items in flight)
  static constexpr int kBarOff = kValidOff + 2 * kMlaTile * 4;
  static constexpr int kMiscOff = kBarOff + (5 + kMlaBlocks) * 8;
  static constexpr int kBytes = kMiscOff + 16;
  static constexpr int kAlloc = kBytes + 1024;
  static constexpr uint32_t kTmemCols = 5 * HG <= 128 ? 128 : (5 * HG <= 256 ? 256 : 512);
  static_assert(kPOff + 2 * HG * 128 <= kRedOff, "P^T must fit in the query region");
};

// Row sentinel past the tensor (the gather zero-fills it): tile 0 reads the SWA rows.
__device__ __forceinline__ int32_t mla_oob_row(int tile, int64_t swa_rows, const PoolAddr& kv) {
  return tile == 0 ? int32_t(swa_rows) : int32_t(kv.rows);
}

// Row of key slot t of `tile` for sequence b (top-k ids come from the preceding
// kernel): tile 0 is the SWA window, tiles 1.. the selected positions through the
// pool addressing (block table or ring).  The SWA window is the sequence's last
// swa_len positions: by default rows b*128 .. b*128 + swa_len - 1 of the SWA
// tensor (ring row p % 128 holds position p); with swa_ring, the rows
// first + (p + offset) % slots of an SWA row pool for those positions.  `oob`
// when the slot holds no key.
__device__ __forceinline__ int32_t mla_key_row(int tile, int b, int t, int32_t oob, const PoolAddr& kv,
                                               const int64_t* __restrict__ swa_ring, int64_t swa_rows,
                                               const int32_t* __restrict__ visible,
                                               const int32_t* __restrict__ topk, int k,
                                               const int32_t* __restrict__ swa_len, int64_t id_base,
                                               int foreign_ok, int32_t* err) {
  int32_t row = oob;
  if (tile == 0) {
    int len = swa_len[b];
    if (len < 0 || len > DSR_SWA_ROWS) {
      if (t == 0) flag(err, DSR_ERR_ID);
      len = 0;
    }
    if (t < len) {
      if (swa_ring == nullptr) {
        row = b * DSR_SWA_ROWS + t;
      } else {
        const PoolAddr sa{nullptr, 0, swa_ring, swa_rows};
        int64_t first, slots, offset;
        const int64_t end = id_base + visible[b];  // one past the sequence's last position
        if (!ring_desc(sa, b, first, slots, offset) || slots < len) {
          if (t == 0) flag(err, DSR_ERR_ID);
        } else {
          row = int32_t(first + (end - len + t + offset) % slots);
        }
      }
    }
  } else {
    const int idx = (tile - 1) * kMlaTile + t;
    if (idx < k) {
      const int id = __ldcg(topk + int64_t(b) * k + idx);  // written in this launch when fused
      if (id != -1) {
        // position id lives in this pool at local row id - id_base; with
        // foreign_ok, ids owned by another shard are skipped, not errors
        const int64_t local = int64_t(id) - id_base;
        if (id < 0) {
          flag(err, DSR_ERR_ID);
        } else if (local < 0 || local >= visible[b]) {
          if (!foreign_ok) flag(err, DSR_ERR_ID);
        } else {
          const int64_t r = addr_row(kv, b, local);
          if (r < 0 || r >= kv.rows) flag(err, DSR_ERR_ID);
          else row = int32_t(r);
        }
      }
    }
  }
  return row;
}

// Warp w gathers the rows of key slots 32w..32w+31 (lane l holds slot 32w + l's
// row) as 4-row TMA gathers of 64-column slabs into the 9 swizzled column blocks
// at kv_smem, column-block major: every warp issues block 0 of its 8 row groups
// first, so the score MMA can start on block 0 while later blocks are in flight.
__device__ __forceinline__ void mla_gather_rows(uint32_t kv_smem, const CUtensorMap* map, uint64_t* bar_kv,
                                                int warp, int lane, int32_t row) {
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const int j = lane + 32 * i;
    const int jj = j < 8 * kMlaBlocks ? j : 0;
    const int c = jj >> 3, g = jj & 7;
    const int32_t r0 = __shfl_sync(0xffffffffu, row, 4 * g);
    const int32_t r1 = __shfl_sync(0xffffffffu, row, 4 * g + 1);
    const int32_t r2 = __shfl_sync(0xffffffffu, row, 4 * g + 2);
    const int32_t r3 = __shfl_sync(0xffffffffu, row, 4 * g + 3);
    if (j < 8 * kMlaBlocks)
      tma_gather4(kv_smem + c * 16384 + (warp * 32 + 4 * g) * 128, map, bar_kv + c, c * 64, r0, r1, r2, r3);
  }
}

// The 128 key threads of a tile, after the score MMA (`ok`: it completed): scores
// of key t for the HG heads -> transposed fp32 buffer (query region) -> per-head
// max / exp / sum (kTpk threads per head, HG keys each) -> P^T (bf16, K-major)
// for the O MMA, then one arrival each on bar_p, then the tile's statistics
// (log2-unit max, sum) at part_m / part_l + pidx.  Every thread reaches every
// named barrier, whatever `ok`.
template <int HG>
__device__ __forceinline__ void mla_softmax(uint8_t* smem, uint32_t tmem_s, int warp, int t, bool ok,
                                            const int* valid, float scale_log2, uint64_t* bar_p, float* red,
                                            float* __restrict__ part_m, float* __restrict__ part_l,
                                            int64_t pidx, int32_t* err) {
  using L = MlaLayout<HG>;
  float* sT = reinterpret_cast<float*>(smem + L::kQOff);  // [HG][kSPitch]
  if (ok) {
    tc_fence_after();
    const bool v = valid[t] != 0;
    const uint32_t taddr = tmem_s + (uint32_t(warp * 32) << 16);
    uint32_t r[HG];
#pragma unroll
    for (int c = 0; c < HG; c += 16) tmem_ld16(taddr + c, *reinterpret_cast<uint32_t(*)[16]>(r + c));
    tmem_wait_ld();
#pragma unroll
    for (int c = 0; c < HG; ++c) {
      const float s = __uint_as_float(r[c]) * scale_log2;
      if (v && !isfinite(s)) flag(err, DSR_ERR_NONFINITE);
      sT[c * L::kSPitch + t] = v ? s : -CUDART_INF_F;
    }
  }
  asm volatile("bar.sync 1, 128;" ::: "memory");
  const int h = t % HG, part = t / HG;
  const int kb = part * HG;  // first key of this thread
  float mx = -CUDART_INF_F;
  if (ok) {
    float m4[4] = {-CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F};  // independent chains
#pragma unroll
    for (int i = 0; i < HG; ++i) m4[i & 3] = fmaxf(m4[i & 3], sT[h * L::kSPitch + kb + i]);
    mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
    red[part * HG + h] = mx;
  }
  asm volatile("bar.sync 1, 128;" ::: "memory");
  if (ok) {
    for (int p = 0; p < L::kTpk; ++p) mx = fmaxf(mx, red[p * HG + h]);
    const float base = mx == -CUDART_INF_F ? 0.f : mx;
    uint8_t* pT = smem + L::kPOff;
    float l4[4] = {0.f, 0.f, 0.f, 0.f};  // independent chains
#pragma unroll
    for (int i0 = 0; i0 < HG; i0 += 8) {
      uint32_t packed[4];
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        const float s0 = sT[h * L::kSPitch + kb + i0 + j];
        const float s1 = sT[h * L::kSPitch + kb + i0 + j + 1];
        const __nv_bfloat16 p0 = __float2bfloat16_rn(exp2f(s0 - base));
        const __nv_bfloat16 p1 = __float2bfloat16_rn(exp2f(s1 - base));
        l4[j >> 1] += __bfloat162float(p0) + __bfloat162float(p1);
        packed[j >> 1] = __bfloat16_as_ushort(p0) | (uint32_t(__bfloat16_as_ushort(p1)) << 16);
      }
      const int key = kb + i0;  // P^T[h][key..key+7], K-major: 64 keys per column block
      *reinterpret_cast<uint4*>(pT + (key >> 6) * (HG * 128) + sw128_offset(h, key & 63)) =
          make_uint4(packed[0], packed[1], packed[2], packed[3]);
    }
    red[L::kTpk * HG + part * HG + h] = (l4[0] + l4[1]) + (l4[2] + l4[3]);
  }
  fence_proxy_async_smem();
  mbar_arrive(bar_p);
  asm volatile("bar.sync 1, 128;" ::: "memory");
  // ---- partial statistics of this tile
  if (t < HG) {
    float l = 0.f;
    for (int p = 0; p < L::kTpk; ++p) l += red[L::kTpk * HG + p * HG + t];
    part_m[pidx + t] = mx;  // identical in every thread of head t (log2 units)
    part_l[pidx + t] = l;
  }
}

// O^T (lane = value column, columns = heads) from TMEM to the bf16 tile partial
// at o (the range of fp32, half the bytes).
template <int HG>
__device__ __forceinline__ void mla_store_o(uint32_t tmem_o, int warp, int t, uint16_t* __restrict__ o) {
#pragma unroll 1
  for (int c = 0; c < kMlaDv / 128; ++c) {
    const uint32_t taddr = tmem_o + c * HG + (uint32_t(warp * 32) << 16);
    const int d = c * 128 + t;
    uint32_t r[HG];
#pragma unroll
    for (int hh = 0; hh < HG; hh += 16) tmem_ld16(taddr + hh, *reinterpret_cast<uint32_t(*)[16]>(r + hh));
    tmem_wait_ld();
#pragma unroll
    for (int hh = 0; hh < HG; ++hh)
      o[int64_t(hh) * kMlaDv + d] = __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(r[hh])));
  }
}

// One 128-row tile `tile` of sequence b and head group hg (tile 0 = SWA window,
// tiles 1.. = consecutive 128 top-k ids), its partial (m, l, o) stored at tile
// index (b * tiles + tile) * heads + hg * HG.  The CTA has at least kMlaThreads
// threads: warps 0..3 gather, convert the query and run the softmax, warp 4
// allocates TMEM and issues the MMAs, any further warps only join the two CTA
// barriers.  `smem` (1024-byte aligned) holds MlaLayout<HG>.  The 128 key
// threads call wait_ids() before they read the query image (q_img, every tile)
// or the top-k ids (tiles 1..).
template <int HG, typename WaitIds>
__device__ __forceinline__ void mla_tile_unit(uint8_t* smem, const CUtensorMap* kv_map, const CUtensorMap* swa_map,
                                              const float* __restrict__ q, const PoolAddr& kv,
                                              const int64_t* __restrict__ swa_ring, int64_t swa_rows,
                                              const int32_t* __restrict__ visible, const int32_t* topk, int k,
                                              const int32_t* __restrict__ swa_len, float scale_log2,
                                              uint16_t* __restrict__ part_o, float* __restrict__ part_m,
                                              float* __restrict__ part_l, int32_t* err, int heads, int tile,
                                              int b, int hg, int tiles, const uint16_t* __restrict__ q_img,
                                              int64_t id_base, int foreign_ok, bool pdl, WaitIds wait_ids) {
  using L = MlaLayout<HG>;
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* bar_s = bars + 0;   // S^T complete (commit)
  uint64_t* bar_p = bars + 1;   // P^T written (128 arrivals)
  uint64_t* bar_o = bars + 2;   // O^T complete (commit)
  uint64_t* bar_q = bars + 3;   // BF16 query in place (bulk copy, or converted in-kernel)
  uint64_t* bar_kv = bars + 4;  // [9] column block c of the rows gathered (TMA bytes + 1 arrival)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + L::kMiscOff + 4);
  int* valid = reinterpret_cast<int*>(smem + L::kValidOff);
  float* red = reinterpret_cast<float*>(smem + L::kRedOff);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h0 = hg * HG;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(tile == 0 ? swa_map : kv_map);
    for (int c = 0; c < kMlaBlocks; ++c) mbar_init(bar_kv + c, 1);
    mbar_init(bar_s, 1);
    mbar_init(bar_p, 128);
    mbar_init(bar_o, 1);
    mbar_init(bar_q, q_img != nullptr ? 1 : 128);  // bulk copy, or 128 converting threads
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

  if (pdl) pdl_launch_dependents();  // the combine kernel may start its prologue early

  if (warp < 4) {
    const int t = threadIdx.x;  // key slot of this thread == TMEM lane
    if (q_img != nullptr) {
      // ---- query: the preceding indexer kernel wrote the BF16 image; one bulk copy
      wait_ids();
      if (t == 0) {
        // image groups hold GI = min(heads, 64) heads: [9 blocks][GI rows][128 B];
        // this CTA's HG rows start at a multiple of 16 rows (swizzle phase kept)
        constexpr uint32_t kBytes = kMlaBlocks * HG * 128;
        const int gi = heads < 64 ? heads : 64;
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
      }
    } else {
      // ---- query: FP32 -> BF16, 128-byte swizzled K-major, 9 column blocks of HG rows
      // (8 float4 loads per thread in flight per batch)
      const float4* qsrc = reinterpret_cast<const float4*>(q + (int64_t(b) * heads + h0) * kMlaD);
      uint8_t* qs = smem + L::kQOff;
      constexpr int kTotal = HG * (kMlaD / 4);
      constexpr int kBatch = 8;
      for (int i0 = 0; i0 < kTotal; i0 += 128 * kBatch) {
        float4 xv[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
          const int i = i0 + j * 128 + t;
          if (i < kTotal) xv[j] = __ldg(qsrc + i);
        }
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
          const int i = i0 + j * 128 + t;
          if (i < kTotal) {
            const int h = i / (kMlaD / 4), d = (i % (kMlaD / 4)) * 4;
            const float4 x = xv[j];
            const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(x.x)) |
                                (uint32_t(__bfloat16_as_ushort(__float2bfloat16_rn(x.y))) << 16);
            const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(x.z)) |
                                (uint32_t(__bfloat16_as_ushort(__float2bfloat16_rn(x.w))) << 16);
            *reinterpret_cast<uint2*>(qs + (d >> 6) * (HG * 128) + sw128_offset(h, d & 63)) =
                make_uint2(lo, hi);
          }
        }
      }
      fence_proxy_async_smem();  // generic-proxy writes become visible to the MMA
      mbar_arrive(bar_q);
      if (tile != 0) wait_ids();
    }
    // ---- resolve the row of key t (top-k ids come from the preceding kernel);
    // rows past the tensor (the OOB sentinel) are zero-filled by the gather
    const int32_t oob = mla_oob_row(tile, swa_rows, kv);
    const int32_t row = mla_key_row(tile, b, t, oob, kv, swa_ring, swa_rows, visible, topk, k, swa_len, id_base,
                                    foreign_ok, err);
    valid[t] = row != oob;
    // ---- gather: 4-row TMA gathers of 64-column slabs into the 9 swizzled
    // column blocks; warp w issues the 8 x 9 gathers of its rows 32w..32w+31
    if (t == 0)
      for (int c = 0; c < kMlaBlocks; ++c) mbar_arrive_expect_tx(bar_kv + c, kMlaTile * 128);
    mla_gather_rows(sbase + L::kKvOff, tile == 0 ? swa_map : kv_map, bar_kv, warp, lane, row);

    // ---- scores, softmax over the tile's keys, P^T for the O MMA, tile statistics
    bool ok = mbar_wait(bar_s, 0, abort, err);
    const int64_t pidx = (int64_t(b) * tiles + tile) * heads + h0;
    mla_softmax<HG>(smem, tmem_s, warp, t, ok, valid, scale_log2, bar_p, red, part_m, part_l, pidx, err);
    // ---- O^T: lane = value column, columns = heads
    if (ok && mbar_wait(bar_o, 0, abort, err)) {
      tc_fence_after();
      mla_store_o<HG>(tmem_o, warp, t, part_o + pidx * kMlaDv);
    }
  } else if (warp == 4 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    // S^T column block by column block, each as soon as its rows have landed
    bool ready = mbar_wait(bar_q, 0, abort, err);
    constexpr uint32_t idesc_s = umma_idesc_bf16(128, HG, false, false);
#pragma unroll 1
    for (int c = 0; c < kMlaBlocks && ready; ++c) {
      ready = mbar_wait(bar_kv + c, 0, abort, err);
      if (!ready) break;
      tc_fence_after();
#pragma unroll
      for (int sub = 0; sub < 4; ++sub) {
        const uint64_t ad = umma_desc_sw128(sbase + L::kKvOff + c * 16384 + sub * 32, 16, 1024);
        const uint64_t bd = umma_desc_sw128(sbase + L::kQOff + c * (HG * 128) + sub * 32, 16, 1024);
        umma_bf16(tmem_s, ad, bd, idesc_s, (c | sub) != 0 ? 1u : 0u);
      }
    }
    if (ready) {
      umma_commit(bar_s);
      if (mbar_wait(bar_p, 0, abort, err)) {
        tc_fence_after();
        constexpr uint32_t idesc_o = umma_idesc_bf16(128, HG, true, false);
        // the four 128-column accumulators interleaved: consecutive MMAs are independent
#pragma unroll 1
        for (int ks = 0; ks < kMlaTile / 16; ++ks) {
#pragma unroll
          for (int c = 0; c < kMlaDv / 128; ++c) {
            // A = V^T (MN-major): 128 value columns = two 64-column blocks (LBO), 16 keys
            const uint64_t ad =
                umma_desc_sw128(sbase + L::kKvOff + (2 * c) * 16384 + ks * 2048, 16384, 1024);
            // B = P^T (K-major): HG rows x 16 keys
            const uint64_t bd = umma_desc_sw128(
                sbase + L::kPOff + (ks >> 2) * (HG * 128) + (ks & 3) * 32, 16, 1024);
            umma_bf16(tmem_o + c * HG, ad, bd, idesc_o, ks > 0 ? 1u : 0u);
          }
        }
        umma_commit(bar_o);
        mbar_wait(bar_o, 0, abort, err);  // MMAs retire before TMEM is released
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (*abort && threadIdx.x == 0) {
    // a wait gave up: let the row gathers and the query copy land before exit
    for (int c = 0; c < kMlaBlocks; ++c) mbar_drain(bar_kv + c, 0);
    if (q_img != nullptr) mbar_drain(bar_q, 0);
  }
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

}  // namespace
}  // namespace dsr
