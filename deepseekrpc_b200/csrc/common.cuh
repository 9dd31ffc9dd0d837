// Shared device helpers for the sm_100a kernels: status words, bounded waits,
// mbarriers, TMA, tcgen05 (UMMA) descriptors and TMEM access.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/dsr_b200.h"
#include "host_common.h"

namespace dsr {

// ---------------------------------------------------------------------------
// status word
// ---------------------------------------------------------------------------
__device__ __forceinline__ void flag(int32_t* err, int code) { atomicCAS(err, 0, code); }

__device__ __forceinline__ float bf16_to_float(uint16_t bits) {
  return __uint_as_float(static_cast<uint32_t>(bits) << 16);
}

// Order-preserving map of an fp32 score to uint32 (larger float -> larger key).
// -0.0 is canonicalised to +0.0 so that both compare equal, as torch does.
__device__ __forceinline__ uint32_t score_key(float s) {
  uint32_t b = __float_as_uint(s);
  if (b == 0x80000000u) b = 0u;
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key_score(uint32_t u) {
  uint32_t b = (u & 0x80000000u) ? (u & 0x7fffffffu) : ~u;
  return __uint_as_float(b);
}

// ---------------------------------------------------------------------------
// pool addressing: where logical position p of sequence b lives in a row pool
// ---------------------------------------------------------------------------
// Paged (ring == nullptr): 64-row blocks, block table i32[batch, stride]:
//   row = table[b * stride + p / 64] * 64 + p % 64.
// Ring (table == nullptr): the reference's DeviceRowPool / SlotMap layout
// (src/deepseekrpc/cache_pool.py:24-113, bootstrap.py:185-192), one region per
// sequence, ring[3b .. 3b+2] = {first row, slots, offset}:
//   row = first + (p + offset) % slots,
// valid when slots > 0, 0 <= offset < slots and first + slots <= rows.
// Ring descriptor of sequence b; false (and zeros) when it is invalid.
__device__ __forceinline__ bool ring_desc(const PoolAddr& a, int b, int64_t& first, int64_t& slots,
                                          int64_t& offset) {
  first = a.ring[3 * int64_t(b)];
  slots = a.ring[3 * int64_t(b) + 1];
  offset = a.ring[3 * int64_t(b) + 2];
  if (slots <= 0 || offset < 0 || offset >= slots || first < 0 || first > a.rows - slots) {
    first = slots = offset = 0;
    return false;
  }
  return true;
}

// Positions a sequence may hold: the table's capacity, or the ring's slots.
__device__ __forceinline__ int64_t addr_capacity(const PoolAddr& a, int b) {
  if (a.ring == nullptr) return a.stride * 64;
  int64_t first, slots, offset;
  return ring_desc(a, b, first, slots, offset) ? slots : 0;
}

// Pool row of position p (0 <= p < capacity) of sequence b; -1 when unmapped.
__device__ __forceinline__ int64_t addr_row(const PoolAddr& a, int b, int64_t p) {
  if (p < 0) return -1;
  if (a.ring == nullptr) {
    if ((p >> 6) >= a.stride) return -1;
    const int64_t blk = a.table[int64_t(b) * a.stride + (p >> 6)];
    if (blk < 0 || blk * 64 >= a.rows) return -1;
    return blk * 64 + (p & 63);
  }
  int64_t first, slots, offset;
  if (!ring_desc(a, b, first, slots, offset)) return -1;
  return first + (p + offset) % slots;
}

// ---------------------------------------------------------------------------
// bounded waits: every spin in this library gives up after kWaitNs of device
// time (globaltimer) and reports DSR_ERR_TIMEOUT instead of hanging the GPU.
// ---------------------------------------------------------------------------
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// The dynamic shared memory rounded up to a 1024-byte boundary (swizzled TMA and
// UMMA tiles), as an offset from the array itself: a pointer derived from the
// __shared__ array by arithmetic keeps its address space, so the accesses through
// it compile to shared-memory instructions rather than generic ones.
__device__ __forceinline__ uint8_t* align_smem_1024(uint8_t* raw) {
  return raw + ((1024u - (smem_u32(raw) & 1023u)) & 1023u);
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
// Raises the barrier's expected transaction bytes without arriving (several
// threads may each announce the copies they issue).
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete.  Returns false (and
// raises *abort and the status word) when the wait exceeds kWaitNs or another
// role of the CTA already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          int32_t* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_ns();
  for (uint32_t spin = 0;; ++spin) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((spin & 63u) == 63u) {
      if (*abort) return false;
      if (global_ns() - start > kWaitNs) {
        *abort = 1;
        flag(err, DSR_ERR_TIMEOUT);
        return false;
      }
    }
  }
}

// After an abort: waits (bounded, ignoring the abort flag) for a barrier that
// TMA copies complete, so that no copy lands in shared memory after the CTA exits.
__device__ __forceinline__ bool mbar_drain(uint64_t* bar, uint32_t parity) {
  const uint64_t start = global_ns();
  for (uint32_t spin = 0;; ++spin) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((spin & 63u) == 63u && global_ns() - start > kWaitNs) return false;
  }
}

// ---------------------------------------------------------------------------
// proxy fences
// ---------------------------------------------------------------------------
// Generic-proxy shared-memory writes (st.shared, cp.async) become visible to
// the async proxy (TMA, tcgen05.mma).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// TMA: every load lands in the issuing CTA's own shared memory
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, uint64_t* bar, int32_t x,
                                            int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
// The same load with an L2 eviction policy (from l2_evict_first_policy): data
// read once streams through L2 without displacing what stays in use.
__device__ __forceinline__ void tma_load_2d_hint(uint32_t dst, const void* tmap, uint64_t* bar, int32_t x,
                                                 int32_t y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
// L2 prefetch of `bytes` bytes at p (16-byte aligned, a multiple of 16 bytes).
__device__ __forceinline__ void bulk_prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
// An L2 cache policy that marks every line it covers evict-first.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}
// L2 prefetch of the box a 2D tiled load at (x, y) would fetch (no shared memory).
__device__ __forceinline__ void tma_prefetch_2d(const void* tmap, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(tmap)),
               "r"(x), "r"(y)
               : "memory");
}
// Row gather: four rows (y0..y3) of one box-wide column slab starting at column
// x, from a tensor map whose box is one row high; 4 x box bytes land at dst
// (128-byte aligned), swizzled like a tiled load to that address.  Rows outside
// the tensor read the fill value (zero).
__device__ __forceinline__ void tma_gather4(uint32_t dst, const void* tmap, uint64_t* bar, int32_t x,
                                            int32_t y0, int32_t y1, int32_t y2, int32_t y3) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y0), "r"(y1), "r"(y2),
      "r"(y3)
      : "memory");
}
// 1-D bulk copy global -> shared (addresses 16-byte aligned, bytes % 16 == 0).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------
// Ampere-style 16-byte async copies (used for row gathers)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst),
               "l"(reinterpret_cast<uint64_t>(src))
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// ---------------------------------------------------------------------------
// tcgen05 / TMEM
// ---------------------------------------------------------------------------
// Shared-memory matrix descriptor for a 128-byte-swizzled canonical layout.
// K-major: rows of 64 bf16 (128 B), 8-row groups `sbo` bytes apart.
// MN-major: 128 B rows along MN, consecutive K rows 128 B apart, 8-K groups
// `sbo` apart, 64-element MN blocks `lbo` apart.  Atoms are 1024-byte aligned;
// moving the start address inside a 128-byte row selects a K sub-block.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm_100
  d |= static_cast<uint64_t>(2) << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16 with BF16 A/B and FP32 accumulation.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int m, int n, bool a_mn_major,
                                                       bool b_mn_major) {
  return (1u << 4)                                   // D format F32
         | (1u << 7)                                 // A format BF16
         | (1u << 10)                                // B format BF16
         | (static_cast<uint32_t>(a_mn_major) << 15) // A major
         | (static_cast<uint32_t>(b_mn_major) << 16) // B major
         | (static_cast<uint32_t>(n >> 3) << 17)     // N
         | (static_cast<uint32_t>(m >> 4) << 24);    // M
}

// Byte offset of element (row, col) of a bf16 tile stored as 128-byte
// swizzled rows; `row` counts 128-byte rows from a 1024-byte aligned base.
__host__ __device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t col_in_row) {
  const uint32_t chunk = (col_in_row >> 3) ^ (row & 7u);
  return row * 128u + chunk * 16u + (col_in_row & 7u) * 2u;
}

__device__ __forceinline__ void tmem_alloc(uint32_t* slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] * B[smem]
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 consecutive 32-bit columns; thread i of the warp receives lane
// (taddr.lane + i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ uint32_t elect_lane0() { return (threadIdx.x & 31u) == 0u; }

// Programmatic dependent launch: wait for the preceding kernel's results /
// allow the next kernel to start its prologue.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// The MLA query of the same decode step, FP32 [batch, heads, 576] -> BF16 in the
// shared-memory image the sparse MLA kernel contracts against: per (sequence,
// 64-head group) nine 64-column blocks of group_heads rows x 128 B, 128-byte
// swizzled (dsr_mla_query_image_bytes()).  This CTA converts its share.
__device__ __forceinline__ void mla_query_image(const float* __restrict__ q, uint16_t* __restrict__ img,
                                                int batch, int heads, int tid, int nthreads) {
  const int hg = heads < 64 ? heads : 64;
  const int64_t total = int64_t(batch) * heads * (DSR_KV_DIM / 4);  // float4 units
  const int64_t lo = total * blockIdx.x / gridDim.x, hi = total * (blockIdx.x + 1) / gridDim.x;
  constexpr int kBatch = 8;
  for (int64_t i0 = lo; i0 < hi; i0 += int64_t(nthreads) * kBatch) {
    float4 v[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int64_t i = i0 + int64_t(j) * nthreads + tid;
      if (i < hi) v[j] = __ldg(reinterpret_cast<const float4*>(q) + i);
    }
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int64_t i = i0 + int64_t(j) * nthreads + tid;
      if (i < hi) {
        const int64_t bh = i / (DSR_KV_DIM / 4);
        const int d = int(i % (DSR_KV_DIM / 4)) * 4;
        const int h = int(bh % heads);
        const int64_t g = (bh / heads) * (heads / hg) + h / hg;  // (sequence, head group)
        uint8_t* base = reinterpret_cast<uint8_t*>(img) + (g * (DSR_KV_DIM / 64) + d / 64) * hg * 128;
        const uint32_t w0 = __bfloat16_as_ushort(__float2bfloat16_rn(v[j].x)) |
                            (uint32_t(__bfloat16_as_ushort(__float2bfloat16_rn(v[j].y))) << 16);
        const uint32_t w1 = __bfloat16_as_ushort(__float2bfloat16_rn(v[j].z)) |
                            (uint32_t(__bfloat16_as_ushort(__float2bfloat16_rn(v[j].w))) << 16);
        *reinterpret_cast<uint2*>(base + sw128_offset(h % hg, d & 63)) = make_uint2(w0, w1);
      }
    }
  }
}

}  // namespace dsr
