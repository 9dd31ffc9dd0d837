// Host-side helpers shared by the C-ABI translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/dsr_b200.h"

namespace dsr {

// Where a sequence's logical positions live in a row pool (see common.cuh):
// paged through a block table of 64-row blocks, or ring-offset.
struct PoolAddr {
  const int32_t* table;  // paged: i32[batch, stride] physical 64-row block of logical block j
  int64_t stride;
  const int64_t* ring;   // ring: i64[batch][3] = {first row, slots, offset}
  int64_t rows;          // rows of the pool tensor
};
// Checked constructors (DSR_EINVAL with a message on bad arguments).
int paged_addr(PoolAddr* a, const int32_t* table, int64_t stride, int64_t pool_blocks, const char* what);
int ring_addr(PoolAddr* a, const int64_t* ring, int64_t rows, const char* what);

// Records a message for dsr_last_error() and returns `code`.
int fail(int code, const char* fmt, ...);
// Clears the calling thread's message.
void clear_error();
// Converts a pending launch error into DSR_ECUDA.
int launch_status(const char* what);
// Multiprocessor count of the current device (cached per device).
int sm_count();
// Raises the dynamic shared-memory limit of kernel `fn` on the CURRENT device to
// at least `bytes` (the attribute belongs to the device's copy of the kernel).
// Remembered per (device, kernel), thread-safe; returns DSR_OK or DSR_ECUDA.
int set_max_smem_raw(const void* fn, int bytes, const char* what);
template <typename F>
inline int set_max_smem(F* fn, size_t bytes, const char* what) {
  return set_max_smem_raw(reinterpret_cast<const void*>(fn), int(bytes), what);
}
// Encodes a 2-D bf16 tensor map (row-major [outer, inner]) with 128-byte swizzle.
int encode_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                        uint32_t box_inner, uint32_t box_outer);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

#define DSR_REQUIRE(cond, ...)                      \
  do {                                              \
    if (!(cond)) return ::dsr::fail(DSR_EINVAL, __VA_ARGS__); \
  } while (0)

// Launch helpers implemented by the kernel translation units.
int launch_topk(const float* scores, const int32_t* ids, const int32_t* lengths, int32_t* out_ids,
                float* out_scores, int32_t* err, int64_t rows, int64_t row_stride, int64_t k,
                int64_t id_base, void* workspace, size_t workspace_bytes, cudaStream_t stream,
                bool pdl, bool hist_ready);
// Top-k scratch; its first rows * 2048 uint32 are the per-row score histograms.
size_t topk_workspace_bytes(int64_t rows, int64_t row_stride);
// Leading bytes of that scratch (histograms, tickets, counts) that must be zero at launch.
size_t topk_zeroed_prefix_bytes(int64_t rows, int64_t row_stride);
struct SelectArgs;
// The sparse MLA attention and LSE combine of a decode step, run inside the
// cooperative indexer launch after the selection: one tile unit per CTA, so
// units <= the grid; units == 0: not fused (indexer_decode.cu).
struct MlaFuse {
  const float* q;  // [batch, heads, 576] fp32 query
  const uint16_t* kv_pool;
  PoolAddr kv;
  const int64_t* swa_ring;
  int64_t swa_rows;
  const int32_t* swa_len;
  const float* sink;
  float scale_log2;
  uint16_t* part_o;  // tile partials, layout of mla_workspace_bytes()
  float* part_m;
  float* part_l;
  float* out;  // [batch, heads, 512]
  int heads, hg, tiles, units;
};
struct MlaFuseLaunch {
  MlaFuse args;
  CUtensorMap kv_map, swa_map;  // one-row gather boxes over the KV pool and the SWA rows
};
// Plans the fused attention of a decode step: the checks of launch_mla_decode,
// the head group, the tensor maps.  plan->args.units stays 0 (not an error) when
// the step has more tile units than CTAs or its tile needs more than `room`
// bytes of the indexer CTA's shared memory.
int plan_fused_mla(MlaFuseLaunch* plan, size_t room, const float* q, const uint16_t* kv_pool, const PoolAddr& kv,
                   const int32_t* visible, const int32_t* topk, const uint16_t* swa, const int64_t* swa_ring,
                   int64_t swa_rows,
                   const int32_t* swa_len, const float* sink, float scale, float* out, void* workspace,
                   size_t workspace_bytes, int32_t* err, int64_t batch, int64_t heads, int64_t k);
// Tile units of a decode step's attention when it fuses into the indexer
// launch (room: indexer_attention_room()), else 0.
int fused_mla_units(size_t room, int64_t batch, int64_t heads, int64_t k);
// Shared memory of the indexer CTA (idx_heads index heads) a fused attention
// tile may use.
size_t indexer_attention_room(int64_t idx_heads);
// The decode indexer; with `sel`, the exact top-k of its scores in the same
// (cooperative) launch (select.cuh); with `fuse` (and `sel`), the step's sparse
// attention and combine too.
int launch_indexer_decode(const float* q, const float* weights, const uint16_t* index_pool,
                          const PoolAddr& pa, const int32_t* visible, float* scores, int64_t score_stride,
                          int32_t* err, int64_t batch, int64_t heads, cudaStream_t stream,
                          bool pdl, const float* mla_q = nullptr, uint16_t* mla_img = nullptr,
                          int64_t mla_heads = 0, uint32_t* hist = nullptr, const SelectArgs* sel = nullptr,
                          const MlaFuseLaunch* fuse = nullptr);
// Bytes of the fused selection's workspace (zero before first use, left zero by every completed launch).
size_t select_workspace_bytes(int64_t batch, int64_t k);
// Binds a SelectArgs to a workspace of select_workspace_bytes(batch, k).
int select_args(SelectArgs* a, void* workspace, int64_t batch, int64_t k, int64_t id_base, int32_t* out_ids,
                float* out_scores);
// Bytes of the per-group maxima (SelectArgs::gmax) for rows of score_stride
// scores, and their row pitch in groups.
inline int64_t select_group_stride(int64_t score_stride) { return 4 * (score_stride / 128 + 2); }
inline size_t select_group_bytes(int64_t batch, int64_t score_stride) {
  return ((size_t(batch) * size_t(select_group_stride(score_stride)) * 2 + 255) / 256) * 256;
}
int launch_indexer_prefill(const float* q, const float* weights, const uint16_t* index_pool,
                           int64_t pool_blocks, const int32_t* block_table, int64_t table_stride,
                           const int32_t* visible, float* scores, int64_t score_stride, int32_t* err,
                           int64_t queries, int64_t heads, cudaStream_t stream);
// Bytes of the BF16 MLA query image the indexer can emit for the MLA kernel.
inline size_t mla_query_image_bytes(int64_t batch, int64_t heads) {
  return size_t(batch) * size_t(heads) * DSR_KV_DIM * 2;
}
int launch_mla_decode(const float* q, const uint16_t* kv_pool, const PoolAddr& kv, const int32_t* visible,
                      const int32_t* topk, int64_t k, const uint16_t* swa, const int64_t* swa_ring,
                      int64_t swa_rows, const int32_t* swa_len, const float* sink, float scale, float* out,
                      void* workspace, size_t workspace_bytes, int32_t* err, int64_t batch,
                      int64_t heads, cudaStream_t stream, bool pdl,
                      const uint16_t* q_img = nullptr, int64_t id_base = 0,
                      bool partial = false, float* out_m = nullptr, float* out_l = nullptr);
size_t mla_workspace_bytes(int64_t batch, int64_t heads, int64_t k);
int launch_lse_combine(const float* part_o, const float* part_m, const float* part_l,
                       int64_t parts, const float* sink, float* out, float* out_m, float* out_l,
                       int32_t* err, int64_t batch, int64_t heads, int64_t dv,
                       cudaStream_t stream, bool pdl);

}  // namespace dsr
