// NVLink peer exchange for the sequence-sharded decode step (sm_100a).
//
// The sharded step exchanges two payloads per decode step: every rank's ranked
// candidate lists (before the exact merge) and every rank's attention partials
// (before the log-sum-exp combine).  Both are all-gathers: rank r's payload lands
// in slot r of every rank's receive buffer.  This kernel does it with plain
// stores through CUDA IPC peer mappings over NVLink (no collective library; each
// store goes to one peer): CTA (peer p, chunk c) copies chunk c of the local payload into
// slot `rank` of p's receive buffer, then adds one to p's arrival counter for
// `rank` with a system-scope release; CTA 0 then waits (bounded) until every
// source's counter reaches epoch * chunks, and advances the local epoch.  A wait
// that runs out sets DSR_ERR_TIMEOUT and still advances the epoch; the slots of
// that exchange then hold a mix of steps, so after a timeout every rank
// re-creates its exchange buffers before exchanging again.
//
// Exchange buffer (identical layout on every rank; allocated and mapped by
// dsr_p2p_alloc / dsr_p2p_open):
//   [0, 256)                 control: u32 arrivals[DSR_P2P_MAX_WORLD], u32 epoch
//   [256, 256 + world*slot)  receive slots, slot r = rank r's payload
// Counters only grow, so no reset is needed between steps.  One receive buffer
// per exchange is enough because a decode step runs both exchanges in order on
// every rank: a peer can only write step e+1's lists after this rank sent its
// step e partials, which it does after it has read step e's lists (and likewise
// for the partials against the next step's lists).
#include "common.cuh"
#include "host_common.h"

#include <cstring>

namespace dsr {
namespace {

constexpr int kP2pThreads = 512;
constexpr int kP2pMaxWorld = DSR_P2P_MAX_WORLD;
constexpr int kCtlBytes = 256;
constexpr int kEpochIdx = kP2pMaxWorld;  // u32 index of the local epoch in the control block

struct PeerTable {
  uint8_t* buf[kP2pMaxWorld];  // exchange buffer of rank w as mapped in this process
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_sys_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__global__ void __launch_bounds__(kP2pThreads) p2p_allgather_kernel(
    const uint4* __restrict__ src, uint64_t payload16, const __grid_constant__ PeerTable peers,
    int rank, int world, uint64_t slot_bytes, int chunks, int32_t* err) {
  const int peer = int(blockIdx.x) / chunks, chunk = int(blockIdx.x) % chunks;
  uint32_t* ctl = reinterpret_cast<uint32_t*>(peers.buf[rank]);
  pdl_launch_dependents();
  pdl_wait();  // the payload comes from the preceding kernel

  // ---- chunk `chunk` of the payload into slot `rank` of peer `peer`
  const uint64_t lo = payload16 * uint64_t(chunk) / uint64_t(chunks);
  const uint64_t hi = payload16 * uint64_t(chunk + 1) / uint64_t(chunks);
  uint4* dst = reinterpret_cast<uint4*>(peers.buf[peer] + kCtlBytes + uint64_t(rank) * slot_bytes);
  for (uint64_t i = lo + threadIdx.x; i < hi; i += kP2pThreads) dst[i] = src[i];
  __syncthreads();
  if (threadIdx.x == 0)  // release at system scope: the CTA's stores (ordered by the barrier) come first
    red_release_sys_add(reinterpret_cast<uint32_t*>(peers.buf[peer]) + rank, 1u);
  if (blockIdx.x != 0) return;

  // ---- CTA 0: every source's chunks have landed here (only this CTA reads and
  // advances the local epoch, once per exchange)
  if (threadIdx.x < 32) {
    const uint32_t epoch = ctl[kEpochIdx] + 1u;
    const int w = int(threadIdx.x);
    const uint32_t target = epoch * uint32_t(chunks);
    bool done = w >= world;
    const uint64_t start = global_ns();
    for (uint32_t spin = 0;; ++spin) {
      if (!done) done = int32_t(ld_acquire_sys(ctl + w) - target) >= 0;
      if (__all_sync(0xffffffffu, done)) break;
      if ((spin & 63u) == 63u && global_ns() - start > kWaitNs) {
        if (threadIdx.x == 0) flag(err, DSR_ERR_TIMEOUT);
        break;  // a peer never arrived: the status is set
      }
    }
    // read by this rank's next exchange only; advanced after a timeout too, so
    // that a late arrival of the abandoned exchange cannot complete the next one
    if (threadIdx.x == 0) ctl[kEpochIdx] = epoch;
  }
}

}  // namespace
}  // namespace dsr

extern "C" size_t dsr_p2p_buffer_bytes(int64_t world, int64_t slot_bytes) {
  return size_t(dsr::kCtlBytes) + size_t(world) * size_t(slot_bytes);
}

extern "C" int dsr_p2p_alloc(size_t bytes, void** buffer, uint8_t* ipc_handle) {
  dsr::clear_error();
  DSR_REQUIRE(buffer && ipc_handle && bytes >= size_t(dsr::kCtlBytes), "p2p_alloc: invalid arguments");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return dsr::fail(DSR_ECUDA, "p2p_alloc: %s", cudaGetErrorString(e));
  e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return dsr::fail(DSR_ECUDA, "p2p_alloc: %s", cudaGetErrorString(e));
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *buffer = p;
  return DSR_OK;
}

extern "C" int dsr_p2p_open(const uint8_t* ipc_handle, void** peer_buffer) {
  dsr::clear_error();
  DSR_REQUIRE(ipc_handle && peer_buffer, "p2p_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return dsr::fail(DSR_ECUDA, "p2p_open: %s", cudaGetErrorString(e));
  *peer_buffer = p;
  return DSR_OK;
}

extern "C" int dsr_p2p_close(void* peer_buffer) {
  dsr::clear_error();
  const cudaError_t e = cudaIpcCloseMemHandle(peer_buffer);
  if (e != cudaSuccess) return dsr::fail(DSR_ECUDA, "p2p_close: %s", cudaGetErrorString(e));
  return DSR_OK;
}

extern "C" int dsr_p2p_free(void* buffer) {
  dsr::clear_error();
  const cudaError_t e = cudaFree(buffer);
  if (e != cudaSuccess) return dsr::fail(DSR_ECUDA, "p2p_free: %s", cudaGetErrorString(e));
  return DSR_OK;
}

extern "C" int dsr_p2p_allgather(const void* payload, int64_t payload_bytes, void* const* buffers,
                                 int64_t rank, int64_t world, int64_t slot_bytes, int64_t chunks,
                                 int32_t* err, void* stream) {
  dsr::clear_error();
  DSR_REQUIRE(payload && buffers && err, "p2p_allgather: null pointer");
  DSR_REQUIRE(world >= 1 && world <= dsr::kP2pMaxWorld && rank >= 0 && rank < world,
              "p2p_allgather: rank %lld of world %lld", (long long)rank, (long long)world);
  DSR_REQUIRE(payload_bytes > 0 && payload_bytes % 16 == 0 && slot_bytes % 16 == 0 &&
                  payload_bytes <= slot_bytes,
              "p2p_allgather: payload and slot must be 16-byte multiples, payload <= slot");
  DSR_REQUIRE(chunks >= 1 && chunks <= 64, "p2p_allgather: chunks per peer in [1, 64]");
  DSR_REQUIRE((reinterpret_cast<uintptr_t>(payload) & 15u) == 0, "p2p_allgather: payload alignment");
  dsr::PeerTable t = {};
  for (int w = 0; w < world; ++w) {
    DSR_REQUIRE(buffers[w] && (reinterpret_cast<uintptr_t>(buffers[w]) & 255u) == 0,
                "p2p_allgather: buffer %d null or not 256-byte aligned", w);
    t.buf[w] = static_cast<uint8_t*>(buffers[w]);
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(world * chunks), 1, 1);
  cfg.blockDim = dim3(dsr::kP2pThreads, 1, 1);
  cfg.stream = dsr::as_stream(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, dsr::p2p_allgather_kernel,
                                           static_cast<const uint4*>(payload), uint64_t(payload_bytes / 16),
                                           t, int(rank), int(world), uint64_t(slot_bytes), int(chunks), err);
  if (e != cudaSuccess) return dsr::fail(DSR_ECUDA, "p2p_allgather launch: %s", cudaGetErrorString(e));
  return DSR_OK;
}
