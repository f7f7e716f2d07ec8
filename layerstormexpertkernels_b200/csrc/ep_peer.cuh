// Expert-parallel peer domain: one symmetric device buffer per rank, mapped
// into every other rank of the node through CUDA IPC, so dispatch and combine
// kernels store straight into the destination GPU's memory over NVLink.
//
// Layout of each rank's buffer (all offsets 256-byte aligned):
//   control    4 KiB   dispatch_flag[64] (indexed by source rank),
//                      combine_flag[64] (indexed by expert rank), and two
//                      local completion counters (push, combine GEMM)
//   recv_rows  [cap_rows, H] bf16   rows pushed by the sources, source-major,
//                                    each source's rows in its send order
//   recv_ids   [cap_rows, k] int32  local expert id per slot (-1: elsewhere)
//   recv_w     [cap_rows, k] fp32   routing weight per slot (0 there)
//   back       [cap_slots, H] bf16  weighted per-slot rows returned by the
//                                    expert ranks, expert-rank-major, each
//                                    part in this rank's send-row/slot order
// cap_rows = max_tokens * world (a source sends a token at most once to a
// rank), cap_slots = max_tokens * topk.
//
// Synchronisation: a kernel that stores into peers publishes with a
// last-CTA-done release: every thread fences at system scope, the CTA counts
// itself on a local counter, and the last CTA stores the layer's epoch into
// the matching flag of every peer.  The consumer waits (bounded by a time
// limit, then records a device error) until every flag it needs holds the
// epoch.  Epochs grow by one per layer call; flags start at 0.
#pragma once

#include <cstring>

#include "common.cuh"

namespace lsek {

constexpr int kMaxPeers = 16;

constexpr size_t kCtrlBytes = 16384;
constexpr size_t kCtrlDispatchFlags = 0;    // uint32 [64]
constexpr size_t kCtrlCombineFlags = 256;   // uint32 [64]
constexpr size_t kCtrlPushDone = 512;       // uint32, local
constexpr size_t kCtrlGemmDone = 768;       // uint32, local
// Token-chunked combine: chunk c's flags (uint32 [64] at kCtrlChunkFlags +
// 256 c) and its local CTA counter (uint32 at kCtrlChunkDone + 4 c).
constexpr int kMaxCombineChunks = 16;
constexpr size_t kCtrlChunkFlags = 4096;
constexpr size_t kCtrlChunkDone = kCtrlChunkFlags + 256 * kMaxCombineChunks;
static_assert(kCtrlChunkDone + 4 * kMaxCombineChunks <= kCtrlBytes, "control block layout");

struct EpLayout {
  size_t recv_rows, recv_ids, recv_w, recv_tok, back, total;
  int64_t cap_rows, cap_slots;
};

inline size_t align256(size_t v) { return (v + 255) / 256 * 256; }

inline EpLayout ep_layout(int64_t max_tokens, int64_t H, int64_t k, int64_t G) {
  EpLayout l;
  l.cap_rows = max_tokens * G;
  l.cap_slots = max_tokens * k;
  l.recv_rows = kCtrlBytes;
  l.recv_ids = l.recv_rows + align256(static_cast<size_t>(l.cap_rows * H * 2));
  l.recv_w = l.recv_ids + align256(static_cast<size_t>(l.cap_rows * k * 4));
  l.recv_tok = l.recv_w + align256(static_cast<size_t>(l.cap_rows * k * 4));
  l.back = l.recv_tok + align256(static_cast<size_t>(l.cap_rows * 4));
  l.total = l.back + align256(static_cast<size_t>(l.cap_slots * H * 2));
  return l;
}

struct EpDomain {
  int device;
  int rank, world;
  int64_t max_tokens, H, k;
  EpLayout lay;
  char* local;                 // this rank's buffer (cudaMalloc)
  char* peer[kMaxPeers];       // every rank's buffer as seen from here (peer[rank] = local)
  bool imported[kMaxPeers];    // opened through IPC (closed on destroy)
};

}  // namespace lsek

// The opaque domain handle of the C ABI.
struct lsek_ep_domain {
  lsek::EpDomain d;
};

namespace lsek {

// Peer pointer table passed to kernels by value.
struct PeerTable {
  char* base[kMaxPeers];
};

inline PeerTable peer_table(const EpDomain& d) {
  PeerTable t;
  for (int g = 0; g < kMaxPeers; ++g) t.base[g] = g < d.world ? d.peer[g] : nullptr;
  return t;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Called by every thread of every CTA after its last store to peer memory:
// the last CTA to arrive stores `epoch` into flag slot `me` of the control
// block at `flag_offset` on every peer.  `done` is a zeroed local counter.
__device__ __forceinline__ void grid_release_to_peers(const PeerTable& peers, int world, int me,
                                                      size_t flag_offset, uint32_t* done,
                                                      uint32_t epoch) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t prev = atomicAdd(done, 1u);
    if (prev == gridDim.x * gridDim.y * gridDim.z - 1) {
      __threadfence_system();
      for (int g = 0; g < world; ++g)
        st_release_sys(reinterpret_cast<uint32_t*>(peers.base[g] + flag_offset) + me, epoch);
    }
  }
}

}  // namespace lsek
