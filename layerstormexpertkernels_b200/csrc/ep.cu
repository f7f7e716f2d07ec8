// Expert-parallel dispatch and combine: the device side.
//
// Experts are sharded over G ranks (rank g owns experts [g*E/G, (g+1)*E/G)).
// A token goes once to every rank that owns at least one of its experts; the
// expert rank sends back one weighted bf16 row per (token, slot) it served,
// and the token's rank sums the slots in fixed slot order.  The reference
// defines this canonical per-slot combine (smxx/permute/moe_permute.h:67-99,
// moe_permute.cu:310-329, 378-388) and models the cross-GPU step as an
// all-reduce of [T, topk, H] (tests/test_kernels.py:131-142, 187-200); here
// the exchange is two all-to-alls carrying only the rows that cross ranks.
//
// Layouts (all produced and consumed by the kernels below; the all-to-alls
// between them are issued by the host over NCCL):
//   pair keys    [T*G]  key of (token t, rank g): g if t has an expert on g,
//                       else G; a stable counting sort of the keys gives
//   send_off     [G+1]  start of each rank's send rows (send_off[G] = rows)
//   pair_row     [T*G]  send row of (t, g) (>= send_off[G] when not sent)
//   send rows    [rows, H] hidden rows, rank-major, token order inside a rank
//   send ids/w   [rows, k] per slot: the expert's index on the target rank
//                       (-1 when the slot's expert lives elsewhere) and weight
//   slot_row     [rows+1] exclusive scan of the valid slots per row; on the
//                       sender it locates each returned slot, on the expert
//                       rank it places each outgoing slot
//   combine rows [sum of valid slots, H] bf16(w * y), in received-row order
#include "common.cuh"
#include "ep_peer.cuh"

namespace lsek {
lsek_status launch_route(const int32_t* idx, int64_t n, int E, int32_t* offsets, int32_t* s2d,
                         int32_t* perm, void* ws, cudaStream_t st);
size_t permute_workspace_bytes(int64_t n_keys, int num_experts);

namespace {

constexpr int kThreads = 128;

__device__ __forceinline__ bool owned_by(int32_t e, int E, int per_rank, int g) {
  return e >= 0 && e < E && e / per_rank == g;
}

// keys[t*G + g] = g when token t has an expert on rank g, else G; adds the
// number of (t, slot) pairs served by rank g into counts[2g + 1].
__global__ void __launch_bounds__(256) ep_pair_keys_kernel(const int32_t* __restrict__ idx, int T,
                                                           int k, int E, int G,
                                                           int32_t* __restrict__ keys,
                                                           int32_t* __restrict__ counts) {
  __shared__ int s_slots[64];
  for (int g = threadIdx.x; g < G; g += blockDim.x) s_slots[g] = 0;
  __syncthreads();
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i < static_cast<int64_t>(T) * G) {
    const int t = static_cast<int>(i / G), g = static_cast<int>(i - static_cast<int64_t>(t) * G);
    const int per = E / G;
    int n = 0;
    for (int j = 0; j < k; ++j) n += owned_by(__ldg(idx + static_cast<int64_t>(t) * k + j), E, per, g);
    keys[i] = n > 0 ? g : G;
    if (n > 0) atomicAdd(&s_slots[g], n);
  }
  __syncthreads();
  for (int g = threadIdx.x; g < G; g += blockDim.x)
    if (s_slots[g] > 0) atomicAdd(counts + 2 * g + 1, s_slots[g]);
}

// counts[2g] = rows sent to rank g.
__global__ void ep_row_counts_kernel(const int32_t* __restrict__ send_off, int G,
                                     int32_t* __restrict__ counts) {
  const int g = threadIdx.x;
  if (g < G) counts[2 * g] = send_off[g + 1] - send_off[g];
}

// One CTA per token: reads its row once and writes it to each send row,
// with the per-slot local ids and weights of that row.
__global__ void __launch_bounds__(kThreads) ep_dispatch_pack_kernel(
    uint4* __restrict__ send_rows, int32_t* __restrict__ send_ids, float* __restrict__ send_w,
    const uint4* __restrict__ hidden, const int32_t* __restrict__ idx, const float* __restrict__ w,
    const int32_t* __restrict__ pair_row, const int32_t* __restrict__ send_off, int32_t capacity,
    int k, int64_t vec_per_row, int E, int G) {
  __shared__ int32_t s_row[64];
  const int t = blockIdx.x;
  const int32_t rows = min(__ldg(send_off + G), capacity);
  const int per = E / G;
  for (int g = threadIdx.x; g < G; g += kThreads) s_row[g] = __ldg(pair_row + static_cast<int64_t>(t) * G + g);
  __syncthreads();
  // metadata: thread (g, j) pairs
  for (int i = threadIdx.x; i < G * k; i += kThreads) {
    const int g = i / k, j = i - (i / k) * k;
    const int32_t row = s_row[g];
    if (row >= rows) continue;
    const int32_t e = __ldg(idx + static_cast<int64_t>(t) * k + j);
    const bool mine = owned_by(e, E, per, g);
    send_ids[static_cast<int64_t>(row) * k + j] = mine ? e - g * per : -1;
    send_w[static_cast<int64_t>(row) * k + j] = mine ? __ldg(w + static_cast<int64_t>(t) * k + j) : 0.0f;
  }
  const uint4* src = hidden + static_cast<int64_t>(t) * vec_per_row;
  for (int64_t v0 = threadIdx.x; v0 < vec_per_row; v0 += kThreads * 4) {
    uint4 r[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t v = v0 + i * kThreads;
      if (v < vec_per_row) r[i] = ldg_nc_v4(src + v);
    }
    for (int g = 0; g < G; ++g) {
      const int32_t row = s_row[g];
      if (row >= rows) continue;
      uint4* dst = send_rows + static_cast<int64_t>(row) * vec_per_row;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int64_t v = v0 + i * kThreads;
        if (v < vec_per_row) dst[v] = r[i];
      }
    }
  }
}

// Exclusive scan of the number of valid ids (>= 0) per row:
// slot_row[r] = valid slots in rows < r, slot_row[R] = total.  One CTA of
// 1024 threads; in each pass a thread owns up to kScanRows consecutive rows
// and has all their loads in flight before the block-wide scan of the
// per-thread totals (16384 rows a pass, the running total carried across
// passes).  `vec` says ids rows are 8 int32 on a 16-byte boundary (k = 8),
// read as two 16-byte loads.
constexpr int kScanRows = 16;

__device__ __forceinline__ int valid_ids_in_row(const int32_t* __restrict__ ids, int64_t r, int k,
                                                bool vec) {
  if (vec) {
    const int4 a = __ldg(reinterpret_cast<const int4*>(ids + r * 8));
    const int4 b = __ldg(reinterpret_cast<const int4*>(ids + r * 8) + 1);
    return (a.x >= 0) + (a.y >= 0) + (a.z >= 0) + (a.w >= 0) + (b.x >= 0) + (b.y >= 0) +
           (b.z >= 0) + (b.w >= 0);
  }
  int c = 0;
  for (int j = 0; j < k; ++j) c += __ldg(ids + r * k + j) >= 0;
  return c;
}

__global__ void __launch_bounds__(1024) ep_slot_scan_kernel(const int32_t* __restrict__ ids, int R,
                                                            int k, int vec,
                                                            int32_t* __restrict__ slot_row) {
  __shared__ int s_warp[33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int carry = 0;
  for (int base = 0; base < R; base += 1024 * kScanRows) {
    const int per = min(kScanRows, (R - base + 1023) / 1024);
    const int r0 = base + threadIdx.x * per;
    int cnt[kScanRows];
    int tot = 0;
#pragma unroll
    for (int i = 0; i < kScanRows; ++i) {
      cnt[i] = (i < per && r0 + i < R) ? valid_ids_in_row(ids, r0 + i, k, vec != 0) : 0;
      tot += cnt[i];
    }
    int incl = tot;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += o;
    }
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      const int wv = s_warp[lane];
      int wi = wv;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, wi, off);
        if (lane >= off) wi += o;
      }
      s_warp[lane] = wi - wv;
      if (lane == 31) s_warp[32] = wi;
    }
    __syncthreads();
    int run = carry + s_warp[warp] + incl - tot;
#pragma unroll
    for (int i = 0; i < kScanRows; ++i) {
      if (i < per && r0 + i < R) slot_row[r0 + i] = run;
      run += cnt[i];
    }
    carry += s_warp[32];
    __syncthreads();
  }
  if (threadIdx.x == 0) slot_row[R] = carry;
}

// One CTA per (received row, slot): the slot's weighted expert output,
// rounded once to bf16, goes to combine row slot_row[i] + (valid slots of
// row i before j) - the per-slot product of moe_unpermute_bf16_perslot.
__global__ void __launch_bounds__(kThreads) ep_combine_pack_kernel(
    __nv_bfloat16* __restrict__ comb, const __nv_bfloat16* __restrict__ y,
    const int32_t* __restrict__ s2d, const int32_t* __restrict__ ids, const float* __restrict__ w,
    const int32_t* __restrict__ slot_row, int32_t capacity, int k, int H) {
  const int64_t i = blockIdx.x / k;
  const int j = static_cast<int>(blockIdx.x - i * k);
  const int32_t id = __ldg(ids + i * k + j);
  if (id < 0) return;
  int rank = 0;
  for (int jj = 0; jj < j; ++jj) rank += __ldg(ids + i * k + jj) >= 0;
  const int64_t dst_row = __ldg(slot_row + i) + rank;
  if (dst_row >= capacity) return;
  const float wk = __ldg(w + i * k + j);
  const __nv_bfloat16* src = y + static_cast<int64_t>(__ldg(s2d + i * k + j)) * H;
  __nv_bfloat16* dst = comb + dst_row * H;
  for (int v = threadIdx.x; v < H / 8; v += kThreads) {
    const uint4 raw = ldg_nc_v4(src + v * 8);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
    uint4 out;
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(&out);
#pragma unroll
    for (int q = 0; q < 8; ++q) o[q] = __float2bfloat16_rn(__fmul_rn(wk, __bfloat162float(e[q])));
    *reinterpret_cast<uint4*>(dst + v * 8) = out;
  }
}

// One CTA per (token, slice of H): out[t] = bf16(sum over slots j, in order,
// of the returned combine row of (t, j)), fp32 from 0 - the fixed-order
// reduce of moe_combine_reduce_slots_bf16_to_bf16.  A slot without a valid
// expert adds +0.  Rows at or past comb_count are never read.  K > 0 fixes
// the slot count at compile time, so all K rows' loads are in flight before
// the first add; K = 0 takes it from k.
template <int K>
__global__ void __launch_bounds__(kThreads) ep_combine_reduce_kernel(
    __nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ comb,
    const int32_t* __restrict__ idx, const int32_t* __restrict__ pair_row,
    const int32_t* __restrict__ slot_row, int32_t comb_count, int k_rt, int H, int E, int G,
    int span) {
  const int k = K > 0 ? K : k_rt;
  __shared__ int64_t s_src[32];
  const int t = blockIdx.x;
  const int per = E / G;
  if (threadIdx.x < k) {
    const int j = threadIdx.x;
    const int32_t e = __ldg(idx + static_cast<int64_t>(t) * k + j);
    int64_t src = -1;
    if (e >= 0 && e < E) {
      const int g = e / per;
      int rank = 0;
      for (int jj = 0; jj < j; ++jj) rank += owned_by(__ldg(idx + static_cast<int64_t>(t) * k + jj), E, per, g);
      src = static_cast<int64_t>(__ldg(slot_row + __ldg(pair_row + static_cast<int64_t>(t) * G + g))) + rank;
      if (src >= comb_count) src = -1;  // inconsistent plan: never read past the buffer
    }
    s_src[j] = src;
  }
  __syncthreads();
  const int nvec = H / 8;
  const int v_end = min(nvec, (blockIdx.y + 1) * span);
  for (int v = blockIdx.y * span + threadIdx.x; v < v_end; v += kThreads) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (K > 0) {
      uint4 raw[K > 0 ? K : 1];
#pragma unroll
      for (int j = 0; j < K; ++j)
        raw[j] = s_src[j] >= 0 ? ldg_nc_v4(comb + s_src[j] * H + v * 8) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int j = 0; j < K; ++j) {
        const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw[j]);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] = __fadd_rn(acc[q], __bfloat162float(e[q]));
      }
    }
    for (int j = 0; K == 0 && j < k; ++j) {
      if (s_src[j] < 0) {
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] = __fadd_rn(acc[q], 0.0f);
        continue;
      }
      const uint4 raw = ldg_nc_v4(comb + s_src[j] * H + v * 8);
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] = __fadd_rn(acc[q], __bfloat162float(e[q]));
    }
    uint4 o;
    __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
    for (int q = 0; q < 8; ++q) oe[q] = __float2bfloat16_rn(acc[q]);
    *reinterpret_cast<uint4*>(out + static_cast<int64_t>(t) * H + v * 8) = o;
  }
}

// Row copy that skips destinations at or beyond *n_valid (slots whose expert
// lives on another rank) or beyond the destination's capacity: the
// expert-side permute copies only its own slots.
__global__ void __launch_bounds__(kThreads) copy_valid_rows_kernel(
    const uint4* __restrict__ src, uint4* __restrict__ dst, const int32_t* __restrict__ s2d,
    const int32_t* __restrict__ n_valid, int32_t capacity, int topk, int64_t vec_per_row) {
  __shared__ int32_t s_dest[32];
  const int t = blockIdx.x;
  const int32_t nv = min(__ldg(n_valid), capacity);
  if (threadIdx.x < topk) s_dest[threadIdx.x] = __ldg(s2d + static_cast<int64_t>(t) * topk + threadIdx.x);
  __syncthreads();
  bool any = false;
  for (int j = 0; j < topk; ++j) any |= s_dest[j] < nv;
  if (!any) return;
  const uint4* srow = src + static_cast<int64_t>(t) * vec_per_row;
  // Eight 16-byte loads in flight per thread before the stores.
  for (int64_t v0 = threadIdx.x; v0 < vec_per_row; v0 += 8 * kThreads) {
    uint4 r[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int64_t v = v0 + u * kThreads;
      if (v < vec_per_row) r[u] = ldg_nc_v4(srow + v);
    }
    for (int j = 0; j < topk; ++j) {
      if (s_dest[j] >= nv) continue;
      uint4* drow = dst + static_cast<int64_t>(s_dest[j]) * vec_per_row;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int64_t v = v0 + u * kThreads;
        if (v < vec_per_row) drow[v] = r[u];
      }
    }
  }
}

// ---- peer-memory (NVLink) dispatch -------------------------------------------

__device__ int32_t g_ep_error = 0;

struct PushParams {
  PeerTable peers;
  int world, me;
  int32_t dest_base[kMaxPeers];  // first row of this rank's rows in each destination's recv_rows
  int64_t cap_rows;
  size_t off_rows, off_ids, off_w, off_tok;
  uint32_t* done;
  uint32_t epoch;
};

// One CTA per token (at least one CTA, so an empty rank still publishes):
// the token's row is read once and stored into the recv_rows of every rank
// that owns one of its experts, with the per-slot local ids and weights; the
// ids also go to the local send_ids (the sender's combine needs them).
__global__ void __launch_bounds__(kThreads) ep_dispatch_push_kernel(
    const __grid_constant__ PushParams pp, int32_t* __restrict__ send_ids, int32_t capacity,
    const uint4* __restrict__ hidden, const int32_t* __restrict__ idx, const float* __restrict__ w,
    const int32_t* __restrict__ pair_row, const int32_t* __restrict__ send_off, int T, int k,
    int64_t vec_per_row, int E) {
  __shared__ int32_t s_row[kMaxPeers];   // send row (global index), or -1
  __shared__ int64_t s_dst[kMaxPeers];   // row in the destination's recv_rows
  const int t = blockIdx.x;
  const int G = pp.world;
  if (t < T) {
    const int32_t rows = min(__ldg(send_off + G), capacity);
    const int per = E / G;
    if (threadIdx.x < G) {
      const int g = threadIdx.x;
      const int32_t row = __ldg(pair_row + static_cast<int64_t>(t) * G + g);
      const int64_t dst = pp.dest_base[g] + static_cast<int64_t>(row - __ldg(send_off + g));
      const bool ok = row < rows && dst >= 0 && dst < pp.cap_rows;
      s_row[g] = ok ? row : -1;
      s_dst[g] = dst;
      // The token index travels with the row (the token-chunked combine cuts by it).
      if (ok) reinterpret_cast<int32_t*>(pp.peers.base[g] + pp.off_tok)[dst] = t;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < G * k; i += kThreads) {
      const int g = i / k, j = i - (i / k) * k;
      if (s_row[g] < 0) continue;
      const int32_t e = __ldg(idx + static_cast<int64_t>(t) * k + j);
      const bool mine = owned_by(e, E, per, g);
      const int32_t id = mine ? e - g * per : -1;
      const float wt = mine ? __ldg(w + static_cast<int64_t>(t) * k + j) : 0.0f;
      char* base = pp.peers.base[g];
      reinterpret_cast<int32_t*>(base + pp.off_ids)[s_dst[g] * k + j] = id;
      reinterpret_cast<float*>(base + pp.off_w)[s_dst[g] * k + j] = wt;
      send_ids[static_cast<int64_t>(s_row[g]) * k + j] = id;
    }
    const uint4* src = hidden + static_cast<int64_t>(t) * vec_per_row;
    for (int64_t v0 = threadIdx.x; v0 < vec_per_row; v0 += kThreads * 4) {
      uint4 r[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int64_t v = v0 + i * kThreads;
        if (v < vec_per_row) r[i] = ldg_nc_v4(src + v);
      }
      for (int g = 0; g < G; ++g) {
        if (s_row[g] < 0) continue;
        uint4* dst = reinterpret_cast<uint4*>(pp.peers.base[g] + pp.off_rows) + s_dst[g] * vec_per_row;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int64_t v = v0 + i * kThreads;
          if (v < vec_per_row) dst[v] = r[i];
        }
      }
    }
  }
  grid_release_to_peers(pp.peers, G, pp.me, kCtrlDispatchFlags, pp.done, pp.epoch);
}

// Thread g waits until flags[g] has reached `epoch` (wrap-safe compare), at
// most limit_ns; on expiry it records `code` and returns.
__global__ void ep_wait_kernel(const uint32_t* flags, int G, uint32_t epoch, uint64_t limit_ns,
                               int32_t code) {
  const int g = threadIdx.x;
  if (g >= G) return;
  const uint64_t t0 = global_ns();
  while (static_cast<int32_t>(ld_acquire_sys(flags + g) - epoch) < 0) {
    if (global_ns() - t0 > limit_ns) {
      atomicCAS(&g_ep_error, 0, code);
      return;
    }
    __nanosleep(100);
  }
}

struct RecvSplit {
  int32_t recv_start[kMaxPeers + 1];  // first received row of each source
  int32_t back_base[kMaxPeers];       // first row of this rank's part in each source's back buffer
};

// Per permuted row p (a valid received slot): the source rank, the row of
// its back buffer that receives bf16(w * y[p]), and w.  With kChunks, p is
// also appended to the list of its token chunk, chunk c = (source token of
// the received row) / chunk_tokens capped at chunks - 1: list c is
// order[c * seg ..] and order_count[c] its length (seg = valid slots, so no
// list can overflow).  The appends of one warp take one atomic per chunk
// present in it; the order inside a list is arbitrary (every row has a
// fixed destination, so the push result does not depend on it).
template <bool kChunks>
__global__ void ep_combine_plan_kernel(int32_t* __restrict__ dst_rank, int32_t* __restrict__ dst_row,
                                       float* __restrict__ dst_w, const int32_t* __restrict__ ids,
                                       const float* __restrict__ w, const int32_t* __restrict__ s2d,
                                       const int32_t* __restrict__ slot_row,
                                       const __grid_constant__ RecvSplit sp, int R, int k, int G,
                                       int32_t valid, const int32_t* __restrict__ recv_tok,
                                       int chunk_tokens, int chunks, int32_t* __restrict__ order,
                                       int32_t* __restrict__ order_count) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int r = static_cast<int>(i / k), j = static_cast<int>(i - static_cast<int64_t>(r) * k);
  int32_t p = -1;
  if (i < static_cast<int64_t>(R) * k && __ldg(ids + i) >= 0) {
    p = __ldg(s2d + i);
    if (p >= valid) p = -1;
  }
  if (p >= 0) {
    int src = 0;
    while (src + 1 < G && sp.recv_start[src + 1] <= r) ++src;
    int rank = 0;
    for (int jj = 0; jj < j; ++jj) rank += __ldg(ids + static_cast<int64_t>(r) * k + jj) >= 0;
    dst_rank[p] = src;
    dst_row[p] = sp.back_base[src] + (__ldg(slot_row + r) - __ldg(slot_row + sp.recv_start[src])) + rank;
    dst_w[p] = __ldg(w + i);
  }
  if (kChunks) {
    int c = -1;
    if (p >= 0) {
      const int32_t t = __ldg(recv_tok + r);
      c = t < 0 ? 0 : min(t / chunk_tokens, chunks - 1);
    }
    const unsigned same = __match_any_sync(0xffffffffu, c);
    if (c >= 0) {
      const int lane = threadIdx.x & 31;
      const int leader = __ffs(same) - 1;
      int32_t at = 0;
      if (lane == leader) at = atomicAdd(order_count + c, __popc(same));
      at = __shfl_sync(same, at, leader);
      unsigned below;
      asm("mov.u32 %0, %%lanemask_lt;" : "=r"(below));
      order[static_cast<int64_t>(c) * valid + at + __popc(same & below)] = p;
    }
  }
}

// Row p of y becomes bf16(dst_w[p] * y[p]) at row dst_row[p] of rank
// dst_rank[p]'s combine buffer (a row with an out-of-range plan is skipped).
// One CTA per row; eight 16-byte loads in flight per thread before the
// first store.
__device__ __forceinline__ void push_combine_row(const PeerTable& peers, size_t back_off,
                                                 const __nv_bfloat16* __restrict__ y,
                                                 const int32_t* __restrict__ dst_rank,
                                                 const int32_t* __restrict__ dst_row,
                                                 const float* __restrict__ dst_w, int32_t p,
                                                 int64_t cap_slots, int H, int world) {
  const int nvec = H / 8;
  const int32_t rk = __ldg(dst_rank + p);
  const int32_t dr = __ldg(dst_row + p);
  if (rk < 0 || rk >= world || dr < 0 || dr >= cap_slots) return;
  const float wt = __ldg(dst_w + p);
  const __nv_bfloat16* src = y + static_cast<int64_t>(p) * H;
  __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(peers.base[rk] + back_off) +
                       static_cast<int64_t>(dr) * H;
  for (int v0 = threadIdx.x; v0 < nvec; v0 += 8 * kThreads) {
    uint4 raw[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int v = v0 + u * kThreads;
      if (v < nvec) raw[u] = ldg_nc_v4(src + v * 8);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int v = v0 + u * kThreads;
      if (v >= nvec) break;
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw[u]);
      uint4 out;
      __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(&out);
#pragma unroll
      for (int q = 0; q < 8; ++q) o[q] = __float2bfloat16_rn(__fmul_rn(wt, __bfloat162float(e[q])));
      *reinterpret_cast<uint4*>(dst + v * 8) = out;
    }
  }
}

// The combine without a GEMM in front (expert outputs already in memory):
// push_combine_row for the rows p0 .. p1-1, or with `order` for the rows of
// chunk `chunk`'s list that lie in [p0, p1); then, if `publish`, the last CTA
// publishes the epoch at flag_offset.
__global__ void __launch_bounds__(kThreads) ep_combine_push_kernel(
    const __grid_constant__ PeerTable peers, size_t back_off, const __nv_bfloat16* __restrict__ y,
    const int32_t* __restrict__ dst_rank, const int32_t* __restrict__ dst_row,
    const float* __restrict__ dst_w, int32_t rows, const int32_t* __restrict__ row_lo,
    const int32_t* __restrict__ row_hi, int publish, int64_t cap_slots, int H, int world, int me,
    uint32_t* done, uint32_t epoch, const int32_t* __restrict__ order,
    const int32_t* __restrict__ order_count, int64_t order_stride, int chunk, size_t flag_offset) {
  const int32_t p0 = row_lo ? max(__ldg(row_lo), 0) : 0;
  const int32_t p1 = row_hi ? min(__ldg(row_hi), rows) : rows;
  if (order != nullptr) {
    // A chunk list holds its rows in received-row order, grouped by source
    // rank, so walking it in order would send every CTA's stores to one rank
    // at a time (on every rank at once).  The walk interleaves `world` equal
    // segments instead: v -> (v % world) * seg + v / world is a bijection of
    // [0, world * seg), and the images past the list's end are skipped.
    order += chunk * order_stride;
    const int64_t listed = __ldg(order_count + chunk);
    const int64_t n = listed < order_stride ? listed : order_stride;
    const int64_t seg = (n + world - 1) / world;
    for (int64_t v = blockIdx.x; v < seg * world; v += gridDim.x) {
      const int64_t d = (v % world) * seg + v / world;
      if (d >= n) continue;
      const int32_t p = __ldg(order + d);
      if (p < p0 || p >= p1) continue;
      push_combine_row(peers, back_off, y, dst_rank, dst_row, dst_w, p, cap_slots, H, world);
    }
  } else {
    for (int32_t p = p0 + blockIdx.x; p < p1; p += gridDim.x)
      push_combine_row(peers, back_off, y, dst_rank, dst_row, dst_w, p, cap_slots, H, world);
  }
  if (publish) grid_release_to_peers(peers, world, me, flag_offset, done, epoch);
  else __threadfence_system();  // ordered before the publishing call that follows on the stream
}

}  // namespace

lsek_status ep_take_device_error(int32_t* code) {
  int32_t zero = 0;
  LSEK_CUDA_TRY(cudaMemcpyFromSymbol(code, g_ep_error, sizeof(int32_t)));
  LSEK_CUDA_TRY(cudaMemcpyToSymbol(g_ep_error, &zero, sizeof(int32_t)));
  return LSEK_OK;
}

}  // namespace lsek

using namespace lsek;

static lsek_status ep_check(int T, int k, int E, int G, const char* name) {
  LSEK_REQUIRE(T >= 0 && k >= 1 && k <= 32, "%s: need T >= 0 and 1 <= topk <= 32", name);
  LSEK_REQUIRE(G >= 1 && G <= 64, "%s: world size must be in [1, 64]", name);
  LSEK_REQUIRE(E >= G && E % G == 0, "%s: num_experts must be a multiple of the world size", name);
  return LSEK_OK;
}

extern "C" size_t lsek_ep_plan_workspace_size(int32_t num_tokens, int32_t world_size) {
  if (num_tokens < 0 || world_size < 1) return 0;
  const int64_t n = static_cast<int64_t>(num_tokens) * world_size;
  return static_cast<size_t>(((n * 4 + 255) / 256) * 256) + permute_workspace_bytes(n, world_size);
}

extern "C" lsek_status lsek_ep_plan(int32_t* send_off, int32_t* send_counts, int32_t* pair_row,
                                    int32_t* row_pair, const int32_t* topk_indices,
                                    int32_t num_tokens, int32_t topk, int32_t num_experts,
                                    int32_t world_size, void* workspace, size_t workspace_bytes,
                                    void* stream) {
  lsek_status s = ep_check(num_tokens, topk, num_experts, world_size, "ep_plan");
  if (s != LSEK_OK) return s;
  LSEK_REQUIRE(send_off && send_counts, "ep_plan: NULL tensor pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t n = static_cast<int64_t>(num_tokens) * world_size;
  LSEK_CUDA_TRY(cudaMemsetAsync(send_counts, 0, sizeof(int32_t) * 2 * world_size, st));
  if (n == 0) {
    LSEK_CUDA_TRY(cudaMemsetAsync(send_off, 0, sizeof(int32_t) * (world_size + 1), st));
    return LSEK_OK;
  }
  const size_t need = lsek_ep_plan_workspace_size(num_tokens, world_size);
  LSEK_REQUIRE(workspace != nullptr && workspace_bytes >= need,
               "ep_plan: workspace of %zu bytes required, got %zu", need, workspace_bytes);
  LSEK_REQUIRE(pair_row && row_pair && topk_indices, "ep_plan: NULL tensor pointer");
  int32_t* keys = static_cast<int32_t*>(workspace);
  char* route_ws = static_cast<char*>(workspace) + ((n * 4 + 255) / 256) * 256;
  ep_pair_keys_kernel<<<static_cast<unsigned>(ceil_div(n, 256)), 256, 0, st>>>(
      topk_indices, num_tokens, topk, num_experts, world_size, keys, send_counts);
  if ((s = check_launch("ep_plan")) != LSEK_OK) return s;
  s = launch_route(keys, n, world_size, send_off, pair_row, row_pair, route_ws, st);
  if (s != LSEK_OK) return s;
  ep_row_counts_kernel<<<1, 64, 0, st>>>(send_off, world_size, send_counts);
  return check_launch("ep_plan");
}

extern "C" lsek_status lsek_ep_dispatch_pack(void* send_rows, int32_t* send_ids, float* send_w,
                                             int32_t send_capacity, const void* hidden,
                                             const int32_t* topk_indices,
                                             const float* topk_weights, const int32_t* pair_row,
                                             const int32_t* send_off, int32_t num_tokens,
                                             int32_t topk, int32_t hidden_dim, int32_t num_experts,
                                             int32_t world_size, void* stream) {
  lsek_status s = ep_check(num_tokens, topk, num_experts, world_size, "ep_dispatch_pack");
  if (s != LSEK_OK) return s;
  LSEK_REQUIRE(hidden_dim > 0 && hidden_dim % 8 == 0, "ep_dispatch_pack: hidden_dim must be a multiple of 8");
  LSEK_REQUIRE(send_capacity >= 0, "ep_dispatch_pack: send_capacity must be >= 0");
  if (num_tokens == 0 || send_capacity == 0) return LSEK_OK;
  LSEK_REQUIRE(send_rows && send_ids && send_w && hidden && topk_indices && topk_weights && pair_row &&
                   send_off,
               "ep_dispatch_pack: NULL tensor pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  ep_dispatch_pack_kernel<<<num_tokens, kThreads, 0, st>>>(
      static_cast<uint4*>(send_rows), send_ids, send_w, static_cast<const uint4*>(hidden),
      topk_indices, topk_weights, pair_row, send_off, send_capacity, topk, hidden_dim / 8,
      num_experts, world_size);
  return check_launch("ep_dispatch_pack");
}

extern "C" lsek_status lsek_ep_slot_scan(int32_t* slot_row, const int32_t* ids, int32_t rows,
                                         int32_t topk, void* stream) {
  LSEK_REQUIRE(rows >= 0 && topk >= 1 && topk <= 32, "ep_slot_scan: bad sizes");
  LSEK_REQUIRE(slot_row != nullptr && (rows == 0 || ids != nullptr), "ep_slot_scan: NULL pointer");
  const int vec = topk == 8 && reinterpret_cast<uintptr_t>(ids) % 16 == 0;
  ep_slot_scan_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(ids, rows, topk, vec,
                                                                         slot_row);
  return check_launch("ep_slot_scan");
}

extern "C" lsek_status lsek_ep_expert_permute(void* permuted, int32_t permuted_rows,
                                              int32_t* expert_offsets, int32_t* s2d,
                                              int32_t* perm, const void* rows_in,
                                              const int32_t* local_ids, int32_t rows, int32_t topk,
                                              int32_t hidden_dim, int32_t local_experts,
                                              void* workspace, size_t workspace_bytes,
                                              void* stream) {
  LSEK_REQUIRE(rows >= 0 && topk >= 1 && topk <= 32 && hidden_dim > 0 && hidden_dim % 8 == 0 &&
                   permuted_rows >= 0,
               "ep_expert_permute: bad sizes");
  LSEK_REQUIRE(local_experts >= 1 && local_experts <= 1023, "ep_expert_permute: local experts in [1, 1023]");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t n = static_cast<int64_t>(rows) * topk;
  if (n == 0) {
    LSEK_CUDA_TRY(cudaMemsetAsync(expert_offsets, 0, sizeof(int32_t) * (local_experts + 1), st));
    return LSEK_OK;
  }
  const size_t need = permute_workspace_bytes(n, local_experts);
  LSEK_REQUIRE(n <= 4096 || (workspace != nullptr && workspace_bytes >= need),
               "ep_expert_permute: workspace of %zu bytes required", need);
  LSEK_REQUIRE(rows_in && local_ids && expert_offsets && s2d && perm &&
                   (permuted_rows == 0 || permuted),
               "ep_expert_permute: NULL pointer");
  lsek_status s = launch_route(local_ids, n, local_experts, expert_offsets, s2d, perm, workspace, st);
  if (s != LSEK_OK) return s;
  if (permuted_rows == 0) return LSEK_OK;
  copy_valid_rows_kernel<<<rows, kThreads, 0, st>>>(static_cast<const uint4*>(rows_in),
                                                    static_cast<uint4*>(permuted), s2d,
                                                    expert_offsets + local_experts, permuted_rows,
                                                    topk, hidden_dim / 8);
  return check_launch("ep_expert_permute");
}

extern "C" lsek_status lsek_ep_combine_pack(void* comb_rows, int32_t comb_capacity,
                                            const void* expert_out, const int32_t* s2d,
                                            const int32_t* ids, const float* w,
                                            const int32_t* slot_row, int32_t rows, int32_t topk,
                                            int32_t hidden_dim, void* stream) {
  LSEK_REQUIRE(rows >= 0 && topk >= 1 && topk <= 32 && hidden_dim > 0 && hidden_dim % 8 == 0 &&
                   comb_capacity >= 0,
               "ep_combine_pack: bad sizes");
  if (rows == 0 || comb_capacity == 0) return LSEK_OK;
  LSEK_REQUIRE(comb_rows && expert_out && s2d && ids && w && slot_row, "ep_combine_pack: NULL pointer");
  const int64_t blocks = static_cast<int64_t>(rows) * topk;
  ep_combine_pack_kernel<<<static_cast<unsigned>(blocks), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<__nv_bfloat16*>(comb_rows), static_cast<const __nv_bfloat16*>(expert_out), s2d, ids,
      w, slot_row, comb_capacity, topk, hidden_dim);
  return check_launch("ep_combine_pack");
}

extern "C" lsek_status lsek_ep_combine_reduce(void* out, const void* comb_rows,
                                              int32_t comb_count, const int32_t* topk_indices,
                                              const int32_t* pair_row,
                                              const int32_t* slot_row, int32_t num_tokens,
                                              int32_t topk, int32_t hidden_dim,
                                              int32_t num_experts, int32_t world_size,
                                              void* stream) {
  lsek_status s = ep_check(num_tokens, topk, num_experts, world_size, "ep_combine_reduce");
  if (s != LSEK_OK) return s;
  LSEK_REQUIRE(hidden_dim > 0 && hidden_dim % 8 == 0, "ep_combine_reduce: hidden_dim must be a multiple of 8");
  LSEK_REQUIRE(comb_count >= 0, "ep_combine_reduce: comb_count must be >= 0");
  if (num_tokens == 0) return LSEK_OK;
  LSEK_REQUIRE(out && (comb_rows || comb_count == 0) && topk_indices && pair_row && slot_row,
               "ep_combine_reduce: NULL pointer");
  const int nvec = hidden_dim / 8;
  const int64_t want = 4ll * num_sms();
  int slices = num_tokens >= want ? 1 : static_cast<int>(ceil_div(want, num_tokens));
  const int max_slices = static_cast<int>(ceil_div(nvec, kThreads));
  if (slices > max_slices) slices = max_slices;
  const int span = static_cast<int>(ceil_div(nvec, slices));
  const dim3 grid(num_tokens, static_cast<unsigned>(ceil_div(nvec, span)));
  auto kernel = topk == 8 ? ep_combine_reduce_kernel<8> : ep_combine_reduce_kernel<0>;
  kernel<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<__nv_bfloat16*>(out), static_cast<const __nv_bfloat16*>(comb_rows), topk_indices,
      pair_row, slot_row, comb_count, topk, hidden_dim, num_experts, world_size, span);
  return check_launch("ep_combine_reduce");
}

// ---- peer domain -----------------------------------------------------------------

static lsek_status domain_check(const lsek_ep_domain* h, const char* name) {
  LSEK_REQUIRE(h != nullptr, "%s: domain is NULL", name);
  for (int g = 0; g < h->d.world; ++g)
    LSEK_REQUIRE(h->d.peer[g] != nullptr, "%s: rank %d of the domain has not been imported", name, g);
  int dev = -1;
  LSEK_CUDA_TRY(cudaGetDevice(&dev));
  LSEK_REQUIRE(dev == h->d.device, "%s: the domain lives on device %d, current device is %d", name,
               h->d.device, dev);
  return LSEK_OK;
}

// counts [G][G][2]: row s = (rows, slots) source s sends to each rank.
static int64_t col_sum(const int32_t* counts, int G, int upto_s, int g, int c) {
  int64_t v = 0;
  for (int s = 0; s < upto_s; ++s) v += counts[(static_cast<int64_t>(s) * G + g) * 2 + c];
  return v;
}

extern "C" size_t lsek_ep_domain_bytes(int32_t max_tokens, int32_t hidden_dim, int32_t topk,
                                       int32_t world_size) {
  if (max_tokens < 0 || hidden_dim <= 0 || topk <= 0 || world_size <= 0) return 0;
  return ep_layout(max_tokens, hidden_dim, topk, world_size).total;
}

extern "C" lsek_status lsek_ep_domain_create(lsek_ep_domain** out, int32_t rank, int32_t world_size,
                                             int32_t max_tokens, int32_t hidden_dim, int32_t topk) {
  LSEK_REQUIRE(out != nullptr, "ep_domain_create: out is NULL");
  *out = nullptr;
  LSEK_REQUIRE(world_size >= 1 && world_size <= kMaxPeers,
               "ep_domain_create: world size must be in [1, %d]", kMaxPeers);
  LSEK_REQUIRE(rank >= 0 && rank < world_size, "ep_domain_create: rank out of range");
  LSEK_REQUIRE(max_tokens >= 1 && hidden_dim > 0 && hidden_dim % 8 == 0 && topk >= 1 && topk <= 32,
               "ep_domain_create: bad sizes");
  auto* h = new lsek_ep_domain();
  EpDomain& d = h->d;
  d.rank = rank;
  d.world = world_size;
  d.max_tokens = max_tokens;
  d.H = hidden_dim;
  d.k = topk;
  d.lay = ep_layout(max_tokens, hidden_dim, topk, world_size);
  d.local = nullptr;
  for (int g = 0; g < kMaxPeers; ++g) {
    d.peer[g] = nullptr;
    d.imported[g] = false;
  }
  cudaError_t e = cudaGetDevice(&d.device);
  if (e == cudaSuccess) e = cudaMalloc(&d.local, d.lay.total);
  if (e == cudaSuccess) e = cudaMemset(d.local, 0, d.lay.total);
  if (e != cudaSuccess) {
    if (d.local) cudaFree(d.local);
    delete h;
    return fail(LSEK_ERR_CUDA, "ep_domain_create: %s", cudaGetErrorString(e));
  }
  d.peer[rank] = d.local;
  *out = h;
  return LSEK_OK;
}

extern "C" lsek_status lsek_ep_domain_export(const lsek_ep_domain* h, void* handle,
                                             size_t handle_bytes) {
  LSEK_REQUIRE(h != nullptr && handle != nullptr, "ep_domain_export: NULL argument");
  LSEK_REQUIRE(handle_bytes >= sizeof(cudaIpcMemHandle_t),
               "ep_domain_export: handle buffer needs %zu bytes", sizeof(cudaIpcMemHandle_t));
  cudaIpcMemHandle_t ipc;
  LSEK_CUDA_TRY(cudaIpcGetMemHandle(&ipc, h->d.local));
  std::memcpy(handle, &ipc, sizeof(ipc));
  return LSEK_OK;
}

extern "C" lsek_status lsek_ep_domain_import(lsek_ep_domain* h, int32_t peer, const void* handle,
                                             size_t handle_bytes) {
  LSEK_REQUIRE(h != nullptr && handle != nullptr, "ep_domain_import: NULL argument");
  EpDomain& d = h->d;
  LSEK_REQUIRE(peer >= 0 && peer < d.world, "ep_domain_import: peer out of range");
  LSEK_REQUIRE(handle_bytes >= sizeof(cudaIpcMemHandle_t), "ep_domain_import: short handle");
  if (peer == d.rank) return LSEK_OK;
  LSEK_REQUIRE(d.peer[peer] == nullptr, "ep_domain_import: rank %d already imported", peer);
  cudaIpcMemHandle_t ipc;
  std::memcpy(&ipc, handle, sizeof(ipc));
  void* ptr = nullptr;
  LSEK_CUDA_TRY(cudaIpcOpenMemHandle(&ptr, ipc, cudaIpcMemLazyEnablePeerAccess));
  d.peer[peer] = static_cast<char*>(ptr);
  d.imported[peer] = true;
  return LSEK_OK;
}

extern "C" lsek_status lsek_ep_domain_buffers(const lsek_ep_domain* h, void** recv_rows,
                                              int32_t** recv_ids, float** recv_w, void** back,
                                              int64_t* cap_rows, int64_t* cap_slots) {
  LSEK_REQUIRE(h != nullptr, "ep_domain_buffers: domain is NULL");
  const EpDomain& d = h->d;
  if (recv_rows) *recv_rows = d.local + d.lay.recv_rows;
  if (recv_ids) *recv_ids = reinterpret_cast<int32_t*>(d.local + d.lay.recv_ids);
  if (recv_w) *recv_w = reinterpret_cast<float*>(d.local + d.lay.recv_w);
  if (back) *back = d.local + d.lay.back;
  if (cap_rows) *cap_rows = d.lay.cap_rows;
  if (cap_slots) *cap_slots = d.lay.cap_slots;
  return LSEK_OK;
}

extern "C" void lsek_ep_domain_destroy(lsek_ep_domain* h) {
  if (h == nullptr) return;
  EpDomain& d = h->d;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(d.device);
  cudaDeviceSynchronize();
  for (int g = 0; g < d.world; ++g)
    if (d.imported[g] && d.peer[g]) cudaIpcCloseMemHandle(d.peer[g]);
  if (d.local) cudaFree(d.local);
  if (prev >= 0) cudaSetDevice(prev);
  delete h;
}

extern "C" lsek_status lsek_ep_dispatch_push(lsek_ep_domain* h, int32_t* send_ids,
                                             int32_t send_capacity, const int32_t* counts,
                                             const void* hidden, const int32_t* topk_indices,
                                             const float* topk_weights, const int32_t* pair_row,
                                             const int32_t* send_off, int32_t num_tokens,
                                             int32_t num_experts, uint32_t epoch, void* stream) {
  lsek_status s = domain_check(h, "ep_dispatch_push");
  if (s != LSEK_OK) return s;
  const EpDomain& d = h->d;
  const int G = d.world;
  s = ep_check(num_tokens, static_cast<int>(d.k), num_experts, G, "ep_dispatch_push");
  if (s != LSEK_OK) return s;
  LSEK_REQUIRE(num_tokens <= d.max_tokens, "ep_dispatch_push: %d tokens exceed the domain's %lld",
               num_tokens, static_cast<long long>(d.max_tokens));
  LSEK_REQUIRE(counts != nullptr && send_capacity >= 0, "ep_dispatch_push: bad counts / capacity");
  LSEK_REQUIRE(num_tokens == 0 || (hidden && topk_indices && topk_weights && pair_row && send_off &&
                                   (send_capacity == 0 || send_ids)),
               "ep_dispatch_push: NULL tensor pointer");
  PushParams pp;
  pp.peers = peer_table(d);
  pp.world = G;
  pp.me = d.rank;
  for (int g = 0; g < kMaxPeers; ++g) pp.dest_base[g] = 0;
  for (int g = 0; g < G; ++g) {
    const int64_t base = col_sum(counts, G, d.rank, g, 0);
    const int64_t total = col_sum(counts, G, G, g, 0);
    LSEK_REQUIRE(total <= d.lay.cap_rows, "ep_dispatch_push: rank %d would receive %lld rows (capacity %lld)",
                 g, static_cast<long long>(total), static_cast<long long>(d.lay.cap_rows));
    pp.dest_base[g] = static_cast<int32_t>(base);
  }
  pp.cap_rows = d.lay.cap_rows;
  pp.off_rows = d.lay.recv_rows;
  pp.off_ids = d.lay.recv_ids;
  pp.off_w = d.lay.recv_w;
  pp.off_tok = d.lay.recv_tok;
  pp.done = reinterpret_cast<uint32_t*>(d.local + kCtrlPushDone);
  pp.epoch = epoch;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  LSEK_CUDA_TRY(cudaMemsetAsync(pp.done, 0, sizeof(uint32_t), st));
  ep_dispatch_push_kernel<<<num_tokens > 0 ? num_tokens : 1, kThreads, 0, st>>>(
      pp, send_ids, send_capacity, static_cast<const uint4*>(hidden), topk_indices, topk_weights,
      pair_row, send_off, num_tokens, static_cast<int>(d.k), d.H / 8, num_experts);
  return check_launch("ep_dispatch_push");
}

namespace lsek {
namespace {
__global__ void copy_words_kernel(uint32_t* __restrict__ dst, const uint32_t* __restrict__ src,
                                  int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = src[i];
}
}  // namespace
}  // namespace lsek

extern "C" lsek_status lsek_copy_to_mapped_host(void* host_dst, const void* dev_src, size_t bytes,
                                                void* stream) {
  LSEK_REQUIRE(bytes % 4 == 0, "copy_to_mapped_host: bytes must be a multiple of 4");
  if (bytes == 0) return LSEK_OK;
  LSEK_REQUIRE(host_dst && dev_src, "copy_to_mapped_host: NULL pointer");
  LSEK_REQUIRE(reinterpret_cast<uintptr_t>(host_dst) % 4 == 0 &&
                   reinterpret_cast<uintptr_t>(dev_src) % 4 == 0,
               "copy_to_mapped_host: pointers must be 4-byte aligned");
  void* mapped = nullptr;
  if (cudaHostGetDevicePointer(&mapped, host_dst, 0) != cudaSuccess || mapped == nullptr) {
    cudaGetLastError();  // the failed query leaves a (non-sticky) error behind: clear it
    return fail(LSEK_ERR_INVALID_ARG, "copy_to_mapped_host: destination is not page-locked host memory");
  }
  const int64_t n = static_cast<int64_t>(bytes / 4);
  const unsigned grid = static_cast<unsigned>(n < 256 * 64 ? ceil_div(n, 256) : 64);
  copy_words_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint32_t*>(mapped), static_cast<const uint32_t*>(dev_src), n);
  return check_launch("copy_to_mapped_host");
}

extern "C" lsek_status lsek_ep_wait(lsek_ep_domain* h, int32_t what, uint32_t epoch,
                                    int64_t timeout_ns, void* stream) {
  lsek_status s = domain_check(h, "ep_wait");
  if (s != LSEK_OK) return s;
  LSEK_REQUIRE(what >= 0 && what < 2 + kMaxCombineChunks,
               "ep_wait: what must be 0 (dispatch), 1 (combine) or 2 + c (combine chunk c < %d)",
               kMaxCombineChunks);
  const EpDomain& d = h->d;
  const size_t off = what == 0   ? kCtrlDispatchFlags
                     : what == 1 ? kCtrlCombineFlags
                                 : kCtrlChunkFlags + 256 * static_cast<size_t>(what - 2);
  const uint32_t* flags = reinterpret_cast<const uint32_t*>(d.local + off);
  const uint64_t limit = timeout_ns > 0 ? static_cast<uint64_t>(timeout_ns) : kWaitLimitNs;
  ep_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      flags, d.world, epoch, limit, what == 0 ? kDevErrEpDispatchWait : kDevErrEpCombineWait);
  return check_launch("ep_wait");
}

static lsek_status combine_plan(lsek_ep_domain* h, int32_t* dst_rank, int32_t* dst_row,
                                float* dst_w, const int32_t* src_to_dest_map,
                                const int32_t* slot_row, const int32_t* counts, int32_t recv_rows,
                                int32_t valid_slots, int32_t chunk_tokens, int32_t chunks,
                                int32_t* order, int32_t* order_count, void* stream,
                                const char* name) {
  lsek_status s = domain_check(h, name);
  if (s != LSEK_OK) return s;
  const EpDomain& d = h->d;
  const int G = d.world;
  LSEK_REQUIRE(counts != nullptr, "%s: counts is NULL", name);
  LSEK_REQUIRE(recv_rows >= 0 && recv_rows <= d.lay.cap_rows && valid_slots >= 0,
               "%s: bad sizes", name);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (chunks > 0) {
    LSEK_REQUIRE(chunk_tokens >= 1, "%s: chunk_tokens must be >= 1", name);
    LSEK_REQUIRE(chunks <= kMaxCombineChunks, "%s: chunks must be in [1, %d]", name,
                 kMaxCombineChunks);
    LSEK_REQUIRE(order_count != nullptr, "%s: order_count is NULL", name);
    LSEK_CUDA_TRY(cudaMemsetAsync(order_count, 0, sizeof(int32_t) * chunks, st));
  }
  RecvSplit sp;
  for (int g = 0; g <= kMaxPeers; ++g) sp.recv_start[g] = 0;
  for (int g = 0; g < kMaxPeers; ++g) sp.back_base[g] = 0;
  for (int src = 0; src <= G; ++src) sp.recv_start[src] = static_cast<int32_t>(col_sum(counts, G, src, d.rank, 0));
  LSEK_REQUIRE(sp.recv_start[G] == recv_rows, "%s: recv_rows disagrees with counts", name);
  for (int src = 0; src < G; ++src) {
    int64_t b = 0;
    for (int g = 0; g < d.rank; ++g) b += counts[(static_cast<int64_t>(src) * G + g) * 2 + 1];
    sp.back_base[src] = static_cast<int32_t>(b);
  }
  const int64_t n = static_cast<int64_t>(recv_rows) * d.k;
  if (n == 0 || valid_slots == 0) return LSEK_OK;
  LSEK_REQUIRE(dst_rank && dst_row && dst_w && src_to_dest_map && slot_row,
               "%s: NULL tensor pointer", name);
  LSEK_REQUIRE(chunks == 0 || order != nullptr, "%s: order is NULL", name);
  auto kernel = chunks > 0 ? ep_combine_plan_kernel<true> : ep_combine_plan_kernel<false>;
  kernel<<<static_cast<unsigned>(ceil_div(n, 256)), 256, 0, st>>>(
      dst_rank, dst_row, dst_w, reinterpret_cast<const int32_t*>(d.local + d.lay.recv_ids),
      reinterpret_cast<const float*>(d.local + d.lay.recv_w), src_to_dest_map, slot_row, sp,
      recv_rows, static_cast<int>(d.k), G, valid_slots,
      reinterpret_cast<const int32_t*>(d.local + d.lay.recv_tok), chunk_tokens, chunks, order,
      order_count);
  return check_launch(name);
}

extern "C" lsek_status lsek_ep_combine_plan(lsek_ep_domain* h, int32_t* dst_rank, int32_t* dst_row,
                                            float* dst_w, const int32_t* src_to_dest_map,
                                            const int32_t* slot_row, const int32_t* counts,
                                            int32_t recv_rows, int32_t valid_slots, void* stream) {
  return combine_plan(h, dst_rank, dst_row, dst_w, src_to_dest_map, slot_row, counts, recv_rows,
                      valid_slots, 0, 0, nullptr, nullptr, stream, "ep_combine_plan");
}

extern "C" lsek_status lsek_ep_combine_plan_chunks(lsek_ep_domain* h, int32_t* dst_rank,
                                                   int32_t* dst_row, float* dst_w, int32_t* order,
                                                   int32_t* order_count,
                                                   const int32_t* src_to_dest_map,
                                                   const int32_t* slot_row, const int32_t* counts,
                                                   int32_t recv_rows, int32_t valid_slots,
                                                   int32_t chunk_tokens, int32_t chunks,
                                                   void* stream) {
  if (chunks < 1) return fail(LSEK_ERR_INVALID_ARG, "ep_combine_plan_chunks: chunks must be >= 1");
  return combine_plan(h, dst_rank, dst_row, dst_w, src_to_dest_map, slot_row, counts, recv_rows,
                      valid_slots, chunk_tokens, chunks, order, order_count, stream,
                      "ep_combine_plan_chunks");
}

extern "C" lsek_status lsek_ep_combine_push(lsek_ep_domain* h, const void* expert_out,
                                            const int32_t* dst_rank, const int32_t* dst_row,
                                            const float* dst_w, int32_t rows,
                                            const int32_t* row_lo, const int32_t* row_hi,
                                            int32_t publish, uint32_t epoch, void* stream) {
  lsek_status s = domain_check(h, "ep_combine_push");
  if (s != LSEK_OK) return s;
  const EpDomain& d = h->d;
  LSEK_REQUIRE(rows >= 0, "ep_combine_push: bad row count");
  LSEK_REQUIRE(rows == 0 || (expert_out && dst_rank && dst_row && dst_w),
               "ep_combine_push: NULL tensor pointer");
  LSEK_REQUIRE((row_lo == nullptr) == (row_hi == nullptr), "ep_combine_push: give both row bounds or none");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint32_t* done = reinterpret_cast<uint32_t*>(d.local + kCtrlGemmDone);
  if (publish) LSEK_CUDA_TRY(cudaMemsetAsync(done, 0, sizeof(uint32_t), st));
  const int64_t want = 4ll * num_sms();
  const unsigned grid = static_cast<unsigned>(rows == 0 ? 1 : (rows < want ? rows : want));
  ep_combine_push_kernel<<<grid, kThreads, 0, st>>>(
      peer_table(d), d.lay.back, static_cast<const __nv_bfloat16*>(expert_out), dst_rank, dst_row,
      dst_w, rows, row_lo, row_hi, publish, d.lay.cap_slots, static_cast<int>(d.H), d.world, d.rank,
      done, epoch, nullptr, nullptr, 0, 0, kCtrlCombineFlags);
  return check_launch("ep_combine_push");
}

extern "C" lsek_status lsek_ep_combine_push_chunk(lsek_ep_domain* h, const void* expert_out,
                                                  const int32_t* dst_rank, const int32_t* dst_row,
                                                  const float* dst_w, int32_t rows,
                                                  const int32_t* row_lo, const int32_t* row_hi,
                                                  const int32_t* order, const int32_t* order_count,
                                                  int32_t chunk, uint32_t epoch, void* stream) {
  lsek_status s = domain_check(h, "ep_combine_push_chunk");
  if (s != LSEK_OK) return s;
  const EpDomain& d = h->d;
  LSEK_REQUIRE(rows >= 0, "ep_combine_push_chunk: bad row count");
  LSEK_REQUIRE(chunk >= 0 && chunk < kMaxCombineChunks,
               "ep_combine_push_chunk: chunk must be in [0, %d)", kMaxCombineChunks);
  LSEK_REQUIRE(rows == 0 || (expert_out && dst_rank && dst_row && dst_w && order && order_count),
               "ep_combine_push_chunk: NULL tensor pointer");
  LSEK_REQUIRE((row_lo == nullptr) == (row_hi == nullptr),
               "ep_combine_push_chunk: give both row bounds or none");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint32_t* done = reinterpret_cast<uint32_t*>(d.local + kCtrlChunkDone) + chunk;
  LSEK_CUDA_TRY(cudaMemsetAsync(done, 0, sizeof(uint32_t), st));
  const int64_t want = 4ll * num_sms();
  const unsigned grid = static_cast<unsigned>(rows == 0 ? 1 : (rows < want ? rows : want));
  ep_combine_push_kernel<<<grid, kThreads, 0, st>>>(
      peer_table(d), d.lay.back, static_cast<const __nv_bfloat16*>(expert_out), dst_rank, dst_row,
      dst_w, rows, row_lo, row_hi, 1, d.lay.cap_slots, static_cast<int>(d.H), d.world, d.rank,
      done, epoch, rows == 0 ? nullptr : order, order_count, static_cast<int64_t>(rows), chunk,
      kCtrlChunkFlags + 256 * static_cast<size_t>(chunk));
  return check_launch("ep_combine_push_chunk");
}
