// Permute / unpermute family for sm_100a.
//
// Permute is a stable counting sort of the T*topk slot ids by expert, with no
// radix sort library.  "Routing" (offsets and the two maps) is integer work
// on T*topk keys; the row copy is the HBM-bound part.
//
//   route   Keys are split into contiguous per-warp runs.  For each 32-key
//           step a warp finds the lanes holding an equal key with one ballot
//           per key bit (the keys need at most 11 bits): a key's rank inside
//           the step is popc(peers & lanes-below), and the lowest peer lane
//           adds popc(peers) to the warp's running count for that expert.
//           Pass 1 counts, a scan over (expert, chunk, warp) turns counts into
//           start positions, pass 2 repeats the walk and writes
//           dest = start + rank.  Every position is fixed by the key order,
//           so the result is the stable order of torch.argsort(stable=True)
//           (tests/test_reference.py:534-558), which is the order the
//           reference's CUB radix sort produces (smxx/permute/moe_permute.cu:553-563).
//           Up to kSingleMaxKeys keys run as one 1024-thread CTA
//           (route_single); larger inputs use route_count -> route_scan ->
//           route_rank over chunks of kChunkKeys keys.
//   copy    One CTA per (token, slice of the row): each thread loads its
//           16-byte vectors of the token's row once and stores them to the
//           token's topk destination rows, so `hidden` is read once
//           (the reference reads it once per destination row,
//           moe_permute.cu:98-137).
//
// Unpermute kernels gather the topk rows of a token with 16-byte loads, all
// issued before the arithmetic so they are in flight together, and follow
// the reference's arithmetic exactly:
//   sum       acc = fma(w_k, x_k, acc) for k = 0..topk-1 from acc = 0
//             (finalize_moe_routing_bf16, moe_permute.cu:182-246, whose
//             `accum += w * x` nvcc contracts to this fma)
//   perslot   out[t,k] = w_k * x_k in fp32, or rounded once to 16 bits
//             (moe_permute.cu:330-434)
//   reduce    out[t] = bf16(((0 + in_0) + in_1) + ...) in fp32
//             (moe_permute.cu:440-474)
#include <mutex>

#include "common.cuh"

namespace lsek {
namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kRouteThreads = 1024;
constexpr int kRouteWarps = kRouteThreads / 32;
constexpr int kSingleMaxKeys = 4096;            // one CTA, up to 4 keys per lane
constexpr int kChunkKeyPerLane = 2;             // multi-CTA: 2 keys per lane
constexpr int kChunkKeys = kRouteWarps * 32 * kChunkKeyPerLane;  // 2048

__device__ __forceinline__ int clamp_key(int32_t v, int E) {
  return (v < 0 || v >= E) ? E : v;
}

__device__ __forceinline__ unsigned lanemask_lt() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Bits needed for every key value 0..E plus the padding key (all ones).
__host__ __device__ __forceinline__ int key_bits(int E) {
  int b = 1;
  while ((1 << b) - 1 <= E) ++b;
  return b;
}

// Loads this warp's run of keys: lane l holds keys at run_begin + i*32 + l;
// positions past the run hold the padding key (1 << nbits) - 1.
template <int KPL>
__device__ __forceinline__ void load_keys(int (&key)[KPL], const int32_t* __restrict__ idx,
                                          int run_begin, int run_end, int lane, int E,
                                          int nbits) {
#pragma unroll
  for (int i = 0; i < KPL; ++i) {
    const int pos = run_begin + i * 32 + lane;
    key[i] = pos < run_end ? clamp_key(__ldg(idx + pos), E) : (1 << nbits) - 1;
  }
}

// Lanes of the warp whose key equals this lane's key: one ballot per bit.
__device__ __forceinline__ unsigned match_key(int key, int nbits) {
  unsigned peers = kFull;
  for (int b = 0; b < nbits; ++b) {
    const bool bit = (key >> b) & 1;
    const unsigned set = __ballot_sync(kFull, bit);
    peers &= bit ? set : ~set;
  }
  return peers;
}

// Adds this warp's per-expert counts into cnt[0..E] (row of the warp).
template <int KPL>
__device__ __forceinline__ void count_keys(const int (&key)[KPL], int* cnt, int lane, int E,
                                           int nbits) {
#pragma unroll
  for (int i = 0; i < KPL; ++i) {
    const unsigned peers = match_key(key[i], nbits);
    if (key[i] <= E && lane == __ffs(peers) - 1) cnt[key[i]] += __popc(peers);
    __syncwarp();
  }
}

// Assigns destinations; cnt[e] holds the warp's next free slot of expert e.
template <int KPL>
__device__ __forceinline__ void rank_keys(const int (&key)[KPL], int* cnt, int run_begin,
                                          int lane, int E, int nbits, int32_t* __restrict__ s2d,
                                          int32_t* __restrict__ perm) {
  const unsigned lt = lanemask_lt();
#pragma unroll
  for (int i = 0; i < KPL; ++i) {
    const unsigned peers = match_key(key[i], nbits);
    int dest = 0;
    if (key[i] <= E) dest = cnt[key[i]] + __popc(peers & lt);
    __syncwarp();
    if (key[i] <= E) {
      if (lane == __ffs(peers) - 1) cnt[key[i]] += __popc(peers);
      const int pos = run_begin + i * 32 + lane;
      s2d[pos] = dest;
      perm[dest] = pos;
    }
    __syncwarp();
  }
}

// Block-wide exclusive scan of v (one value per thread of a 1024-thread
// block); returns the exclusive prefix and writes the block total to *total.
__device__ __forceinline__ int block_exclusive_scan(int v, int* s_warp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int o = __shfl_up_sync(kFull, incl, off);
    if (lane >= off) incl += o;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = s_warp[lane];
    int wi = w;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(kFull, wi, off);
      if (lane >= off) wi += o;
    }
    s_warp[lane] = wi - w;  // exclusive prefix of warp totals
    if (lane == 31) s_warp[32] = wi;
  }
  __syncthreads();
  const int r = s_warp[warp] + incl - v;
  *total = s_warp[32];
  __syncthreads();
  return r;
}

// One CTA routes everything: count, scan, rank.
template <int KPL>
__global__ void __launch_bounds__(kRouteThreads) route_single_kernel(
    const int32_t* __restrict__ idx, int n, int E, int32_t* __restrict__ offsets,
    int32_t* __restrict__ s2d, int32_t* __restrict__ perm) {
  extern __shared__ int s_cnt[];  // [kRouteWarps][E+1]
  __shared__ int s_warp[33];
  const int nb = E + 1;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < kRouteWarps * nb; i += kRouteThreads) s_cnt[i] = 0;
  const int run = KPL * 32;
  const int rb = warp * run;
  const int re = min(n, rb + run);
  const int nbits = key_bits(E);
  int key[KPL];
  load_keys<KPL>(key, idx, rb, re, lane, E, nbits);
  __syncthreads();
  int* cnt = s_cnt + warp * nb;
  count_keys<KPL>(key, cnt, lane, E, nbits);
  __syncthreads();
  // Exclusive prefix over warps per expert; expert totals to scan.
  const int e = threadIdx.x;
  int tot = 0;
  if (e < nb) {
    for (int w = 0; w < kRouteWarps; ++w) {
      const int c = s_cnt[w * nb + e];
      s_cnt[w * nb + e] = tot;
      tot += c;
    }
  }
  int all;
  const int base = block_exclusive_scan(e < E ? tot : 0, s_warp, &all);
  if (e < nb) {
    if (e < E) offsets[e] = base;
    else offsets[E] = all;  // the sentinel bin starts after every valid slot
    const int start = (e < E) ? base : all;
    for (int w = 0; w < kRouteWarps; ++w) s_cnt[w * nb + e] += start;
  }
  __syncthreads();
  rank_keys<KPL>(key, cnt, rb, lane, E, nbits, s2d, perm);
}

// Multi-CTA pass 1: per-chunk expert counts -> chunk_counts[chunk][E+1].
__global__ void __launch_bounds__(kRouteThreads) route_count_kernel(
    const int32_t* __restrict__ idx, int n, int E, int32_t* __restrict__ chunk_counts) {
  extern __shared__ int s_cnt[];
  const int nb = E + 1;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < kRouteWarps * nb; i += kRouteThreads) s_cnt[i] = 0;
  const int rb = blockIdx.x * kChunkKeys + warp * kChunkKeyPerLane * 32;
  const int re = min(n, rb + kChunkKeyPerLane * 32);
  const int nbits = key_bits(E);
  int key[kChunkKeyPerLane];
  load_keys<kChunkKeyPerLane>(key, idx, rb, re, lane, E, nbits);
  __syncthreads();
  count_keys<kChunkKeyPerLane>(key, s_cnt + warp * nb, lane, E, nbits);
  __syncthreads();
  for (int e = threadIdx.x; e < nb; e += kRouteThreads) {
    int s = 0;
    for (int w = 0; w < kRouteWarps; ++w) s += s_cnt[w * nb + e];
    chunk_counts[static_cast<int64_t>(blockIdx.x) * nb + e] = s;
  }
}

// Multi-CTA scan: chunk_counts[c][e] -> start of chunk c's first key of
// expert e; writes offsets[0..E].
__global__ void __launch_bounds__(kRouteThreads) route_scan_kernel(
    int32_t* __restrict__ chunk_counts, int nchunks, int E, int32_t* __restrict__ offsets) {
  __shared__ int s_warp[33];
  const int nb = E + 1;
  const int e = threadIdx.x;
  int tot = 0;
  if (e < nb) {
    for (int c = 0; c < nchunks; ++c) {
      const int64_t i = static_cast<int64_t>(c) * nb + e;
      const int v = chunk_counts[i];
      chunk_counts[i] = tot;
      tot += v;
    }
  }
  int all;
  const int base = block_exclusive_scan(e < E ? tot : 0, s_warp, &all);
  if (e < nb) {
    const int start = (e < E) ? base : all;
    offsets[e] = start;
    for (int c = 0; c < nchunks; ++c) chunk_counts[static_cast<int64_t>(c) * nb + e] += start;
  }
}

// Multi-CTA pass 2: recount per warp, add the chunk base, rank.
__global__ void __launch_bounds__(kRouteThreads) route_rank_kernel(
    const int32_t* __restrict__ idx, int n, int E, const int32_t* __restrict__ chunk_start,
    int32_t* __restrict__ s2d, int32_t* __restrict__ perm) {
  extern __shared__ int s_cnt[];
  const int nb = E + 1;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < kRouteWarps * nb; i += kRouteThreads) s_cnt[i] = 0;
  const int rb = blockIdx.x * kChunkKeys + warp * kChunkKeyPerLane * 32;
  const int re = min(n, rb + kChunkKeyPerLane * 32);
  const int nbits = key_bits(E);
  int key[kChunkKeyPerLane];
  load_keys<kChunkKeyPerLane>(key, idx, rb, re, lane, E, nbits);
  __syncthreads();
  int* cnt = s_cnt + warp * nb;
  count_keys<kChunkKeyPerLane>(key, cnt, lane, E, nbits);
  __syncthreads();
  for (int e = threadIdx.x; e < nb; e += kRouteThreads) {
    int run = chunk_start[static_cast<int64_t>(blockIdx.x) * nb + e];
    for (int w = 0; w < kRouteWarps; ++w) {
      const int c = s_cnt[w * nb + e];
      s_cnt[w * nb + e] = run;
      run += c;
    }
  }
  __syncthreads();
  rank_keys<kChunkKeyPerLane>(key, cnt, rb, lane, E, nbits, s2d, perm);
}

// ---- route by expert ---------------------------------------------------------------
//
// One CTA per kRbeExperts consecutive experts (the sentinel bin E is the last
// "expert"), no workspace and one launch.  Every CTA reads all n keys (they
// were just written by the gating kernel, so they come from L2).  For its
// experts e the CTA needs
//   offsets[e] = #{keys < e}                      (a block sum of counts)
//   dest(pos)  = offsets[e] + #{keys == e at positions < pos}.
// In a round, warp w covers 32 * kRbeKeys consecutive positions; lane l loads
// 16-byte vectors at chunk c = 0..kRbeVecs-1, positions c*128 + 4l .. +3 (one
// 512-byte coalesced load per warp and chunk), so inside a warp the position
// order is chunk, then lane, then vector element.  A key's rank is: matches
// of the earlier warps (a scan of per-warp counts through shared memory) +
// matches in the warp's earlier chunks + matches of lower lanes in its chunk
// (ballots) + its own earlier matches.  That is the order of a stable sort by
// expert, the order of torch.argsort(stable=True)
// (tests/test_reference.py:534-558) and of the reference's CUB radix sort
// (smxx/permute/moe_permute.cu:553-563).  With more than one round the
// totals are counted in a first pass.
constexpr int kRbeVecs = 8;                   // 16-byte key vectors per lane per round
constexpr int kRbeKeys = 4 * kRbeVecs;        // keys per lane per round
constexpr int kRbeWarpKeys = 32 * kRbeKeys;   // keys per warp per round
constexpr int kRbeExperts = 2;                // experts per CTA
constexpr uint32_t kRbePad = 0xffffffffu;     // past the end: below no expert (see rbe_load)

// v[4c + q] = raw key at position wb + 128c + 4*lane + q, or kRbePad past n;
// returns the mask of this lane's positions below n.  Keys are not clamped:
// compared as unsigned, a key below e0 (<= E) is a valid expert id, and a
// key outside [0, E) falls in the sentinel bin.  A padded position equals no
// valid id and is below no e0, and the returned mask keeps it out of the
// sentinel bin (every 32-bit pattern is a possible key).
__device__ __forceinline__ uint32_t rbe_load(uint32_t (&v)[kRbeKeys], const int32_t* __restrict__ idx,
                                             int64_t wb, int lane, int64_t n, bool vec_ok) {
  uint32_t valid = 0xffffffffu;
#pragma unroll
  for (int c = 0; c < kRbeVecs; ++c) {
    const int64_t p = wb + 128 * c + 4 * lane;
    if (vec_ok && p + 4 <= n) {
      const int4 q = __ldg(reinterpret_cast<const int4*>(idx + p));
      v[4 * c] = static_cast<uint32_t>(q.x);
      v[4 * c + 1] = static_cast<uint32_t>(q.y);
      v[4 * c + 2] = static_cast<uint32_t>(q.z);
      v[4 * c + 3] = static_cast<uint32_t>(q.w);
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const bool in = p + q < n;
        v[4 * c + q] = in ? static_cast<uint32_t>(__ldg(idx + p + q)) : kRbePad;
        if (!in) valid &= ~(1u << (4 * c + q));
      }
    }
  }
  return valid;
}

// Key v falls in bin b (b < E: equal ids; b == E: any id outside [0, E);
// b > E, a CTA's slot past the sentinel bin: nothing).  Padded positions are
// removed from the sentinel bin by the caller's mask.
__device__ __forceinline__ bool rbe_in_bin(uint32_t v, int b, int E) {
  return b < E ? v == static_cast<uint32_t>(b) : (b == E && v >= static_cast<uint32_t>(E));
}

// Sum over the block of per-warp values published in s[0..nw) (after a
// barrier); every thread gets the total, lane-parallel.
__device__ __forceinline__ int rbe_sum_warps(const int* s, int nw, int lane) {
  return __reduce_add_sync(kFull, lane < nw ? s[lane] : 0);
}

__global__ void __launch_bounds__(1024) route_by_expert_kernel(
    const int32_t* __restrict__ idx, int64_t n, int E, int vec_ok, int32_t* __restrict__ offsets,
    int32_t* __restrict__ s2d, int32_t* __restrict__ perm) {
  __shared__ int s_cnt[kRbeExperts + 1][32];  // per warp: matches of each expert; keys below e0
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  const int e0 = blockIdx.x * kRbeExperts;
  const int64_t per_round = static_cast<int64_t>(nw) * kRbeWarpKeys;
  const int64_t rounds = (n + per_round - 1) / per_round;
  int off[kRbeExperts];
  int base[kRbeExperts];
#pragma unroll
  for (int j = 0; j < kRbeExperts; ++j) base[j] = 0;
  if (rounds > 1) {
    int lt = 0, eq[kRbeExperts] = {};
    for (int64_t r = 0; r < rounds; ++r) {
      uint32_t v[kRbeKeys];
      const uint32_t valid =
          rbe_load(v, idx, r * per_round + static_cast<int64_t>(warp) * kRbeWarpKeys, lane, n, vec_ok);
#pragma unroll
      for (int i = 0; i < kRbeKeys; ++i) {
        lt += v[i] < static_cast<uint32_t>(e0);
#pragma unroll
        for (int j = 0; j < kRbeExperts; ++j)
          eq[j] += rbe_in_bin(v[i], e0 + j, E) && ((valid >> i) & 1u);
      }
    }
    lt = __reduce_add_sync(kFull, lt);
#pragma unroll
    for (int j = 0; j < kRbeExperts; ++j) eq[j] = __reduce_add_sync(kFull, eq[j]);
    if (lane == 0) {
      s_cnt[kRbeExperts][warp] = lt;
#pragma unroll
      for (int j = 0; j < kRbeExperts; ++j) s_cnt[j][warp] = eq[j];
    }
    __syncthreads();
    off[0] = rbe_sum_warps(s_cnt[kRbeExperts], nw, lane);
#pragma unroll
    for (int j = 1; j < kRbeExperts; ++j) off[j] = off[j - 1] + rbe_sum_warps(s_cnt[j - 1], nw, lane);
    __syncthreads();
  }
  const unsigned lanes_below = lanemask_lt();
  for (int64_t r = 0; r < rounds; ++r) {
    const int64_t wb = r * per_round + static_cast<int64_t>(warp) * kRbeWarpKeys;
    uint32_t v[kRbeKeys];
    const uint32_t valid = rbe_load(v, idx, wb, lane, n, vec_ok);
    int lt = 0;
    uint32_t m[kRbeExperts] = {};
#pragma unroll
    for (int i = 0; i < kRbeKeys; ++i) {
      lt += v[i] < static_cast<uint32_t>(e0);
#pragma unroll
      for (int j = 0; j < kRbeExperts; ++j)
        m[j] |= static_cast<uint32_t>(rbe_in_bin(v[i], e0 + j, E)) << i;
    }
#pragma unroll
    for (int j = 0; j < kRbeExperts; ++j) m[j] &= valid;
    lt = __reduce_add_sync(kFull, lt);
    int cw[kRbeExperts];
#pragma unroll
    for (int j = 0; j < kRbeExperts; ++j) cw[j] = __reduce_add_sync(kFull, __popc(m[j]));
    if (lane == 0) {
      s_cnt[kRbeExperts][warp] = lt;
#pragma unroll
      for (int j = 0; j < kRbeExperts; ++j) s_cnt[j][warp] = cw[j];
    }
    __syncthreads();
    // Lane l holds warp l's count: an inclusive scan over lanes gives every
    // warp its prefix and the block total.
    int wpre[kRbeExperts], tot[kRbeExperts];
#pragma unroll
    for (int j = 0; j < kRbeExperts; ++j) {
      const int c = lane < nw ? s_cnt[j][lane] : 0;
      int inc = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(kFull, inc, o);
        if (lane >= o) inc += t;
      }
      wpre[j] = __shfl_sync(kFull, inc - c, warp);
      tot[j] = __shfl_sync(kFull, inc, 31);
    }
    if (rounds == 1) {
      off[0] = rbe_sum_warps(s_cnt[kRbeExperts], nw, lane);
#pragma unroll
      for (int j = 1; j < kRbeExperts; ++j) off[j] = off[j - 1] + tot[j - 1];
    }
    __syncthreads();  // s_cnt is rewritten by the next round
#pragma unroll
    for (int j = 0; j < kRbeExperts; ++j) {
      int d = off[j] + base[j] + wpre[j];
#pragma unroll
      for (int c = 0; c < kRbeVecs; ++c) {
        uint32_t own = (m[j] >> (4 * c)) & 0xFu;
        if (!__any_sync(kFull, own != 0u)) continue;
        const uint32_t b0 = __ballot_sync(kFull, own & 1u), b1 = __ballot_sync(kFull, own & 2u);
        const uint32_t b2 = __ballot_sync(kFull, own & 4u), b3 = __ballot_sync(kFull, own & 8u);
        int dd = d + __popc(b0 & lanes_below) + __popc(b1 & lanes_below) +
                 __popc(b2 & lanes_below) + __popc(b3 & lanes_below);
        while (own != 0u) {
          const int q = __ffs(own) - 1;
          own &= own - 1u;
          const int64_t pos = wb + 128 * c + 4 * lane + q;
          s2d[pos] = dd;
          perm[dd] = static_cast<int32_t>(pos);
          ++dd;
        }
        d += __popc(b0) + __popc(b1) + __popc(b2) + __popc(b3);
      }
      base[j] += tot[j];
    }
  }
  if (threadIdx.x == 0) {
#pragma unroll
    for (int j = 0; j < kRbeExperts; ++j)
      if (e0 + j <= E) offsets[e0 + j] = off[j];
  }
}

// ---- row copy ------------------------------------------------------------------

constexpr int kCopyThreads = 128;
constexpr int kCopyVecPerThread = 8;   // up to 8 x 16 B per thread in flight

// grid = (num_tokens, slices); slice y covers vectors [y*span, (y+1)*span).
__global__ void __launch_bounds__(kCopyThreads) permute_rows_vec_kernel(
    const uint4* __restrict__ src, uint4* __restrict__ dst, const int32_t* __restrict__ s2d,
    int topk, int64_t vec_per_row, int span) {
  __shared__ int32_t s_dest[32];
  const int t = blockIdx.x;
  if (threadIdx.x < topk) s_dest[threadIdx.x] = __ldg(s2d + static_cast<int64_t>(t) * topk + threadIdx.x);
  __syncthreads();
  const int64_t v_begin = static_cast<int64_t>(blockIdx.y) * span;
  const int64_t v_end = min(vec_per_row, v_begin + span);
  const uint4* srow = src + static_cast<int64_t>(t) * vec_per_row;
  for (int64_t v0 = v_begin + threadIdx.x; v0 < v_end; v0 += kCopyThreads * kCopyVecPerThread) {
    uint4 r[kCopyVecPerThread];
#pragma unroll
    for (int i = 0; i < kCopyVecPerThread; ++i) {
      const int64_t v = v0 + static_cast<int64_t>(i) * kCopyThreads;
      if (v < v_end) r[i] = ldg_nc_v4(srow + v);
    }
    for (int k = 0; k < topk; ++k) {
      uint4* drow = dst + static_cast<int64_t>(s_dest[k]) * vec_per_row;
#pragma unroll
      for (int i = 0; i < kCopyVecPerThread; ++i) {
        const int64_t v = v0 + static_cast<int64_t>(i) * kCopyThreads;
        if (v < v_end) drow[v] = r[i];
      }
    }
  }
}

// Rows whose byte length is not a multiple of 16: 2-byte units.
__global__ void permute_rows_u16_kernel(const uint16_t* __restrict__ src, uint16_t* __restrict__ dst,
                                        const int32_t* __restrict__ s2d, int topk,
                                        int64_t u16_per_row) {
  const int t = blockIdx.x;
  const uint16_t* srow = src + static_cast<int64_t>(t) * u16_per_row;
  for (int k = 0; k < topk; ++k) {
    uint16_t* drow = dst + static_cast<int64_t>(__ldg(s2d + static_cast<int64_t>(t) * topk + k)) * u16_per_row;
    for (int64_t i = threadIdx.x; i < u16_per_row; i += blockDim.x) drow[i] = srow[i];
  }
}

// ---- unpermute -----------------------------------------------------------------

constexpr int kUnpThreads = 128;

// Loads the token's (dest row, weight) pairs into shared memory.
__device__ __forceinline__ void load_slots(const float* __restrict__ w, const int32_t* __restrict__ s2d,
                                           int t, int topk, float* s_w, int32_t* s_d) {
  if (threadIdx.x < topk) {
    const int64_t i = static_cast<int64_t>(t) * topk + threadIdx.x;
    s_w[threadIdx.x] = __ldg(w + i);
    s_d[threadIdx.x] = __ldg(s2d + i);
  }
  __syncthreads();
}

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& raw, float (&f)[8]) {
  const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int j = 0; j < 8; ++j) f[j] = Elem<T>::to_f(e[j]);
}

template <typename T>
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 raw;
  T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
  for (int j = 0; j < 8; ++j) e[j] = Elem<T>::from_f(f[j]);
  return raw;
}

// out[t] = round(sum_k fma(w_k, x_k, acc)); grid = (T, slices), vector path.
template <typename T, int KMAX>
__global__ void __launch_bounds__(kUnpThreads) unpermute_sum_kernel(
    T* __restrict__ out, const T* __restrict__ in, const float* __restrict__ w,
    const int32_t* __restrict__ s2d, int topk, int H, int span) {
  __shared__ float s_w[32];
  __shared__ int32_t s_d[32];
  const int t = blockIdx.x;
  load_slots(w, s2d, t, topk, s_w, s_d);
  const int nvec = H / 8;
  const int v_end = min(nvec, (blockIdx.y + 1) * span);
  for (int v = blockIdx.y * span + threadIdx.x; v < v_end; v += kUnpThreads) {
    uint4 raw[KMAX];
#pragma unroll
    for (int k = 0; k < KMAX; ++k)
      if (k < topk) raw[k] = ldg_nc_v4(in + static_cast<int64_t>(s_d[k]) * H + v * 8);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
      if (k < topk) {
        float x[8];
        unpack8<T>(raw[k], x);
        const float wk = s_w[k];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = __fmaf_rn(wk, x[j], acc[j]);
      }
    }
    *reinterpret_cast<uint4*>(out + static_cast<int64_t>(t) * H + v * 8) = pack8<T>(acc);
  }
}

// Scalar variant for any H and topk <= 32.
template <typename T>
__global__ void unpermute_sum_scalar_kernel(T* __restrict__ out, const T* __restrict__ in,
                                            const float* __restrict__ w,
                                            const int32_t* __restrict__ s2d, int topk, int H) {
  __shared__ float s_w[32];
  __shared__ int32_t s_d[32];
  const int t = blockIdx.x;
  load_slots(w, s2d, t, topk, s_w, s_d);
  for (int h = threadIdx.x; h < H; h += blockDim.x) {
    float acc = 0.0f;
    for (int k = 0; k < topk; ++k)
      acc = __fmaf_rn(s_w[k], Elem<T>::to_f(in[static_cast<int64_t>(s_d[k]) * H + h]), acc);
    out[static_cast<int64_t>(t) * H + h] = Elem<T>::from_f(acc);
  }
}

// Per-slot: one CTA per (token, slot) row; OUT_F32 writes fp32, else 16-bit.
template <typename T, bool OUT_F32>
__global__ void __launch_bounds__(kUnpThreads) unpermute_perslot_kernel(
    void* __restrict__ out, const T* __restrict__ in, const float* __restrict__ w,
    const int32_t* __restrict__ s2d, int H, int vec_ok) {
  const int64_t slot = blockIdx.x;  // t * topk + k
  const float wk = __ldg(w + slot);
  const T* row = in + static_cast<int64_t>(__ldg(s2d + slot)) * H;
  if (vec_ok) {
    const int nvec = H / 8;
    for (int v = threadIdx.x; v < nvec; v += kUnpThreads) {
      float x[8];
      unpack8<T>(ldg_nc_v4(row + v * 8), x);
#pragma unroll
      for (int j = 0; j < 8; ++j) x[j] = __fmul_rn(wk, x[j]);
      if (OUT_F32) {
        float4* o = reinterpret_cast<float4*>(static_cast<float*>(out) + slot * H + v * 8);
        o[0] = make_float4(x[0], x[1], x[2], x[3]);
        o[1] = make_float4(x[4], x[5], x[6], x[7]);
      } else {
        *reinterpret_cast<uint4*>(static_cast<T*>(out) + slot * H + v * 8) = pack8<T>(x);
      }
    }
  } else {
    for (int h = threadIdx.x; h < H; h += kUnpThreads) {
      const float v = __fmul_rn(wk, Elem<T>::to_f(row[h]));
      if (OUT_F32) static_cast<float*>(out)[slot * H + h] = v;
      else static_cast<T*>(out)[slot * H + h] = Elem<T>::from_f(v);
    }
  }
}

// Fixed-order slot reduce.  Each thread owns 8 consecutive h of one token.
template <bool IN_F32>
__global__ void __launch_bounds__(256) reduce_slots_vec_kernel(
    __nv_bfloat16* __restrict__ out, const void* __restrict__ in, int T, int topk, int H) {
  const int nvec = H / 8;
  const int64_t total = static_cast<int64_t>(T) * nvec;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / nvec;
    const int v = static_cast<int>(i - t * nvec);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < topk; ++k) {
      const int64_t off = (t * topk + k) * H + static_cast<int64_t>(v) * 8;
      float x[8];
      if (IN_F32) {
        const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(in) + off);
        const float4 a = __ldg(p), b = __ldg(p + 1);
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
        x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
      } else {
        unpack8<__nv_bfloat16>(ldg_nc_v4(static_cast<const __nv_bfloat16*>(in) + off), x);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = __fadd_rn(acc[j], x[j]);
    }
    *reinterpret_cast<uint4*>(out + t * H + static_cast<int64_t>(v) * 8) = pack8<__nv_bfloat16>(acc);
  }
}

template <bool IN_F32>
__global__ void reduce_slots_scalar_kernel(__nv_bfloat16* __restrict__ out, const void* __restrict__ in,
                                           int T, int topk, int H) {
  const int64_t total = static_cast<int64_t>(T) * H;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / H, h = i - t * H;
    float acc = 0.0f;
    for (int k = 0; k < topk; ++k) {
      const int64_t off = (t * topk + k) * H + h;
      const float x = IN_F32 ? static_cast<const float*>(in)[off]
                             : __bfloat162float(static_cast<const __nv_bfloat16*>(in)[off]);
      acc = __fadd_rn(acc, x);
    }
    out[i] = __float2bfloat16_rn(acc);
  }
}

// Vectors per row slice so a row gets ~4 CTAs when there are few tokens.
int copy_span(int64_t vec_per_row, int64_t tokens) {
  const int64_t want_ctas = 4ll * num_sms();
  int64_t slices = tokens >= want_ctas ? 1 : ceil_div(want_ctas, tokens);
  const int64_t max_slices = ceil_div(vec_per_row, kCopyThreads);
  if (slices > max_slices) slices = max_slices;
  if (slices < 1) slices = 1;
  return static_cast<int>(ceil_div(vec_per_row, slices));
}

}  // namespace

// Workspace of the multi-CTA route: per-chunk counts, 256-byte aligned.
size_t permute_workspace_bytes(int64_t n_keys, int num_experts) {
  if (n_keys <= kSingleMaxKeys) return 256;
  const int64_t nchunks = ceil_div(n_keys, kChunkKeys);
  return static_cast<size_t>(ceil_div(nchunks * (num_experts + 1) * 4, 256) * 256);
}

// Routing only (offsets and maps).  `ws` must hold permute_workspace_bytes.
lsek_status launch_route(const int32_t* idx, int64_t n, int E, int32_t* offsets, int32_t* s2d,
                         int32_t* perm, void* ws, cudaStream_t st) {
  const size_t smem = static_cast<size_t>(kRouteWarps) * (E + 1) * sizeof(int);
  static PerDeviceOnce attrs;
  const cudaError_t ae = once_per_device(attrs, [] {
    const int max_smem = kRouteWarps * 1024 * 4;
    cudaError_t e = cudaSuccess;
    auto set = [&](const void* fn) {
      const cudaError_t r =
          cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
      if (r != cudaSuccess) e = r;
    };
    set(reinterpret_cast<const void*>(route_single_kernel<1>));
    set(reinterpret_cast<const void*>(route_single_kernel<2>));
    set(reinterpret_cast<const void*>(route_single_kernel<4>));
    set(reinterpret_cast<const void*>(route_count_kernel));
    set(reinterpret_cast<const void*>(route_rank_kernel));
    return e;
  });
  if (ae != cudaSuccess) return fail(LSEK_ERR_CUDA, "moe_permute: %s", cudaGetErrorString(ae));
  if (n <= kSingleMaxKeys) {
    const int kpl = static_cast<int>(ceil_div(n, kRouteThreads));
    if (kpl <= 1)      route_single_kernel<1><<<1, kRouteThreads, smem, st>>>(idx, static_cast<int>(n), E, offsets, s2d, perm);
    else if (kpl <= 2) route_single_kernel<2><<<1, kRouteThreads, smem, st>>>(idx, static_cast<int>(n), E, offsets, s2d, perm);
    else               route_single_kernel<4><<<1, kRouteThreads, smem, st>>>(idx, static_cast<int>(n), E, offsets, s2d, perm);
    return check_launch("moe_permute(route)");
  }
  const int nchunks = static_cast<int>(ceil_div(n, kChunkKeys));
  int32_t* chunk = static_cast<int32_t*>(ws);
  route_count_kernel<<<nchunks, kRouteThreads, smem, st>>>(idx, static_cast<int>(n), E, chunk);
  route_scan_kernel<<<1, kRouteThreads, 0, st>>>(chunk, nchunks, E, offsets);
  route_rank_kernel<<<nchunks, kRouteThreads, smem, st>>>(idx, static_cast<int>(n), E, chunk, s2d, perm);
  return check_launch("moe_permute(route)");
}

// Routing in one launch with no workspace (route_by_expert_kernel).
lsek_status launch_route_by_expert(const int32_t* idx, int64_t n, int E, int32_t* offsets,
                                   int32_t* s2d, int32_t* perm, cudaStream_t st) {
  int64_t threads = ceil_div(n, kRbeWarpKeys) * 32;
  if (threads < 32) threads = 32;
  if (threads > 1024) threads = 1024;
  const int grid = static_cast<int>(ceil_div(E + 1, kRbeExperts));
  const int vec_ok = reinterpret_cast<uintptr_t>(idx) % 16 == 0;
  route_by_expert_kernel<<<grid, static_cast<unsigned>(threads), 0, st>>>(idx, n, E, vec_ok,
                                                                         offsets, s2d, perm);
  return check_launch("moe_permute(route)");
}

lsek_status launch_permute_rows(void* dst, const void* src, const int32_t* s2d, int64_t T,
                                int topk, int64_t row_bytes, cudaStream_t st) {
  if (row_bytes % 16 == 0 && reinterpret_cast<uintptr_t>(dst) % 16 == 0 &&
      reinterpret_cast<uintptr_t>(src) % 16 == 0) {
    const int64_t vpr = row_bytes / 16;
    const int span = copy_span(vpr, T);
    const dim3 grid(static_cast<unsigned>(T), static_cast<unsigned>(ceil_div(vpr, span)));
    permute_rows_vec_kernel<<<grid, kCopyThreads, 0, st>>>(
        static_cast<const uint4*>(src), static_cast<uint4*>(dst), s2d, topk, vpr, span);
  } else {
    permute_rows_u16_kernel<<<static_cast<unsigned>(T), 256, 0, st>>>(
        static_cast<const uint16_t*>(src), static_cast<uint16_t*>(dst), s2d, topk, row_bytes / 2);
  }
  return check_launch("moe_permute(copy)");
}

template <typename T>
static lsek_status launch_unpermute_sum_t(void* out, const void* in, const float* w,
                                          const int32_t* s2d, int Tn, int topk, int H,
                                          cudaStream_t st) {
  const bool vec_ok = H % 8 == 0 && reinterpret_cast<uintptr_t>(in) % 16 == 0 &&
                      reinterpret_cast<uintptr_t>(out) % 16 == 0;
  if (vec_ok && topk <= 16) {
    const int nvec = H / 8;
    const int64_t want = 4ll * num_sms();
    int slices = Tn >= want ? 1 : static_cast<int>(ceil_div(want, Tn));
    const int max_slices = static_cast<int>(ceil_div(nvec, kUnpThreads));
    if (slices > max_slices) slices = max_slices;
    const int span = static_cast<int>(ceil_div(nvec, slices));
    const dim3 grid(Tn, static_cast<unsigned>(ceil_div(nvec, span)));
    if (topk <= 8)
      unpermute_sum_kernel<T, 8><<<grid, kUnpThreads, 0, st>>>(
          static_cast<T*>(out), static_cast<const T*>(in), w, s2d, topk, H, span);
    else
      unpermute_sum_kernel<T, 16><<<grid, kUnpThreads, 0, st>>>(
          static_cast<T*>(out), static_cast<const T*>(in), w, s2d, topk, H, span);
  } else {
    unpermute_sum_scalar_kernel<T><<<Tn, 256, 0, st>>>(static_cast<T*>(out),
                                                        static_cast<const T*>(in), w, s2d, topk, H);
  }
  return check_launch("moe_unpermute");
}

template <typename T>
static lsek_status launch_perslot_t(void* out, const void* in, const float* w, const int32_t* s2d,
                                    int Tn, int topk, int H, bool out_f32, cudaStream_t st) {
  const int vec_ok = H % 8 == 0 && reinterpret_cast<uintptr_t>(in) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(out) % 16 == 0;
  const unsigned grid = static_cast<unsigned>(static_cast<int64_t>(Tn) * topk);
  if (out_f32)
    unpermute_perslot_kernel<T, true><<<grid, kUnpThreads, 0, st>>>(out, static_cast<const T*>(in), w, s2d, H, vec_ok);
  else
    unpermute_perslot_kernel<T, false><<<grid, kUnpThreads, 0, st>>>(out, static_cast<const T*>(in), w, s2d, H, vec_ok);
  return check_launch("moe_unpermute(perslot)");
}

}  // namespace lsek

using namespace lsek;

static bool dtype_16bit(int32_t dt) { return dt == LSEK_BF16 || dt == LSEK_FP16; }

// ---- allocation-free permute ------------------------------------------------------------
//
// Scratch of lsek_moe_permute_noalloc: the per-chunk expert counts of the
// multi-CTA route, in a fixed device array instead of a caller workspace.
// The array exists once per GPU that loads this library and lives until
// the process exits.  Host code must not hand `g_noalloc_scratch` itself to
// a kernel: on the host that name is only a stand-in for the symbol, so its
// device address is looked up with cudaGetSymbolAddress, once per device.
static __device__ __align__(256) int32_t g_noalloc_scratch[LSEK_NOALLOC_PERMUTE_SCRATCH_BYTES / 4];

namespace {
constexpr int kMaxDevices = 64;
std::once_flag g_noalloc_once[kMaxDevices];
void* g_noalloc_ptr[kMaxDevices];
cudaError_t g_noalloc_err[kMaxDevices];

// Device address of g_noalloc_scratch on the current device; the first call
// per device performs the lookup with that device current.
lsek_status noalloc_scratch(void** out) {
  int dev = 0;
  LSEK_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices)
    return fail(LSEK_ERR_UNSUPPORTED, "moe_permute_noalloc: device ordinal %d out of range", dev);
  std::call_once(g_noalloc_once[dev], [dev] {
    g_noalloc_err[dev] = cudaGetSymbolAddress(&g_noalloc_ptr[dev], g_noalloc_scratch);
  });
  if (g_noalloc_err[dev] != cudaSuccess)
    return fail(LSEK_ERR_CUDA, "moe_permute_noalloc: cudaGetSymbolAddress failed: %s",
                cudaGetErrorString(g_noalloc_err[dev]));
  *out = g_noalloc_ptr[dev];
  return LSEK_OK;
}
}  // namespace

extern "C" size_t lsek_moe_permute_workspace_size(int32_t max_tokens, int32_t max_topk,
                                                  int32_t num_experts) {
  if (max_tokens < 0 || max_topk < 0 || num_experts < 0) return 0;
  return permute_workspace_bytes(static_cast<int64_t>(max_tokens) * max_topk, num_experts);
}

extern "C" lsek_status lsek_moe_permute(void* permuted_input, int32_t* expert_offsets,
                                        int32_t* src_to_dest_map, int32_t* permuted_idx,
                                        const void* hidden_states, const int32_t* topk_indices,
                                        int32_t num_tokens, int32_t topk, int32_t hidden_dim,
                                        int32_t num_experts, int32_t elem_size_bytes,
                                        void* workspace, size_t workspace_bytes, void* stream) {
  LSEK_REQUIRE(num_tokens >= 0 && topk >= 0 && hidden_dim >= 0,
               "moe_permute: sizes must be >= 0");
  LSEK_REQUIRE(num_experts >= 1, "moe_permute: num_experts must be >= 1");
  if (num_experts > 1023)
    return fail(LSEK_ERR_UNSUPPORTED, "moe_permute: num_experts must be <= 1023");
  LSEK_REQUIRE(elem_size_bytes == 2 || elem_size_bytes == 4,
               "moe_permute: elem_size_bytes must be 2 or 4, got %d", elem_size_bytes);
  LSEK_REQUIRE(topk <= 32, "moe_permute: topk must be <= 32");
  LSEK_REQUIRE(expert_offsets != nullptr, "moe_permute: expert_offsets is NULL");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t n = static_cast<int64_t>(num_tokens) * topk;
  LSEK_REQUIRE(n < (1ll << 31), "moe_permute: num_tokens * topk must fit in int32");
  if (n == 0) {
    LSEK_CUDA_TRY(cudaMemsetAsync(expert_offsets, 0, sizeof(int32_t) * (num_experts + 1), st));
    return LSEK_OK;
  }
  LSEK_REQUIRE(permuted_input && src_to_dest_map && permuted_idx && hidden_states && topk_indices,
               "moe_permute: NULL tensor pointer");
  const size_t need = permute_workspace_bytes(n, num_experts);
  if (n > kSingleMaxKeys) {
    LSEK_REQUIRE(workspace != nullptr && workspace_bytes >= need,
                 "moe_permute: workspace of %zu bytes required, got %zu", need, workspace_bytes);
  }
  lsek_status s = launch_route(topk_indices, n, num_experts, expert_offsets, src_to_dest_map,
                               permuted_idx, workspace, st);
  if (s != LSEK_OK) return s;
  if (hidden_dim == 0) return LSEK_OK;
  return launch_permute_rows(permuted_input, hidden_states, src_to_dest_map, num_tokens, topk,
                             static_cast<int64_t>(hidden_dim) * elem_size_bytes, st);
}

extern "C" lsek_status lsek_moe_route(int32_t* expert_offsets, int32_t* src_to_dest_map,
                                      int32_t* permuted_idx, const int32_t* topk_indices,
                                      int32_t num_tokens, int32_t topk, int32_t num_experts,
                                      void* stream) {
  LSEK_REQUIRE(num_tokens >= 0 && topk >= 0, "moe_route: sizes must be >= 0");
  LSEK_REQUIRE(num_experts >= 1, "moe_route: num_experts must be >= 1");
  if (num_experts > 1023)
    return fail(LSEK_ERR_UNSUPPORTED, "moe_route: num_experts must be <= 1023");
  LSEK_REQUIRE(topk <= 32, "moe_route: topk must be <= 32");
  LSEK_REQUIRE(expert_offsets != nullptr, "moe_route: expert_offsets is NULL");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t n = static_cast<int64_t>(num_tokens) * topk;
  LSEK_REQUIRE(n < (1ll << 31), "moe_route: num_tokens * topk must fit in int32");
  if (n == 0) {
    LSEK_CUDA_TRY(cudaMemsetAsync(expert_offsets, 0, sizeof(int32_t) * (num_experts + 1), st));
    return LSEK_OK;
  }
  LSEK_REQUIRE(src_to_dest_map && permuted_idx && topk_indices, "moe_route: NULL tensor pointer");
  return launch_route_by_expert(topk_indices, n, num_experts, expert_offsets, src_to_dest_map,
                                permuted_idx, st);
}

extern "C" lsek_status lsek_moe_permute_noalloc(void* permuted_input, int32_t* expert_offsets,
                                                int32_t* src_to_dest_map, int32_t* permuted_idx,
                                                const void* hidden_states,
                                                const int32_t* topk_indices, int32_t num_tokens,
                                                int32_t topk, int32_t hidden_dim,
                                                int32_t num_experts, int32_t elem_size_bytes,
                                                void* stream) {
  LSEK_REQUIRE(num_tokens >= 0 && topk >= 0 && hidden_dim >= 0,
               "moe_permute_noalloc: sizes must be >= 0");
  LSEK_REQUIRE(num_experts >= 1, "moe_permute_noalloc: num_experts must be >= 1");
  if (num_experts > 1023)
    return fail(LSEK_ERR_UNSUPPORTED, "moe_permute_noalloc: num_experts must be <= 1023");
  const int64_t n = static_cast<int64_t>(num_tokens) * topk;
  const size_t need = permute_workspace_bytes(n, num_experts);
  LSEK_REQUIRE(need <= LSEK_NOALLOC_PERMUTE_SCRATCH_BYTES,
               "moe_permute_noalloc: %lld slots over %d experts need %zu bytes of scratch, more "
               "than the %u-byte static buffer; call lsek_moe_permute with a workspace instead",
               static_cast<long long>(n), num_experts, need,
               static_cast<unsigned>(LSEK_NOALLOC_PERMUTE_SCRATCH_BYTES));
  void* scratch = nullptr;
  const lsek_status s = noalloc_scratch(&scratch);
  if (s != LSEK_OK) return s;
  return lsek_moe_permute(permuted_input, expert_offsets, src_to_dest_map, permuted_idx,
                          hidden_states, topk_indices, num_tokens, topk, hidden_dim, num_experts,
                          elem_size_bytes, scratch, LSEK_NOALLOC_PERMUTE_SCRATCH_BYTES, stream);
}

extern "C" lsek_status lsek_moe_unpermute(void* output, const void* permuted_output,
                                          const float* topk_weights,
                                          const int32_t* src_to_dest_map, int32_t num_tokens,
                                          int32_t topk, int32_t hidden_dim, int32_t dtype,
                                          int32_t fp32_output, void* stream) {
  LSEK_REQUIRE(num_tokens >= 0 && topk >= 0 && hidden_dim >= 0,
               "moe_unpermute: sizes must be >= 0");
  LSEK_REQUIRE(dtype_16bit(dtype), "moe_unpermute: permuted_output must be bf16 or fp16");
  LSEK_REQUIRE(topk <= 32, "moe_unpermute: topk must be <= 32, got %d", topk);
  if (num_tokens == 0 || hidden_dim == 0) return LSEK_OK;
  LSEK_REQUIRE(topk >= 1, "moe_unpermute: topk must be >= 1");
  LSEK_REQUIRE(output && permuted_output && topk_weights && src_to_dest_map,
               "moe_unpermute: NULL tensor pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (fp32_output) {
    return dtype == LSEK_BF16
               ? launch_perslot_t<__nv_bfloat16>(output, permuted_output, topk_weights,
                                                 src_to_dest_map, num_tokens, topk, hidden_dim,
                                                 true, st)
               : launch_perslot_t<__half>(output, permuted_output, topk_weights, src_to_dest_map,
                                          num_tokens, topk, hidden_dim, true, st);
  }
  return dtype == LSEK_BF16
             ? launch_unpermute_sum_t<__nv_bfloat16>(output, permuted_output, topk_weights,
                                                     src_to_dest_map, num_tokens, topk,
                                                     hidden_dim, st)
             : launch_unpermute_sum_t<__half>(output, permuted_output, topk_weights,
                                              src_to_dest_map, num_tokens, topk, hidden_dim, st);
}

extern "C" lsek_status lsek_moe_unpermute_perslot(void* output, const void* permuted_output,
                                                  const float* topk_weights,
                                                  const int32_t* src_to_dest_map,
                                                  int32_t num_tokens, int32_t topk,
                                                  int32_t hidden_dim, int32_t dtype,
                                                  void* stream) {
  LSEK_REQUIRE(num_tokens >= 0 && topk >= 0 && hidden_dim >= 0,
               "moe_unpermute_perslot: sizes must be >= 0");
  LSEK_REQUIRE(dtype_16bit(dtype), "moe_unpermute_perslot: permuted_output must be bf16 or fp16");
  if (num_tokens == 0 || topk == 0 || hidden_dim == 0) return LSEK_OK;
  LSEK_REQUIRE(output && permuted_output && topk_weights && src_to_dest_map,
               "moe_unpermute_perslot: NULL tensor pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return dtype == LSEK_BF16
             ? launch_perslot_t<__nv_bfloat16>(output, permuted_output, topk_weights,
                                               src_to_dest_map, num_tokens, topk, hidden_dim,
                                               false, st)
             : launch_perslot_t<__half>(output, permuted_output, topk_weights, src_to_dest_map,
                                        num_tokens, topk, hidden_dim, false, st);
}

extern "C" lsek_status lsek_moe_combine_reduce_slots(void* output_bf16, const void* input_perslot,
                                                     int32_t num_tokens, int32_t topk,
                                                     int32_t hidden_dim, int32_t in_dtype,
                                                     void* stream) {
  LSEK_REQUIRE(num_tokens >= 0 && topk >= 0 && hidden_dim >= 0,
               "moe_combine_reduce_slots: sizes must be >= 0");
  LSEK_REQUIRE(in_dtype == LSEK_FP32 || in_dtype == LSEK_BF16,
               "moe_combine_reduce_slots: input must be fp32 or bf16");
  const int64_t total = static_cast<int64_t>(num_tokens) * hidden_dim;
  if (total == 0) return LSEK_OK;
  LSEK_REQUIRE(output_bf16 != nullptr && (topk == 0 || input_perslot != nullptr),
               "moe_combine_reduce_slots: NULL tensor pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool f32 = in_dtype == LSEK_FP32;
  const bool vec_ok = hidden_dim % 8 == 0 && reinterpret_cast<uintptr_t>(output_bf16) % 16 == 0 &&
                      reinterpret_cast<uintptr_t>(input_perslot) % 16 == 0;
  const int threads = 256;
  const int64_t items = vec_ok ? total / 8 : total;
  int64_t grid = ceil_div(items, threads);
  const int64_t cap = 16ll * num_sms();
  if (grid > cap) grid = cap;
  if (vec_ok) {
    if (f32) reduce_slots_vec_kernel<true><<<static_cast<unsigned>(grid), threads, 0, st>>>(
        static_cast<__nv_bfloat16*>(output_bf16), input_perslot, num_tokens, topk, hidden_dim);
    else reduce_slots_vec_kernel<false><<<static_cast<unsigned>(grid), threads, 0, st>>>(
        static_cast<__nv_bfloat16*>(output_bf16), input_perslot, num_tokens, topk, hidden_dim);
  } else {
    if (f32) reduce_slots_scalar_kernel<true><<<static_cast<unsigned>(grid), threads, 0, st>>>(
        static_cast<__nv_bfloat16*>(output_bf16), input_perslot, num_tokens, topk, hidden_dim);
    else reduce_slots_scalar_kernel<false><<<static_cast<unsigned>(grid), threads, 0, st>>>(
        static_cast<__nv_bfloat16*>(output_bf16), input_perslot, num_tokens, topk, hidden_dim);
  }
  return check_launch("moe_combine_reduce_slots");
}
