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
// 1024 threads walks the rows in chunks.
__global__ void __launch_bounds__(1024) ep_slot_scan_kernel(const int32_t* __restrict__ ids, int R,
                                                            int k, int32_t* __restrict__ slot_row) {
  __shared__ int s_warp[33];
  __shared__ int s_carry;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) s_carry = 0;
  __syncthreads();
  for (int base = 0; base < R; base += 1024) {
    const int r = base + threadIdx.x;
    int c = 0;
    if (r < R)
      for (int j = 0; j < k; ++j) c += __ldg(ids + static_cast<int64_t>(r) * k + j) >= 0;
    int incl = c;
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
    if (r < R) slot_row[r] = s_carry + s_warp[warp] + incl - c;
    __syncthreads();
    if (threadIdx.x == 0) s_carry += s_warp[32];
    __syncthreads();
  }
  if (threadIdx.x == 0) slot_row[R] = s_carry;
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
// expert adds +0.  Rows at or past comb_count are never read.
__global__ void __launch_bounds__(kThreads) ep_combine_reduce_kernel(
    __nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ comb,
    const int32_t* __restrict__ idx, const int32_t* __restrict__ pair_row,
    const int32_t* __restrict__ slot_row, int32_t comb_count, int k, int H, int E, int G,
    int span) {
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
    for (int j = 0; j < k; ++j) {
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
  for (int64_t v = threadIdx.x; v < vec_per_row; v += kThreads) {
    const uint4 r = ldg_nc_v4(srow + v);
    for (int j = 0; j < topk; ++j)
      if (s_dest[j] < nv) dst[static_cast<int64_t>(s_dest[j]) * vec_per_row + v] = r;
  }
}

}  // namespace
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
  ep_slot_scan_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(ids, rows, topk, slot_row);
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
  ep_combine_reduce_kernel<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<__nv_bfloat16*>(out), static_cast<const __nv_bfloat16*>(comb_rows), topk_indices,
      pair_row, slot_row, comb_count, topk, hidden_dim, num_experts, world_size, span);
  return check_launch("ep_combine_reduce");
}
