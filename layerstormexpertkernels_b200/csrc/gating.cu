// Top-k gating and adaptive gating for sm_100a.
//
// Top-k gating gives each token a segment of LPT lanes: 16 (two tokens per
// warp, so each selection-round instruction below serves both) when E <= 128,
// topk <= 16 and n_group <= 16, else the whole warp, as at DeepSeek-V3 shape.
// Lane l of a segment owns the EPL consecutive experts [l*EPL, (l+1)*EPL),
// loaded (with the bias) as 16-byte vectors, so a segment reads a token's
// logits row as one contiguous 1 KB (E=256) burst and every later phase runs
// in registers:
//   1. score   s = sigmoid(x) or sqrt(softplus(x)); sel = s + bias
//   2. groups  (n_group > 1) per-group sum of the top-2 sel values, then each
//              lane g computes its group's rank among all groups with
//              shuffles (ties go to the lower group) and a ballot gives the
//              kept-group mask; experts of dropped groups leave the race
//   3. top-k   topk rounds of a segment arg-max on (order-preserving key of sel,
//              expert id), ties to the lower id; the owning lane retires its
//              winner and rescans its EPL candidates
//   4. weights unbiased score of each winner, summed in selection order,
//              optional w *= routed_scaling_factor / sum
// This follows ref_topk_gating (tests/test_reference.py:133-187) and the
// selection order of warp_topk_select (sm120/gating/topk_gating.cu:105-139).
// The reference kernel instead runs one 256-thread block per token with four
// block barriers and a serial thread-0 group pick (topk_gating.cu:244-388).
//
// Scores use exp evaluated in double precision and rounded once to fp32, then
// fp32 add and fp32 division: s = 1 / (1 + e^-x).  That is the exact formula
// of torch.sigmoid rounded at each fp32 step; it removes any dependence on a
// particular single-precision exp implementation.
#include <float.h>

#include <atomic>

#include "common.cuh"

namespace lsek {
namespace {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ float score_sigmoid(float x) {
  const float e = static_cast<float>(exp(-static_cast<double>(x)));
  return __frcp_rn(__fadd_rn(1.0f, e));  // the correctly rounded 1 / (1 + e)
}

// sqrt(softplus(x)) with torch's softplus threshold: x > 20 -> x, else
// log1p(exp(x)); each step rounded to fp32 as torch does.
__device__ __forceinline__ float score_sqrtsoftplus(float x) {
  if (x > 20.0f) return __fsqrt_rn(x);
  const float e = static_cast<float>(exp(static_cast<double>(x)));
  const float l = static_cast<float>(log1p(static_cast<double>(e)));
  return __fsqrt_rn(l);
}

// Maps fp32 to uint32 so that unsigned order equals float order
// (-inf < ... < -0 < +0 < ... < +inf).  Key 0 is reserved for "not a
// candidate" (no float maps below 0x007fffff).
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Merges another lane's (top1, top2) into ours; the result is the top-2 of
// the union as a multiset (the pair logic of grouped_topk_kernel,
// sm120/gating/topk_gating.cu:289-300).
__device__ __forceinline__ void merge_top2(float& t1, float& t2, float o1, float o2) {
  if (t1 >= o1) {
    t2 = (t2 >= o1) ? t2 : o1;
  } else {
    t2 = (o2 >= t1) ? o2 : t1;
    t1 = o1;
  }
}

// LPT lanes per token (32, or 16 so that one warp serves two tokens and
// every instruction of the selection rounds below works for both); lane l of
// a token's segment owns the EPL consecutive experts [l*EPL, (l+1)*EPL).
// Segment-wide reductions use the segment's lane mask, shuffles a width of
// LPT.  The token loop is uniform across the warp, so a segment whose token
// is past the end still takes part in every shuffle (on row 0's values) and
// only skips the stores.
template <int EPL, int LPT>
__global__ void __launch_bounds__(256, (LPT == 16 || EPL >= 16) ? (EPL >= 16 && LPT == 32 ? 1 : 2) : 3) topk_gating_kernel(
    float* __restrict__ out_w, int32_t* __restrict__ out_i,
    const float* __restrict__ logits, const float* __restrict__ bias, int T,
    int E, int topk, int n_group, int topk_group, float rsf, int renorm,
    int scoring, int vec_ok, int seg_lanes) {
  constexpr int TPW = 32 / LPT;  // tokens per warp
  extern __shared__ float s_group[];  // per token slot: sel values, padded 33/32 (general path)
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int warps_per_block = blockDim.x >> 5;
  const int sub = lane / LPT;  // token slot in the warp
  const int l = lane % LPT;    // lane in the token's segment
  const unsigned seg_mask = LPT == 32 ? kFull : (((1u << (LPT & 31)) - 1u) << (sub * LPT));
  const int pad_stride = E + (E >> 5) + 1;
  float* s_sel = s_group + (warp * TPW + sub) * pad_stride;
  const int e0 = l * EPL;
  const int epg = E / n_group;

  for (int wt = blockIdx.x * warps_per_block + warp; wt * TPW < T;
       wt += gridDim.x * warps_per_block) {
    const int t = wt * TPW + sub;
    const bool tok = t < T;
    const float* row = logits + static_cast<int64_t>(tok ? t : 0) * E;
    float x[EPL], bv[EPL];
    if (EPL >= 4 && vec_ok && e0 + EPL <= E) {
#pragma unroll
      for (int j = 0; j < EPL; j += 4) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(row + e0 + j));
        x[j] = v.x; x[j + 1] = v.y; x[j + 2] = v.z; x[j + 3] = v.w;
        const float4 b = bias != nullptr ? __ldg(reinterpret_cast<const float4*>(bias + e0 + j))
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
        bv[j] = b.x; bv[j + 1] = b.y; bv[j + 2] = b.z; bv[j + 3] = b.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < EPL; ++j) {
        const bool in = e0 + j < E;
        x[j] = in ? __ldg(row + e0 + j) : 0.0f;
        bv[j] = (in && bias != nullptr) ? __ldg(bias + e0 + j) : 0.0f;
      }
    }

    // x[] becomes the biased selection score; sc[] keeps the unbiased score.
    float sc[EPL];
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
      const int e = e0 + j;
      const float sv = scoring == LSEK_SCORING_SIGMOID ? score_sigmoid(x[j])
                                                       : score_sqrtsoftplus(x[j]);
      sc[j] = sv;
      x[j] = (e >= E) ? -INFINITY : (bias != nullptr ? __fadd_rn(sv, bv[j]) : sv);
    }
    uint32_t key[EPL];
#pragma unroll
    for (int j = 0; j < EPL; ++j) key[j] = (e0 + j < E) ? order_key(x[j]) : 0u;

    if (n_group > 1) {
      bool kept_mine[EPL];
      if (seg_lanes > 0) {
        // Each lane's experts lie in one group and a group spans seg_lanes
        // aligned lanes: top-2 by xor-shuffles inside the group.
        float t1 = -INFINITY, t2 = -INFINITY;
#pragma unroll
        for (int j = 0; j < EPL; ++j) merge_top2(t1, t2, x[j], -INFINITY);
        for (int off = 1; off < seg_lanes; off <<= 1) {
          const float o1 = __shfl_xor_sync(kFull, t1, off);
          const float o2 = __shfl_xor_sync(kFull, t2, off);
          merge_top2(t1, t2, o1, o2);
        }
        const float mine = (epg >= 2) ? __fadd_rn(t1, t2) : t1;
        const int g_me = l / seg_lanes;
        int rank = 0;
        for (int h = 0; h < n_group; ++h) {
          const float o = __shfl_sync(kFull, mine, h * seg_lanes, LPT);
          rank += (o > mine) || (o == mine && h < g_me);
        }
#pragma unroll
        for (int j = 0; j < EPL; ++j) kept_mine[j] = rank < topk_group;
      } else {
        // General layout: per-group scan through shared memory.
#pragma unroll
        for (int j = 0; j < EPL; ++j) {
          const int e = e0 + j;
          if (e < E) s_sel[e + (e >> 5)] = x[j];
        }
        __syncwarp();
        float gscore = 0.0f;
        if (l < n_group) {
          float t1 = -INFINITY, t2 = -INFINITY;
          const int gb = l * epg;
          for (int i = 0; i < epg; ++i) {
            const int e = gb + i;
            merge_top2(t1, t2, s_sel[e + (e >> 5)], -INFINITY);
          }
          gscore = (epg >= 2) ? __fadd_rn(t1, t2) : t1;
        }
        int rank = 0;
        for (int h = 0; h < n_group; ++h) {
          const float o = __shfl_sync(kFull, gscore, h, LPT);
          rank += (o > gscore) || (o == gscore && h < l);
        }
        const unsigned kept_all = __ballot_sync(kFull, l < n_group && rank < topk_group);
        const unsigned kept = LPT == 32 ? kept_all : (kept_all >> (sub * LPT));
#pragma unroll
        for (int j = 0; j < EPL; ++j) {
          const int e = e0 + j;
          kept_mine[j] = e < E && ((kept >> (e / epg)) & 1u);
        }
        __syncwarp();  // s_sel is rewritten by the next token
      }
#pragma unroll
      for (int j = 0; j < EPL; ++j)
        if (!kept_mine[j]) key[j] = 0u;
    }

    // Local best: highest key, lowest j on ties (lowest expert id).
    uint32_t bk = 0;
    int bj = -1;
#pragma unroll
    for (int j = 0; j < EPL; ++j)
      if (key[j] > bk) { bk = key[j]; bj = j; }

    float wsum = 0.0f;
    float my_w = 0.0f;
    int my_i = 0;
    for (int k = 0; k < topk; ++k) {
      // Segment arg-max: the highest key (one redux), and among the lanes
      // that hold it the lowest one, whose experts have the lowest ids (each
      // lane already keeps its lowest j on ties).
      const uint32_t kmax = __reduce_max_sync(seg_mask, bk);
      const unsigned hit = __ballot_sync(kFull, bk == kmax);
      const int owner = __ffs(LPT == 32 ? hit : (hit >> (sub * LPT)) & ((1u << (LPT & 31)) - 1u)) - 1;
      const int ie = owner * EPL + __shfl_sync(kFull, bj, owner, LPT);
      float mine = 0.0f;
#pragma unroll
      for (int j = 0; j < EPL; ++j)
        if (j == bj) mine = sc[j];
      const float wv = __shfl_sync(kFull, mine, owner, LPT);
      if (l == owner) {
#pragma unroll
        for (int j = 0; j < EPL; ++j)
          if (j == bj) key[j] = 0u;
        bk = 0;
        bj = -1;
#pragma unroll
        for (int j = 0; j < EPL; ++j)
          if (key[j] > bk) { bk = key[j]; bj = j; }
      }
      wsum = __fadd_rn(wsum, wv);
      if (l == k) { my_w = wv; my_i = ie; }
    }
    if (renorm && wsum > 0.0f) my_w = __fmul_rn(my_w, __fdiv_rn(rsf, wsum));
    if (tok && l < topk) {
      out_w[static_cast<int64_t>(t) * topk + l] = my_w;
      out_i[static_cast<int64_t>(t) * topk + l] = my_i;
    }
  }
}

template <int EPL, int LPT>
cudaError_t launch_topk(float* w, int32_t* idx, const float* logits,
                        const float* bias, const lsek_topk_gating_params& p,
                        int vec_ok, cudaStream_t st) {
  constexpr int TPW = 32 / LPT;
  const int threads = 256;
  const int warps = threads / 32;
  // Register path for groups: every lane's EPL experts in one group and a
  // group spanning a power-of-two number of whole lanes.
  int seg = 0;
  if (p.n_group > 1) {
    const int epg = p.num_experts / p.n_group;
    const int lanes = epg / EPL;
    if (p.num_experts == LPT * EPL && epg % EPL == 0 && lanes >= 1 && (lanes & (lanes - 1)) == 0)
      seg = lanes;
  }
  const size_t smem = (p.n_group > 1 && seg == 0)
                          ? static_cast<size_t>(warps) * TPW *
                                (p.num_experts + (p.num_experts >> 5) + 1) * sizeof(float)
                          : 0;
  // One wave of resident blocks at most: a token's latency chain is the
  // kernel's critical path, so no warp takes a second pair of tokens while
  // the SMs could hold more warps.  (The register-path occupancy is cached:
  // the query is a driver call.)
  static std::atomic<int> cached_per_sm{0};
  int per_sm = smem == 0 ? cached_per_sm.load(std::memory_order_relaxed) : 0;
  if (per_sm == 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, topk_gating_kernel<EPL, LPT>,
                                                      threads, smem) != cudaSuccess ||
        per_sm < 1) {
      cudaGetLastError();  // a failed query must not read as a failed launch
      per_sm = 1;
    }
    if (smem == 0) cached_per_sm.store(per_sm, std::memory_order_relaxed);
  }
  const int blocks_needed = static_cast<int>(ceil_div(ceil_div(p.num_tokens, TPW), warps));
  const int cap = num_sms() * per_sm;
  const int grid = blocks_needed < cap ? blocks_needed : cap;
  topk_gating_kernel<EPL, LPT><<<grid, threads, smem, st>>>(
      w, idx, logits, bias, p.num_tokens, p.num_experts, p.topk,
      p.n_group > 1 ? p.n_group : 1, p.topk_group, p.routed_scaling_factor,
      p.renormalize, p.scoring_func, vec_ok, seg);
  return cudaGetLastError();
}

// One thread per token.  Stable insertion sort by weight (descending), then
// the cumulative threshold scan of ref_adaptive_gating
// (tests/test_reference.py:190-225): the total is an fp32 sum, target and
// running sum are formed in double as the reference's Python loop does.
template <int KMAX>
__global__ void adaptive_gating_kernel(float* __restrict__ ow,
                                       int32_t* __restrict__ oi,
                                       int32_t* __restrict__ counts,
                                       const float* __restrict__ iw,
                                       const int32_t* __restrict__ ii, int T,
                                       int topk, double threshold) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  float w[KMAX];
  int32_t id[KMAX];
  const int64_t base = static_cast<int64_t>(t) * topk;
  for (int k = 0; k < topk; ++k) {
    const float wk = iw[base + k];
    const int32_t ik = ii[base + k];
    int j = k - 1;
    while (j >= 0 && w[j] < wk) {
      w[j + 1] = w[j];
      id[j + 1] = id[j];
      --j;
    }
    w[j + 1] = wk;
    id[j + 1] = ik;
  }
  float total = 0.0f;
  for (int k = 0; k < topk; ++k) total = __fadd_rn(total, w[k]);
  const double target = threshold * static_cast<double>(total);
  double cum = 0.0;
  int count = topk;
  for (int k = 0; k < topk; ++k) {
    cum += static_cast<double>(w[k]);
    if (cum >= target) {
      count = k + 1;
      break;
    }
  }
  if (count < 1) count = 1;
  for (int k = 0; k < topk; ++k) {
    ow[base + k] = k < count ? w[k] : 0.0f;
    oi[base + k] = k < count ? id[k] : -1;
  }
  counts[t] = count;
}

}  // namespace
}  // namespace lsek

extern "C" lsek_status lsek_topk_gating(float* topk_weights,
                                        int32_t* topk_indices,
                                        const float* logits, const float* bias,
                                        const lsek_topk_gating_params* params,
                                        void* stream) {
  using namespace lsek;
  LSEK_REQUIRE(params != nullptr, "topk_gating: params is NULL");
  const lsek_topk_gating_params& p = *params;
  LSEK_REQUIRE(p.num_tokens >= 0, "topk_gating: num_tokens must be >= 0");
  if (p.num_tokens == 0) return LSEK_OK;
  LSEK_REQUIRE(p.num_experts > 0, "topk_gating: num_experts must be > 0");
  LSEK_REQUIRE(p.topk >= 1 && p.topk <= p.num_experts,
               "topk_gating: topk must be in [1, num_experts]");
  LSEK_REQUIRE(p.n_group >= 1 && p.num_experts % p.n_group == 0,
               "topk_gating: num_experts must be divisible by n_group");
  if (p.n_group > 1) {
    LSEK_REQUIRE(p.topk_group >= 1 && p.topk_group <= p.n_group,
                 "topk_gating: topk_group must be in [1, n_group]");
    LSEK_REQUIRE(p.topk <= p.topk_group * (p.num_experts / p.n_group),
                 "topk_gating: topk (%d) exceeds the experts of the kept groups (%d)",
                 p.topk, p.topk_group * (p.num_experts / p.n_group));
    LSEK_REQUIRE(p.n_group <= 32, "topk_gating: n_group must be <= 32");
  }
  LSEK_REQUIRE(p.scoring_func == LSEK_SCORING_SIGMOID ||
                   p.scoring_func == LSEK_SCORING_SQRTSOFTPLUS,
               "topk_gating: scoring_func must be sigmoid (0) or sqrtsoftplus (1)");
  if (p.num_experts > 1024 || p.topk > 32)
    return fail(LSEK_ERR_UNSUPPORTED, "topk_gating: supports num_experts <= 1024 and topk <= 32");
  LSEK_REQUIRE(topk_weights && topk_indices && logits, "topk_gating: NULL tensor pointer");

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int vec_ok = (p.num_experts % 4 == 0) &&
                     (reinterpret_cast<uintptr_t>(logits) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(bias) % 16 == 0);
  // Two tokens per warp (16 lanes each) when a token's experts, selections
  // and groups fit in 16 lanes at no more than 8 experts a lane; else one
  // token per warp.  (At E=256, 16 experts a lane doubled the registers and
  // the unrolled code and measured 22 us against 14 us for one token per
  // warp, the same instruction count at half the resident warps.)
  const bool half = p.num_experts <= 128 && p.topk <= 16 && p.n_group <= 16;
  cudaError_t e;
  if (half) {
    const int epl = static_cast<int>(ceil_div(p.num_experts, 16));
    if (epl <= 1)      e = launch_topk<1, 16>(topk_weights, topk_indices, logits, bias, p, vec_ok, st);
    else if (epl <= 2) e = launch_topk<2, 16>(topk_weights, topk_indices, logits, bias, p, vec_ok, st);
    else if (epl <= 4) e = launch_topk<4, 16>(topk_weights, topk_indices, logits, bias, p, vec_ok, st);
    else               e = launch_topk<8, 16>(topk_weights, topk_indices, logits, bias, p, vec_ok, st);
  } else {
    const int epl = static_cast<int>(ceil_div(p.num_experts, 32));
    if (epl <= 1)       e = launch_topk<1, 32>(topk_weights, topk_indices, logits, bias, p, vec_ok, st);
    else if (epl <= 2)  e = launch_topk<2, 32>(topk_weights, topk_indices, logits, bias, p, vec_ok, st);
    else if (epl <= 4)  e = launch_topk<4, 32>(topk_weights, topk_indices, logits, bias, p, vec_ok, st);
    else if (epl <= 8)  e = launch_topk<8, 32>(topk_weights, topk_indices, logits, bias, p, vec_ok, st);
    else if (epl <= 16) e = launch_topk<16, 32>(topk_weights, topk_indices, logits, bias, p, vec_ok, st);
    else                e = launch_topk<32, 32>(topk_weights, topk_indices, logits, bias, p, vec_ok, st);
  }
  if (e != cudaSuccess) return fail(LSEK_ERR_CUDA, "topk_gating: %s", cudaGetErrorString(e));
  return LSEK_OK;
}

extern "C" lsek_status lsek_adaptive_gating(float* out_weights,
                                            int32_t* out_indices,
                                            int32_t* expert_counts,
                                            const float* in_weights,
                                            const int32_t* in_indices,
                                            int32_t num_tokens, int32_t topk,
                                            double threshold, void* stream) {
  using namespace lsek;
  LSEK_REQUIRE(num_tokens >= 0, "adaptive_gating: num_tokens must be >= 0");
  if (num_tokens == 0) return LSEK_OK;
  LSEK_REQUIRE(topk >= 1 && topk <= 32, "adaptive_gating: topk must be in [1, 32]");
  LSEK_REQUIRE(threshold >= 0.0 && threshold <= 1.0,
               "adaptive_gating: threshold must be in [0.0, 1.0]");
  LSEK_REQUIRE(out_weights && out_indices && expert_counts && in_weights && in_indices,
               "adaptive_gating: NULL tensor pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int threads = 128;
  const int grid = static_cast<int>(ceil_div(num_tokens, threads));
  if (topk <= 8)
    adaptive_gating_kernel<8><<<grid, threads, 0, st>>>(out_weights, out_indices, expert_counts,
                                                         in_weights, in_indices, num_tokens, topk,
                                                         threshold);
  else
    adaptive_gating_kernel<32><<<grid, threads, 0, st>>>(out_weights, out_indices, expert_counts,
                                                          in_weights, in_indices, num_tokens, topk,
                                                          threshold);
  return check_launch("adaptive_gating");
}
