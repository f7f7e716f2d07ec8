// Whole routed-expert layer on one stream: gating -> route -> row copy into
// expert order (folded into the GEMM's own TMA loads for small T) -> gate/up
// GEMM with SwiGLU epilogue -> down GEMM -> weighted unpermute.
// The composition is the reference's documented expert flow (USAGE.md:40-57);
// ref_expert_forward (tests/test_reference.py:257-276) is its oracle for
// top-1, generalised here to top-k slots.
//
// Workspace layout (each piece 256-byte aligned):
//   weights f32 [T*k] | indices i32 [T*k] | offsets i32 [E+1] | s2d i32 [T*k]
//   | perm i32 [T*k] | route scratch | GEMM unit counter | X [T*k, H] bf16 (reused for the down
//   GEMM output Y, which is written only after the gate/up GEMM has consumed
//   X on the same stream) | Hact [T*k, I] bf16
#include "common.cuh"

namespace lsek {
size_t permute_workspace_bytes(int64_t n_keys, int num_experts);
lsek_status launch_route(const int32_t* idx, int64_t n, int E, int32_t* offsets, int32_t* s2d,
                         int32_t* perm, void* ws, cudaStream_t st);
lsek_status launch_route_by_expert(const int32_t* idx, int64_t n, int E, int32_t* offsets,
                                   int32_t* s2d, int32_t* perm, cudaStream_t st);
lsek_status grouped_gemm_plain(void* D, const void* A, const void* B, const int32_t* offsets,
                               int E, int rows, int N, int K, int32_t* counter, cudaStream_t st,
                               int max_rows_per_expert);
lsek_status grouped_gemm_swiglu(void* H, const void* A, const void* Wgu, const int32_t* offsets,
                                int E, int rows, int I, int K, float limit, int32_t* counter,
                                cudaStream_t st, int max_rows_per_expert);
lsek_status launch_permute_rows(void* dst, const void* src, const int32_t* s2d, int64_t T,
                                int topk, int64_t row_bytes, cudaStream_t st);
lsek_status grouped_gemm_swiglu_gather(void* H, const void* hidden, const void* Wgu,
                                       const int32_t* offsets, const int32_t* permuted_idx,
                                       int num_tokens, int topk, int E, int rows, int I, int K,
                                       float limit, int32_t* counter, cudaStream_t st,
                                       int max_rows_per_expert);

namespace {
struct LayerWs {
  size_t w, idx, offs, s2d, perm, route, sched, x, h, total;
};
size_t a256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }
LayerWs layer_ws(int64_t T, int64_t H, int64_t I, int64_t E, int64_t k) {
  LayerWs l;
  const int64_t n = T * k;
  size_t o = 0;
  l.w = o;     o += a256(n * 4);
  l.idx = o;   o += a256(n * 4);
  l.offs = o;  o += a256((E + 1) * 4);
  l.s2d = o;   o += a256(n * 4);
  l.perm = o;  o += a256(n * 4);
  l.route = o; o += a256(permute_workspace_bytes(n, static_cast<int>(E)));
  l.sched = o; o += 256;
  l.x = o;     o += a256(n * H * 2);
  l.h = o;     o += a256(n * I * 2);
  l.total = o;
  return l;
}
}  // namespace
}  // namespace lsek

extern "C" lsek_status lsek_moe_unpermute(void* output, const void* permuted_output,
                                          const float* topk_weights,
                                          const int32_t* src_to_dest_map, int32_t num_tokens,
                                          int32_t topk, int32_t hidden_dim, int32_t dtype,
                                          int32_t fp32_output, void* stream);

extern "C" size_t lsek_moe_layer_workspace_size(int32_t num_tokens, int32_t hidden_dim,
                                                int32_t inter_dim, int32_t num_experts,
                                                int32_t topk) {
  if (num_tokens < 0 || hidden_dim < 0 || inter_dim < 0 || num_experts < 0 || topk < 0) return 0;
  return lsek::layer_ws(num_tokens, hidden_dim, inter_dim, num_experts, topk).total;
}

extern "C" lsek_status lsek_moe_layer_forward(
    void* out, const void* hidden, const float* logits, const float* bias, const void* W_gu,
    const void* W_down, const lsek_topk_gating_params* gp, int32_t hidden_dim, int32_t inter_dim,
    float swiglu_limit, float* topk_weights, int32_t* topk_indices, void* workspace,
    size_t workspace_bytes, void* const* stage_events, void* stream) {
  using namespace lsek;
  LSEK_REQUIRE(gp != nullptr, "moe_layer_forward: gating params are NULL");
  const int T = gp->num_tokens, E = gp->num_experts, k = gp->topk;
  LSEK_REQUIRE(T >= 0 && hidden_dim > 0 && inter_dim > 0,
               "moe_layer_forward: num_tokens >= 0, hidden_dim > 0, inter_dim > 0 required");
  LSEK_REQUIRE(swiglu_limit >= 0.0f, "moe_layer_forward: swiglu_limit must be >= 0");
  if (T == 0) return LSEK_OK;
  LSEK_REQUIRE(hidden_dim % 32 == 0 && inter_dim % 32 == 0,
               "moe_layer_forward: hidden_dim and inter_dim must be multiples of 32");
  LSEK_REQUIRE(out && hidden && logits && W_gu && W_down, "moe_layer_forward: NULL tensor pointer");
  LSEK_REQUIRE(reinterpret_cast<uintptr_t>(hidden) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(W_gu) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(W_down) % 16 == 0,
               "moe_layer_forward: hidden, W_gu and W_down must be 16-byte aligned");
  LSEK_REQUIRE(static_cast<int64_t>(T) * k < (1ll << 31), "moe_layer_forward: T*topk too large");
  const LayerWs l = layer_ws(T, hidden_dim, inter_dim, E, k);
  LSEK_REQUIRE(workspace != nullptr && workspace_bytes >= l.total,
               "moe_layer_forward: workspace of %zu bytes required, got %zu", l.total,
               workspace_bytes);
  LSEK_REQUIRE(reinterpret_cast<uintptr_t>(workspace) % 256 == 0,
               "moe_layer_forward: workspace must be 256-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  float* w = topk_weights ? topk_weights : reinterpret_cast<float*>(ws + l.w);
  int32_t* idx = topk_indices ? topk_indices : reinterpret_cast<int32_t*>(ws + l.idx);
  int32_t* offs = reinterpret_cast<int32_t*>(ws + l.offs);
  int32_t* s2d = reinterpret_cast<int32_t*>(ws + l.s2d);
  int32_t* perm = reinterpret_cast<int32_t*>(ws + l.perm);
  int32_t* counter = reinterpret_cast<int32_t*>(ws + l.sched);
  void* x = ws + l.x;
  void* h = ws + l.h;
  const int64_t n = static_cast<int64_t>(T) * k;
  if (E > 1023) return fail(LSEK_ERR_UNSUPPORTED, "moe_layer_forward: num_experts must be <= 1023");
  auto mark = [&](int i) -> lsek_status {
    if (stage_events != nullptr && stage_events[i] != nullptr)
      LSEK_CUDA_TRY(cudaEventRecord(static_cast<cudaEvent_t>(stage_events[i]), st));
    return LSEK_OK;
  };
  lsek_status s;
  if ((s = mark(0)) != LSEK_OK) return s;
  if ((s = lsek_topk_gating(w, idx, logits, bias, gp, stream)) != LSEK_OK) return s;
  if ((s = mark(1)) != LSEK_OK) return s;
  if ((s = launch_route_by_expert(idx, n, E, offs, s2d, perm, st)) != LSEK_OK) return s;
  // The top-k experts of a token are distinct, so no expert gets more than T
  // rows.  Up to kGatherMaxTokens tokens every tile is a small one, and the
  // permute is folded into the gate/up GEMM's A load (a tile's few token rows
  // gathered from `hidden` through permuted_idx, four per TMA gather), which
  // saves the row-copy launch; above it the row copy feeds whole 128-row
  // tiles to tiled TMA loads (gathering 128 rows per k-block costs the TMA
  // unit more than the copy saves).
  constexpr int kGatherMaxTokens = 64;
  const bool gather = T <= kGatherMaxTokens;
  if ((s = mark(2)) != LSEK_OK) return s;
  if (!gather) {
    s = launch_permute_rows(x, hidden, s2d, T, k, static_cast<int64_t>(hidden_dim) * 2, st);
    if (s != LSEK_OK) return s;
  }
  if ((s = mark(3)) != LSEK_OK) return s;
  if (gather)
    s = grouped_gemm_swiglu_gather(h, hidden, W_gu, offs, perm, T, k, E, static_cast<int>(n),
                                   inter_dim, hidden_dim, swiglu_limit, counter, st, T);
  else
    s = grouped_gemm_swiglu(h, x, W_gu, offs, E, static_cast<int>(n), inter_dim, hidden_dim,
                            swiglu_limit, counter, st, T);
  if (s != LSEK_OK) return s;
  if ((s = mark(4)) != LSEK_OK) return s;
  s = grouped_gemm_plain(x, h, W_down, offs, E, static_cast<int>(n), hidden_dim, inter_dim,
                         counter, st, T);
  if (s != LSEK_OK) return s;
  if ((s = mark(5)) != LSEK_OK) return s;
  s = lsek_moe_unpermute(out, x, w, s2d, T, k, hidden_dim, LSEK_BF16, 0, stream);
  if (s != LSEK_OK) return s;
  return mark(6);
}
