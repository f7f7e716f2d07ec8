// Torch binding of liblsek: the operator surface of the reference extension
// `sm120_expert_kernels` (csrc/bindings_python.cu:371-417) with the same op
// names, argument names, defaults, dtypes, shapes and return tuples, plus the
// expert-contraction and whole-layer ops the reference documents but does not
// ship.  Every op checks its tensors, allocates outputs with the caching
// allocator, and calls the C ABI of include/lsek.h on the current stream of
// the input's device (a device guard makes that device current).  Status
// INVALID_ARG raises ValueError, every other failure RuntimeError, as the
// reference's launchers do via pybind11's exception translation.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime_api.h>
#include <pybind11/stl.h>
#include <torch/extension.h>

#include <string>
#include <vector>

#include "lsek.h"

namespace {

void* stream_of(const torch::Tensor& t) {
  return static_cast<void*>(at::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

void check_status(lsek_status s) {
  if (s == LSEK_OK) return;
  const std::string msg = lsek_last_error();
  if (s == LSEK_ERR_INVALID_ARG) throw pybind11::value_error(msg);
  throw std::runtime_error(msg);
}

int32_t dtype_code(const torch::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kBFloat16: return LSEK_BF16;
    case at::kHalf: return LSEK_FP16;
    case at::kFloat: return LSEK_FP32;
    default: return -1;
  }
}

int32_t to_i32(int64_t v, const char* what) {
  TORCH_CHECK(v >= 0 && v <= INT32_MAX, what, " out of range: ", v);
  return static_cast<int32_t>(v);
}

// ---- reference op surface -------------------------------------------------------

torch::Tensor fused_swiglu(torch::Tensor input, double swiglu_limit) {
  TORCH_CHECK(input.is_cuda(), "fused_swiglu: input must be on CUDA");
  TORCH_CHECK(input.is_contiguous(), "fused_swiglu: input must be contiguous");
  TORCH_CHECK(input.dim() == 2, "fused_swiglu: input must be 2D [num_tokens, 2*d]");
  TORCH_CHECK(input.size(1) % 2 == 0, "fused_swiglu: last dim must be even (gate|up interleaved)");
  TORCH_CHECK(input.scalar_type() == at::kBFloat16 || input.scalar_type() == at::kHalf,
              "fused_swiglu: input must be BF16 or FP16");
  TORCH_CHECK(swiglu_limit >= 0.0, "fused_swiglu: swiglu_limit must be >= 0 (0 = no clamp)");
  const c10::cuda::OptionalCUDAGuard guard(input.device());
  const int64_t n = input.size(0), d = input.size(1) / 2;
  auto out = torch::empty({n, d}, input.options());
  check_status(lsek_fused_swiglu(out.data_ptr(), input.data_ptr(), to_i32(n, "num_tokens"),
                                 to_i32(d, "d"), static_cast<float>(swiglu_limit),
                                 dtype_code(input), stream_of(input)));
  return out;
}

std::vector<torch::Tensor> moe_permute(torch::Tensor hidden_states, torch::Tensor topk_indices,
                                       int64_t num_experts) {
  TORCH_CHECK(hidden_states.is_cuda(), "moe_permute: hidden_states must be on CUDA");
  TORCH_CHECK(topk_indices.is_cuda(), "moe_permute: topk_indices must be on CUDA");
  TORCH_CHECK(hidden_states.is_contiguous(), "moe_permute: hidden_states must be contiguous");
  TORCH_CHECK(topk_indices.is_contiguous(), "moe_permute: topk_indices must be contiguous");
  TORCH_CHECK(hidden_states.dim() == 2, "moe_permute: hidden_states must be 2D");
  TORCH_CHECK(topk_indices.dim() == 2, "moe_permute: topk_indices must be 2D [num_tokens, topk]");
  TORCH_CHECK(topk_indices.scalar_type() == at::kInt, "moe_permute: topk_indices must be int32");
  TORCH_CHECK(topk_indices.size(0) == hidden_states.size(0),
              "moe_permute: topk_indices and hidden_states disagree on num_tokens");
  const c10::cuda::OptionalCUDAGuard guard(hidden_states.device());
  const int64_t T = hidden_states.size(0), H = hidden_states.size(1), k = topk_indices.size(1);
  const int64_t n = T * k;
  auto permuted = torch::empty({n, H}, hidden_states.options());
  auto offsets = torch::empty({num_experts + 1}, topk_indices.options());
  auto s2d = torch::empty({n}, topk_indices.options());
  auto perm = torch::empty({n}, topk_indices.options());
  const size_t ws_bytes = lsek_moe_permute_workspace_size(to_i32(T, "num_tokens"), to_i32(k, "topk"),
                                                          to_i32(num_experts, "num_experts"));
  auto ws = torch::empty({static_cast<int64_t>(ws_bytes)}, hidden_states.options().dtype(at::kByte));
  check_status(lsek_moe_permute(permuted.data_ptr(), offsets.data_ptr<int32_t>(),
                                s2d.data_ptr<int32_t>(), perm.data_ptr<int32_t>(),
                                hidden_states.data_ptr(), topk_indices.data_ptr<int32_t>(),
                                static_cast<int32_t>(T), static_cast<int32_t>(k),
                                to_i32(H, "hidden_dim"), static_cast<int32_t>(num_experts),
                                static_cast<int32_t>(hidden_states.element_size()), ws.data_ptr(),
                                ws_bytes, stream_of(hidden_states)));
  return {permuted, offsets, s2d, perm};
}

// Routing only (lsek_moe_route): [expert_offsets int32[E+1], src_to_dest_map
// int32[T*k], permuted_idx int32[T*k]], the maps moe_permute returns.
std::vector<torch::Tensor> moe_route(torch::Tensor topk_indices, int64_t num_experts) {
  TORCH_CHECK(topk_indices.is_cuda(), "moe_route: topk_indices must be on CUDA");
  TORCH_CHECK(topk_indices.is_contiguous(), "moe_route: topk_indices must be contiguous");
  TORCH_CHECK(topk_indices.dim() == 2, "moe_route: topk_indices must be 2D [num_tokens, topk]");
  TORCH_CHECK(topk_indices.scalar_type() == at::kInt, "moe_route: topk_indices must be int32");
  const c10::cuda::OptionalCUDAGuard guard(topk_indices.device());
  const int64_t T = topk_indices.size(0), k = topk_indices.size(1);
  auto offsets = torch::empty({num_experts + 1}, topk_indices.options());
  auto s2d = torch::empty({T * k}, topk_indices.options());
  auto perm = torch::empty({T * k}, topk_indices.options());
  check_status(lsek_moe_route(offsets.data_ptr<int32_t>(), s2d.data_ptr<int32_t>(),
                              perm.data_ptr<int32_t>(), topk_indices.data_ptr<int32_t>(),
                              to_i32(T, "num_tokens"), to_i32(k, "topk"),
                              to_i32(num_experts, "num_experts"), stream_of(topk_indices)));
  return {offsets, s2d, perm};
}

void check_unpermute_args(const char* op, const torch::Tensor& permuted_output,
                          const torch::Tensor& topk_weights, const torch::Tensor& s2d,
                          int64_t num_tokens, int64_t topk) {
  TORCH_CHECK(permuted_output.is_cuda(), op, ": permuted_output must be on CUDA");
  TORCH_CHECK(topk_weights.is_cuda(), op, ": topk_weights must be on CUDA");
  TORCH_CHECK(s2d.is_cuda(), op, ": src_to_dest_map must be on CUDA");
  TORCH_CHECK(permuted_output.is_contiguous(), op, ": permuted_output must be contiguous");
  TORCH_CHECK(topk_weights.is_contiguous() && s2d.is_contiguous(), op,
              ": topk_weights and src_to_dest_map must be contiguous");
  TORCH_CHECK(topk_weights.scalar_type() == at::kFloat, op, ": topk_weights must be float32");
  TORCH_CHECK(s2d.scalar_type() == at::kInt, op, ": src_to_dest_map must be int32");
  TORCH_CHECK(permuted_output.dim() == 2, op, ": permuted_output must be 2D");
  TORCH_CHECK(permuted_output.scalar_type() == at::kBFloat16 ||
                  permuted_output.scalar_type() == at::kHalf,
              op, ": permuted_output must be bf16/fp16 (2 bytes)");
  TORCH_CHECK(topk_weights.numel() == num_tokens * topk && s2d.numel() == num_tokens * topk, op,
              ": topk_weights and src_to_dest_map must hold num_tokens * topk entries");
}

torch::Tensor moe_unpermute(torch::Tensor permuted_output, torch::Tensor topk_weights,
                            torch::Tensor src_to_dest_map, int64_t num_tokens, int64_t topk) {
  check_unpermute_args("moe_unpermute", permuted_output, topk_weights, src_to_dest_map,
                       num_tokens, topk);
  const c10::cuda::OptionalCUDAGuard guard(permuted_output.device());
  const int64_t H = permuted_output.size(1);
  auto out = torch::empty({num_tokens, H}, permuted_output.options());
  check_status(lsek_moe_unpermute(out.data_ptr(), permuted_output.data_ptr(),
                                  topk_weights.data_ptr<float>(), src_to_dest_map.data_ptr<int32_t>(),
                                  to_i32(num_tokens, "num_tokens"), to_i32(topk, "topk"),
                                  to_i32(H, "hidden_dim"), dtype_code(permuted_output), 0,
                                  stream_of(permuted_output)));
  return out;
}

torch::Tensor moe_unpermute_fp32(torch::Tensor permuted_output, torch::Tensor topk_weights,
                                 torch::Tensor src_to_dest_map, int64_t num_tokens, int64_t topk) {
  check_unpermute_args("moe_unpermute_fp32", permuted_output, topk_weights, src_to_dest_map,
                       num_tokens, topk);
  const c10::cuda::OptionalCUDAGuard guard(permuted_output.device());
  const int64_t H = permuted_output.size(1);
  auto out = torch::empty({num_tokens, topk, H}, permuted_output.options().dtype(at::kFloat));
  check_status(lsek_moe_unpermute(out.data_ptr(), permuted_output.data_ptr(),
                                  topk_weights.data_ptr<float>(), src_to_dest_map.data_ptr<int32_t>(),
                                  to_i32(num_tokens, "num_tokens"), to_i32(topk, "topk"),
                                  to_i32(H, "hidden_dim"), dtype_code(permuted_output), 1,
                                  stream_of(permuted_output)));
  return out;
}

torch::Tensor moe_unpermute_bf16_perslot(torch::Tensor permuted_output, torch::Tensor topk_weights,
                                         torch::Tensor src_to_dest_map, int64_t num_tokens,
                                         int64_t topk) {
  check_unpermute_args("moe_unpermute_bf16_perslot", permuted_output, topk_weights,
                       src_to_dest_map, num_tokens, topk);
  const c10::cuda::OptionalCUDAGuard guard(permuted_output.device());
  const int64_t H = permuted_output.size(1);
  auto out = torch::empty({num_tokens, topk, H}, permuted_output.options());
  check_status(lsek_moe_unpermute_perslot(
      out.data_ptr(), permuted_output.data_ptr(), topk_weights.data_ptr<float>(),
      src_to_dest_map.data_ptr<int32_t>(), to_i32(num_tokens, "num_tokens"), to_i32(topk, "topk"),
      to_i32(H, "hidden_dim"), dtype_code(permuted_output), stream_of(permuted_output)));
  return out;
}

torch::Tensor reduce_slots(const char* op, const torch::Tensor& in, at::ScalarType want) {
  TORCH_CHECK(in.is_cuda(), op, ": input must be on CUDA");
  TORCH_CHECK(in.is_contiguous(), op, ": input must be contiguous");
  TORCH_CHECK(in.scalar_type() == want, op, ": input must be ",
              want == at::kFloat ? "float32" : "bfloat16");
  TORCH_CHECK(in.dim() == 3, op, ": input must be [num_tokens, topk, hidden]");
  const c10::cuda::OptionalCUDAGuard guard(in.device());
  auto out = torch::empty({in.size(0), in.size(2)}, in.options().dtype(at::kBFloat16));
  check_status(lsek_moe_combine_reduce_slots(out.data_ptr(), in.data_ptr(),
                                             to_i32(in.size(0), "num_tokens"),
                                             to_i32(in.size(1), "topk"),
                                             to_i32(in.size(2), "hidden_dim"),
                                             want == at::kFloat ? LSEK_FP32 : LSEK_BF16,
                                             stream_of(in)));
  return out;
}

torch::Tensor moe_combine_reduce_slots_fp32_to_bf16(torch::Tensor input_perslot_fp32) {
  return reduce_slots("moe_combine_reduce", input_perslot_fp32, at::kFloat);
}

torch::Tensor moe_combine_reduce_slots_bf16_to_bf16(torch::Tensor input_perslot_bf16) {
  return reduce_slots("moe_combine_reduce_bf16", input_perslot_bf16, at::kBFloat16);
}

std::vector<torch::Tensor> adaptive_gating(torch::Tensor in_weights, torch::Tensor in_indices,
                                           double threshold) {
  TORCH_CHECK(in_weights.is_cuda(), "adaptive_gating: in_weights must be on CUDA");
  TORCH_CHECK(in_indices.is_cuda(), "adaptive_gating: in_indices must be on CUDA");
  TORCH_CHECK(in_weights.is_contiguous() && in_indices.is_contiguous(),
              "adaptive_gating: inputs must be contiguous");
  TORCH_CHECK(in_weights.scalar_type() == at::kFloat, "adaptive_gating: in_weights must be float32");
  TORCH_CHECK(in_indices.scalar_type() == at::kInt, "adaptive_gating: in_indices must be int32");
  TORCH_CHECK(in_weights.dim() == 2, "adaptive_gating: in_weights must be 2D");
  TORCH_CHECK(in_indices.sizes() == in_weights.sizes(),
              "adaptive_gating: in_indices must match in_weights in shape");
  const c10::cuda::OptionalCUDAGuard guard(in_weights.device());
  auto ow = torch::empty_like(in_weights);
  auto oi = torch::empty_like(in_indices);
  auto counts = torch::empty({in_weights.size(0)}, in_indices.options());
  check_status(lsek_adaptive_gating(ow.data_ptr<float>(), oi.data_ptr<int32_t>(),
                                    counts.data_ptr<int32_t>(), in_weights.data_ptr<float>(),
                                    in_indices.data_ptr<int32_t>(),
                                    to_i32(in_weights.size(0), "num_tokens"),
                                    to_i32(in_weights.size(1), "topk"), threshold,
                                    stream_of(in_weights)));
  return {ow, oi, counts};
}

int32_t scoring_code(const std::string& scoring_func) {
  if (scoring_func == "sigmoid") return LSEK_SCORING_SIGMOID;
  if (scoring_func == "sqrtsoftplus") return LSEK_SCORING_SQRTSOFTPLUS;
  TORCH_CHECK(false, "topk_gating: scoring_func must be 'sigmoid' or 'sqrtsoftplus', got '",
              scoring_func, "'");
  return -1;
}

const float* bias_ptr(const c10::optional<torch::Tensor>& bias, int64_t E) {
  if (!bias.has_value()) return nullptr;
  TORCH_CHECK(bias->is_cuda(), "topk_gating: bias must be on CUDA");
  TORCH_CHECK(bias->is_contiguous(), "topk_gating: bias must be contiguous");
  TORCH_CHECK(bias->scalar_type() == at::kFloat, "topk_gating: bias must be float32");
  TORCH_CHECK(bias->numel() == E, "topk_gating: bias must hold num_experts values");
  return bias->data_ptr<float>();
}

std::vector<torch::Tensor> topk_gating(torch::Tensor logits, c10::optional<torch::Tensor> bias,
                                       int64_t topk, int64_t n_group, int64_t topk_group,
                                       double routed_scaling_factor, bool renormalize,
                                       std::string scoring_func) {
  TORCH_CHECK(logits.is_cuda(), "topk_gating: logits must be on CUDA");
  TORCH_CHECK(logits.is_contiguous(), "topk_gating: logits must be contiguous");
  TORCH_CHECK(logits.scalar_type() == at::kFloat, "topk_gating: logits must be float32");
  TORCH_CHECK(logits.dim() == 2, "topk_gating: logits must be 2D [num_tokens, num_experts]");
  const int32_t sf = scoring_code(scoring_func);
  const c10::cuda::OptionalCUDAGuard guard(logits.device());
  const int64_t T = logits.size(0), E = logits.size(1);
  TORCH_CHECK(topk >= 0, "topk_gating: topk must be >= 0");
  auto w = torch::empty({T, topk}, logits.options());
  auto idx = torch::empty({T, topk}, logits.options().dtype(at::kInt));
  lsek_topk_gating_params p;
  p.num_tokens = to_i32(T, "num_tokens");
  p.num_experts = to_i32(E, "num_experts");
  p.topk = static_cast<int32_t>(topk);
  p.n_group = static_cast<int32_t>(n_group);
  p.topk_group = static_cast<int32_t>(topk_group);
  p.routed_scaling_factor = static_cast<float>(routed_scaling_factor);
  p.renormalize = renormalize ? 1 : 0;
  p.scoring_func = sf;
  check_status(lsek_topk_gating(w.data_ptr<float>(), idx.data_ptr<int32_t>(),
                                logits.data_ptr<float>(), bias_ptr(bias, E), &p, stream_of(logits)));
  return {w, idx};
}

// ---- expert contraction and whole layer -----------------------------------------------

void check_gemm_args(const char* op, const torch::Tensor& A, const torch::Tensor& W,
                     const torch::Tensor& offsets) {
  TORCH_CHECK(A.is_cuda() && W.is_cuda() && offsets.is_cuda(), op, ": tensors must be on CUDA");
  TORCH_CHECK(A.is_contiguous() && W.is_contiguous() && offsets.is_contiguous(), op,
              ": tensors must be contiguous");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && W.scalar_type() == at::kBFloat16, op,
              ": A and the weights must be bfloat16");
  TORCH_CHECK(offsets.scalar_type() == at::kInt, op, ": expert_offsets must be int32");
  TORCH_CHECK(A.dim() == 2 && W.dim() == 3, op, ": A must be [rows, K], weights [E, N, K]");
  TORCH_CHECK(W.size(2) == A.size(1), op, ": A and the weights disagree on K");
  TORCH_CHECK(offsets.numel() == W.size(0) + 1, op, ": expert_offsets must hold E+1 entries");
}

// Writes D[rows of the experts in expert_offsets]; other rows of D are left
// as they are, so experts can be computed in chunks into one buffer.
void grouped_gemm_bf16_out(torch::Tensor D, torch::Tensor A, torch::Tensor B,
                           torch::Tensor expert_offsets) {
  check_gemm_args("grouped_gemm_bf16_out", A, B, expert_offsets);
  TORCH_CHECK(D.is_cuda() && D.is_contiguous() && D.scalar_type() == at::kBFloat16 &&
                  D.dim() == 2 && D.size(0) == A.size(0) && D.size(1) == B.size(1),
              "grouped_gemm_bf16_out: D must be a contiguous bf16 CUDA tensor [rows, N]");
  const c10::cuda::OptionalCUDAGuard guard(A.device());
  auto ws = torch::empty({LSEK_GEMM_WORKSPACE_BYTES}, A.options().dtype(at::kByte));
  check_status(lsek_grouped_gemm_bf16(D.data_ptr(), A.data_ptr(), B.data_ptr(),
                                      expert_offsets.data_ptr<int32_t>(), to_i32(B.size(0), "E"),
                                      to_i32(A.size(0), "rows"), to_i32(B.size(1), "N"),
                                      to_i32(A.size(1), "K"), ws.data_ptr(),
                                      LSEK_GEMM_WORKSPACE_BYTES, stream_of(A)));
}

torch::Tensor grouped_gemm_bf16(torch::Tensor A, torch::Tensor B, torch::Tensor expert_offsets) {
  check_gemm_args("grouped_gemm_bf16", A, B, expert_offsets);
  const c10::cuda::OptionalCUDAGuard guard(A.device());
  auto D = torch::empty({A.size(0), B.size(1)}, A.options());
  auto ws = torch::empty({LSEK_GEMM_WORKSPACE_BYTES}, A.options().dtype(at::kByte));
  check_status(lsek_grouped_gemm_bf16(D.data_ptr(), A.data_ptr(), B.data_ptr(),
                                      expert_offsets.data_ptr<int32_t>(), to_i32(B.size(0), "E"),
                                      to_i32(A.size(0), "rows"), to_i32(B.size(1), "N"),
                                      to_i32(A.size(1), "K"), ws.data_ptr(),
                                      LSEK_GEMM_WORKSPACE_BYTES, stream_of(A)));
  return D;
}

torch::Tensor grouped_gemm_swiglu_bf16(torch::Tensor A, torch::Tensor W_gu,
                                       torch::Tensor expert_offsets, double swiglu_limit) {
  check_gemm_args("grouped_gemm_swiglu_bf16", A, W_gu, expert_offsets);
  TORCH_CHECK(W_gu.size(1) % 2 == 0, "grouped_gemm_swiglu_bf16: W_gu rows must be 2*I");
  const c10::cuda::OptionalCUDAGuard guard(A.device());
  const int64_t I = W_gu.size(1) / 2;
  auto H = torch::empty({A.size(0), I}, A.options());
  auto ws = torch::empty({LSEK_GEMM_WORKSPACE_BYTES}, A.options().dtype(at::kByte));
  check_status(lsek_grouped_gemm_swiglu_bf16(
      H.data_ptr(), A.data_ptr(), W_gu.data_ptr(), expert_offsets.data_ptr<int32_t>(),
      to_i32(W_gu.size(0), "E"), to_i32(A.size(0), "rows"), to_i32(I, "I"), to_i32(A.size(1), "K"),
      static_cast<float>(swiglu_limit), ws.data_ptr(), LSEK_GEMM_WORKSPACE_BYTES, stream_of(A)));
  return H;
}

int64_t moe_layer_workspace_size(int64_t num_tokens, int64_t hidden_dim, int64_t inter_dim,
                                 int64_t num_experts, int64_t topk) {
  return static_cast<int64_t>(lsek_moe_layer_workspace_size(
      to_i32(num_tokens, "num_tokens"), to_i32(hidden_dim, "hidden_dim"),
      to_i32(inter_dim, "inter_dim"), to_i32(num_experts, "num_experts"), to_i32(topk, "topk")));
}

// Fills `out` [T,H]; the routing lands in topk_weights / topk_indices when
// they are defined.  `workspace` is a uint8 CUDA tensor of at least
// moe_layer_workspace_size bytes.
void moe_layer_forward_out(torch::Tensor out, torch::Tensor hidden, torch::Tensor logits,
                           c10::optional<torch::Tensor> bias, torch::Tensor w_gu,
                           torch::Tensor w_down, int64_t topk, int64_t n_group,
                           int64_t topk_group, double routed_scaling_factor, bool renormalize,
                           std::string scoring_func, double swiglu_limit,
                           torch::Tensor workspace, c10::optional<torch::Tensor> topk_weights,
                           c10::optional<torch::Tensor> topk_indices,
                           std::vector<int64_t> stage_events) {
  const char* op = "moe_layer_forward";
  TORCH_CHECK(hidden.is_cuda() && logits.is_cuda() && w_gu.is_cuda() && w_down.is_cuda() &&
                  out.is_cuda() && workspace.is_cuda(),
              op, ": tensors must be on CUDA");
  TORCH_CHECK(hidden.is_contiguous() && logits.is_contiguous() && w_gu.is_contiguous() &&
                  w_down.is_contiguous() && out.is_contiguous(),
              op, ": tensors must be contiguous");
  TORCH_CHECK(hidden.scalar_type() == at::kBFloat16 && w_gu.scalar_type() == at::kBFloat16 &&
                  w_down.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16,
              op, ": hidden, weights and out must be bfloat16");
  TORCH_CHECK(logits.scalar_type() == at::kFloat, op, ": logits must be float32");
  TORCH_CHECK(hidden.dim() == 2 && logits.dim() == 2 && w_gu.dim() == 3 && w_down.dim() == 3, op,
              ": hidden [T,H], logits [T,E], w_gu [E,2I,H], w_down [E,H,I] expected");
  const int64_t T = hidden.size(0), H = hidden.size(1), E = logits.size(1);
  const int64_t I = w_down.size(2);
  TORCH_CHECK(logits.size(0) == T && w_gu.size(0) == E && w_down.size(0) == E &&
                  w_gu.size(1) == 2 * I && w_gu.size(2) == H && w_down.size(1) == H,
              op, ": inconsistent shapes");
  TORCH_CHECK(out.size(0) == T && out.size(1) == H, op, ": out must be [T, H]");
  TORCH_CHECK(workspace.scalar_type() == at::kByte, op, ": workspace must be uint8");
  float* wp = nullptr;
  int32_t* ip = nullptr;
  if (topk_weights.has_value()) {
    TORCH_CHECK(topk_weights->scalar_type() == at::kFloat && topk_weights->numel() == T * topk &&
                    topk_weights->is_contiguous() && topk_weights->is_cuda(),
                op, ": topk_weights must be a contiguous float32 CUDA tensor of T*topk");
    wp = topk_weights->data_ptr<float>();
  }
  if (topk_indices.has_value()) {
    TORCH_CHECK(topk_indices->scalar_type() == at::kInt && topk_indices->numel() == T * topk &&
                    topk_indices->is_contiguous() && topk_indices->is_cuda(),
                op, ": topk_indices must be a contiguous int32 CUDA tensor of T*topk");
    ip = topk_indices->data_ptr<int32_t>();
  }
  const c10::cuda::OptionalCUDAGuard guard(hidden.device());
  lsek_topk_gating_params p;
  p.num_tokens = to_i32(T, "num_tokens");
  p.num_experts = to_i32(E, "num_experts");
  p.topk = to_i32(topk, "topk");
  p.n_group = static_cast<int32_t>(n_group);
  p.topk_group = static_cast<int32_t>(topk_group);
  p.routed_scaling_factor = static_cast<float>(routed_scaling_factor);
  p.renormalize = renormalize ? 1 : 0;
  p.scoring_func = scoring_code(scoring_func);
  TORCH_CHECK(stage_events.empty() || stage_events.size() == LSEK_LAYER_STAGES + 1, op,
              ": stage_events must be empty or hold ", LSEK_LAYER_STAGES + 1, " event handles");
  std::vector<void*> ev(stage_events.size());
  for (size_t i = 0; i < ev.size(); ++i) ev[i] = reinterpret_cast<void*>(stage_events[i]);
  check_status(lsek_moe_layer_forward(
      out.data_ptr(), hidden.data_ptr(), logits.data_ptr<float>(), bias_ptr(bias, E),
      w_gu.data_ptr(), w_down.data_ptr(), &p, to_i32(H, "hidden_dim"), to_i32(I, "inter_dim"),
      static_cast<float>(swiglu_limit), wp, ip, workspace.data_ptr(),
      static_cast<size_t>(workspace.numel()), ev.empty() ? nullptr : ev.data(),
      stream_of(hidden)));
}

// ---- expert-parallel device steps (the exchanges are issued from Python) --------

void check_i32_cuda(const torch::Tensor& t, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.is_contiguous() && t.scalar_type() == at::kInt, what,
              " must be a contiguous int32 CUDA tensor");
}

// Returns (send_off [G+1], send_counts [G, 2], pair_row [T*G], row_pair [T*G]).
std::vector<torch::Tensor> ep_plan(torch::Tensor topk_indices, int64_t num_experts,
                                   int64_t world_size) {
  check_i32_cuda(topk_indices, "ep_plan: topk_indices");
  TORCH_CHECK(topk_indices.dim() == 2, "ep_plan: topk_indices must be [T, topk]");
  const c10::cuda::OptionalCUDAGuard guard(topk_indices.device());
  const int64_t T = topk_indices.size(0), k = topk_indices.size(1);
  auto opts = topk_indices.options();
  auto send_off = torch::empty({world_size + 1}, opts);
  auto send_counts = torch::empty({world_size, 2}, opts);
  auto pair_row = torch::empty({T * world_size}, opts);
  auto row_pair = torch::empty({T * world_size}, opts);
  const size_t ws_bytes = lsek_ep_plan_workspace_size(to_i32(T, "T"), to_i32(world_size, "G"));
  auto ws = torch::empty({static_cast<int64_t>(ws_bytes)}, opts.dtype(at::kByte));
  check_status(lsek_ep_plan(send_off.data_ptr<int32_t>(), send_counts.data_ptr<int32_t>(),
                            pair_row.data_ptr<int32_t>(),
                            row_pair.data_ptr<int32_t>(), topk_indices.data_ptr<int32_t>(),
                            to_i32(T, "T"), to_i32(k, "topk"), to_i32(num_experts, "E"),
                            to_i32(world_size, "G"), ws.data_ptr(), ws_bytes,
                            stream_of(topk_indices)));
  return {send_off, send_counts, pair_row, row_pair};
}

// Returns (send_rows [rows, H], send_ids [rows, k], send_w [rows, k]).
std::vector<torch::Tensor> ep_dispatch_pack(torch::Tensor hidden, torch::Tensor topk_indices,
                                            torch::Tensor topk_weights, torch::Tensor pair_row,
                                            torch::Tensor send_off, int64_t rows,
                                            int64_t num_experts, int64_t world_size) {
  TORCH_CHECK(hidden.is_cuda() && hidden.is_contiguous() && hidden.scalar_type() == at::kBFloat16,
              "ep_dispatch_pack: hidden must be a contiguous bf16 CUDA tensor");
  check_i32_cuda(topk_indices, "ep_dispatch_pack: topk_indices");
  check_i32_cuda(pair_row, "ep_dispatch_pack: pair_row");
  check_i32_cuda(send_off, "ep_dispatch_pack: send_off");
  TORCH_CHECK(topk_weights.is_cuda() && topk_weights.is_contiguous() &&
                  topk_weights.scalar_type() == at::kFloat,
              "ep_dispatch_pack: topk_weights must be a contiguous float32 CUDA tensor");
  const c10::cuda::OptionalCUDAGuard guard(hidden.device());
  const int64_t T = hidden.size(0), H = hidden.size(1), k = topk_indices.size(1);
  auto send_rows = torch::empty({rows, H}, hidden.options());
  auto send_ids = torch::empty({rows, k}, topk_indices.options());
  auto send_w = torch::empty({rows, k}, topk_weights.options());
  check_status(lsek_ep_dispatch_pack(
      send_rows.data_ptr(), send_ids.data_ptr<int32_t>(), send_w.data_ptr<float>(),
      to_i32(rows, "rows"), hidden.data_ptr(),
      topk_indices.data_ptr<int32_t>(), topk_weights.data_ptr<float>(), pair_row.data_ptr<int32_t>(),
      send_off.data_ptr<int32_t>(), to_i32(T, "T"), to_i32(k, "topk"), to_i32(H, "H"),
      to_i32(num_experts, "E"), to_i32(world_size, "G"), stream_of(hidden)));
  return {send_rows, send_ids, send_w};
}

torch::Tensor ep_slot_scan(torch::Tensor ids) {
  check_i32_cuda(ids, "ep_slot_scan: ids");
  TORCH_CHECK(ids.dim() == 2, "ep_slot_scan: ids must be [rows, topk]");
  const c10::cuda::OptionalCUDAGuard guard(ids.device());
  auto out = torch::empty({ids.size(0) + 1}, ids.options());
  check_status(lsek_ep_slot_scan(out.data_ptr<int32_t>(), ids.data_ptr<int32_t>(),
                                 to_i32(ids.size(0), "rows"), to_i32(ids.size(1), "topk"),
                                 stream_of(ids)));
  return out;
}

// Returns (permuted [valid_slots, H], offsets [El+1], s2d [rows*k], perm [rows*k]).
std::vector<torch::Tensor> ep_expert_permute(torch::Tensor rows_in, torch::Tensor local_ids,
                                             int64_t local_experts, int64_t valid_slots) {
  TORCH_CHECK(rows_in.is_cuda() && rows_in.is_contiguous() && rows_in.scalar_type() == at::kBFloat16,
              "ep_expert_permute: rows must be a contiguous bf16 CUDA tensor");
  check_i32_cuda(local_ids, "ep_expert_permute: local_ids");
  const c10::cuda::OptionalCUDAGuard guard(rows_in.device());
  const int64_t R = rows_in.size(0), H = rows_in.size(1), k = local_ids.size(1);
  TORCH_CHECK(valid_slots >= 0 && valid_slots <= R * k, "ep_expert_permute: valid_slots out of range");
  auto permuted = torch::empty({valid_slots, H}, rows_in.options());
  auto offsets = torch::empty({local_experts + 1}, local_ids.options());
  auto s2d = torch::empty({R * k}, local_ids.options());
  auto perm = torch::empty({R * k}, local_ids.options());
  const size_t ws_bytes = lsek_moe_permute_workspace_size(to_i32(R, "rows"), to_i32(k, "topk"),
                                                          to_i32(local_experts, "E"));
  auto ws = torch::empty({static_cast<int64_t>(ws_bytes)}, local_ids.options().dtype(at::kByte));
  check_status(lsek_ep_expert_permute(
      permuted.data_ptr(), to_i32(valid_slots, "valid_slots"), offsets.data_ptr<int32_t>(), s2d.data_ptr<int32_t>(),
      perm.data_ptr<int32_t>(), rows_in.data_ptr(), local_ids.data_ptr<int32_t>(), to_i32(R, "rows"),
      to_i32(k, "topk"), to_i32(H, "H"), to_i32(local_experts, "E"), ws.data_ptr(), ws_bytes,
      stream_of(rows_in)));
  return {permuted, offsets, s2d, perm};
}

torch::Tensor ep_combine_pack(torch::Tensor expert_out, torch::Tensor s2d, torch::Tensor ids,
                              torch::Tensor weights, torch::Tensor slot_row, int64_t comb_rows) {
  TORCH_CHECK(expert_out.is_cuda() && expert_out.is_contiguous() &&
                  expert_out.scalar_type() == at::kBFloat16,
              "ep_combine_pack: expert_out must be a contiguous bf16 CUDA tensor");
  check_i32_cuda(s2d, "ep_combine_pack: s2d");
  check_i32_cuda(ids, "ep_combine_pack: ids");
  check_i32_cuda(slot_row, "ep_combine_pack: slot_row");
  const c10::cuda::OptionalCUDAGuard guard(expert_out.device());
  const int64_t H = expert_out.size(1);
  auto comb = torch::empty({comb_rows, H}, expert_out.options());
  check_status(lsek_ep_combine_pack(comb.data_ptr(), to_i32(comb_rows, "comb_rows"),
                                    expert_out.data_ptr(), s2d.data_ptr<int32_t>(),
                                    ids.data_ptr<int32_t>(), weights.data_ptr<float>(),
                                    slot_row.data_ptr<int32_t>(), to_i32(ids.size(0), "rows"),
                                    to_i32(ids.size(1), "topk"), to_i32(H, "H"),
                                    stream_of(expert_out)));
  return comb;
}

torch::Tensor ep_combine_reduce(torch::Tensor comb_rows, torch::Tensor topk_indices,
                                torch::Tensor pair_row, torch::Tensor slot_row,
                                int64_t num_experts, int64_t world_size,
                                c10::optional<torch::Tensor> out_opt) {
  TORCH_CHECK(comb_rows.is_cuda() && comb_rows.is_contiguous() &&
                  comb_rows.scalar_type() == at::kBFloat16,
              "ep_combine_reduce: comb_rows must be a contiguous bf16 CUDA tensor");
  check_i32_cuda(topk_indices, "ep_combine_reduce: topk_indices");
  const c10::cuda::OptionalCUDAGuard guard(comb_rows.device());
  const int64_t T = topk_indices.size(0), k = topk_indices.size(1), H = comb_rows.size(1);
  torch::Tensor out;
  if (out_opt.has_value()) {
    out = *out_opt;
    TORCH_CHECK(out.is_cuda() && out.is_contiguous() && out.scalar_type() == at::kBFloat16 &&
                    out.dim() == 2 && out.size(0) == T && out.size(1) == H,
                "ep_combine_reduce: out must be a contiguous bf16 CUDA tensor [T, H]");
  } else {
    out = torch::empty({T, H}, comb_rows.options());
  }
  check_status(lsek_ep_combine_reduce(out.data_ptr(), comb_rows.data_ptr(),
                                      to_i32(comb_rows.size(0), "comb_rows"),
                                      topk_indices.data_ptr<int32_t>(), pair_row.data_ptr<int32_t>(),
                                      slot_row.data_ptr<int32_t>(), to_i32(T, "T"), to_i32(k, "topk"),
                                      to_i32(H, "H"), to_i32(num_experts, "E"),
                                      to_i32(world_size, "G"), stream_of(comb_rows)));
  return out;
}

// ---- expert-parallel peer domain (handles travel as Python ints) --------------

lsek_ep_domain* domain_of(int64_t h) {
  TORCH_CHECK(h != 0, "ep domain handle is null");
  return reinterpret_cast<lsek_ep_domain*>(static_cast<intptr_t>(h));
}

void check_counts(const torch::Tensor& counts) {
  TORCH_CHECK(!counts.is_cuda() && counts.is_contiguous() && counts.scalar_type() == at::kInt &&
                  counts.dim() == 3 && counts.size(2) == 2,
              "counts must be a contiguous int32 CPU tensor [G, G, 2]");
}

int64_t ep_domain_create(int64_t rank, int64_t world_size, int64_t max_tokens, int64_t hidden_dim,
                         int64_t topk) {
  lsek_ep_domain* d = nullptr;
  check_status(lsek_ep_domain_create(&d, to_i32(rank, "rank"), to_i32(world_size, "world_size"),
                                     to_i32(max_tokens, "max_tokens"), to_i32(hidden_dim, "hidden"),
                                     to_i32(topk, "topk")));
  return static_cast<int64_t>(reinterpret_cast<intptr_t>(d));
}

torch::Tensor ep_domain_export(int64_t h) {
  auto out = torch::empty({LSEK_EP_HANDLE_BYTES}, torch::dtype(torch::kUInt8));
  check_status(lsek_ep_domain_export(domain_of(h), out.data_ptr(), LSEK_EP_HANDLE_BYTES));
  return out;
}

void ep_domain_import(int64_t h, int64_t peer, torch::Tensor handle) {
  TORCH_CHECK(!handle.is_cuda() && handle.is_contiguous() && handle.scalar_type() == at::kByte &&
                  handle.numel() >= LSEK_EP_HANDLE_BYTES,
              "ep_domain_import: handle must be a CPU uint8 tensor of 64 bytes");
  check_status(lsek_ep_domain_import(domain_of(h), to_i32(peer, "peer"), handle.data_ptr(),
                                     static_cast<size_t>(handle.numel())));
}

// Non-owning views of this rank's buffers: (recv_rows, recv_ids, recv_w, back).
std::vector<torch::Tensor> ep_domain_buffers(int64_t h, int64_t hidden_dim, int64_t topk) {
  void *rows = nullptr, *back = nullptr;
  int32_t* ids = nullptr;
  float* w = nullptr;
  int64_t cap_rows = 0, cap_slots = 0;
  check_status(lsek_ep_domain_buffers(domain_of(h), &rows, &ids, &w, &back, &cap_rows, &cap_slots));
  int dev = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  auto o = torch::TensorOptions().device(torch::kCUDA, dev);
  return {torch::from_blob(rows, {cap_rows, hidden_dim}, o.dtype(at::kBFloat16)),
          torch::from_blob(ids, {cap_rows, topk}, o.dtype(at::kInt)),
          torch::from_blob(w, {cap_rows, topk}, o.dtype(at::kFloat)),
          torch::from_blob(back, {cap_slots, hidden_dim}, o.dtype(at::kBFloat16))};
}

void ep_domain_destroy(int64_t h) {
  if (h != 0) lsek_ep_domain_destroy(domain_of(h));
}

torch::Tensor ep_dispatch_push(int64_t h, torch::Tensor counts, torch::Tensor hidden,
                               torch::Tensor topk_indices, torch::Tensor topk_weights,
                               torch::Tensor pair_row, torch::Tensor send_off, int64_t rows,
                               int64_t num_experts, int64_t epoch) {
  check_counts(counts);
  TORCH_CHECK(hidden.is_cuda() && hidden.is_contiguous() && hidden.scalar_type() == at::kBFloat16,
              "ep_dispatch_push: hidden must be a contiguous bf16 CUDA tensor");
  check_i32_cuda(topk_indices, "ep_dispatch_push: topk_indices");
  check_i32_cuda(pair_row, "ep_dispatch_push: pair_row");
  check_i32_cuda(send_off, "ep_dispatch_push: send_off");
  TORCH_CHECK(topk_weights.is_cuda() && topk_weights.is_contiguous() &&
                  topk_weights.scalar_type() == at::kFloat,
              "ep_dispatch_push: topk_weights must be a contiguous float32 CUDA tensor");
  const c10::cuda::OptionalCUDAGuard guard(hidden.device());
  const int64_t T = hidden.size(0), k = topk_indices.size(1);
  auto send_ids = torch::empty({rows, k}, topk_indices.options());
  check_status(lsek_ep_dispatch_push(
      domain_of(h), send_ids.data_ptr<int32_t>(), to_i32(rows, "rows"), counts.data_ptr<int32_t>(),
      hidden.data_ptr(), topk_indices.data_ptr<int32_t>(), topk_weights.data_ptr<float>(),
      pair_row.data_ptr<int32_t>(), send_off.data_ptr<int32_t>(), to_i32(T, "T"),
      to_i32(num_experts, "E"), static_cast<uint32_t>(epoch), stream_of(hidden)));
  return send_ids;
}

void copy_to_mapped_host(torch::Tensor host_dst, torch::Tensor src) {
  TORCH_CHECK(host_dst.device().is_cpu() && host_dst.is_pinned(),
              "copy_to_mapped_host: host_dst must be a pinned CPU tensor");
  TORCH_CHECK(src.is_cuda(), "copy_to_mapped_host: src must be a CUDA tensor");
  TORCH_CHECK(host_dst.is_contiguous() && src.is_contiguous(),
              "copy_to_mapped_host: tensors must be contiguous");
  TORCH_CHECK(host_dst.nbytes() == src.nbytes(), "copy_to_mapped_host: sizes differ");
  const c10::cuda::OptionalCUDAGuard guard(src.device());
  check_status(lsek_copy_to_mapped_host(host_dst.data_ptr(), src.data_ptr(), src.nbytes(),
                                        stream_of(src)));
}

void ep_wait(int64_t h, int64_t what, int64_t epoch, int64_t timeout_ns) {
  check_status(lsek_ep_wait(domain_of(h), to_i32(what, "what"), static_cast<uint32_t>(epoch),
                            timeout_ns, at::cuda::getCurrentCUDAStream().stream()));
}

std::vector<torch::Tensor> ep_combine_plan(int64_t h, torch::Tensor s2d, torch::Tensor slot_row,
                                           torch::Tensor counts, int64_t recv_rows,
                                           int64_t valid_slots) {
  check_counts(counts);
  check_i32_cuda(s2d, "ep_combine_plan: s2d");
  check_i32_cuda(slot_row, "ep_combine_plan: slot_row");
  const c10::cuda::OptionalCUDAGuard guard(s2d.device());
  auto dst_rank = torch::empty({valid_slots}, s2d.options());
  auto dst_row = torch::empty({valid_slots}, s2d.options());
  auto dst_w = torch::empty({valid_slots}, s2d.options().dtype(at::kFloat));
  check_status(lsek_ep_combine_plan(domain_of(h), dst_rank.data_ptr<int32_t>(),
                                    dst_row.data_ptr<int32_t>(), dst_w.data_ptr<float>(),
                                    s2d.data_ptr<int32_t>(), slot_row.data_ptr<int32_t>(),
                                    counts.data_ptr<int32_t>(), to_i32(recv_rows, "recv_rows"),
                                    to_i32(valid_slots, "valid_slots"), stream_of(s2d)));
  return {dst_rank, dst_row, dst_w};
}

void ep_combine_push(int64_t h, torch::Tensor expert_out, torch::Tensor dst_rank,
                     torch::Tensor dst_row, torch::Tensor dst_w, int64_t epoch,
                     c10::optional<torch::Tensor> row_lo, c10::optional<torch::Tensor> row_hi,
                     bool publish) {
  TORCH_CHECK(expert_out.is_cuda() && expert_out.is_contiguous() &&
                  expert_out.scalar_type() == at::kBFloat16,
              "ep_combine_push: expert_out must be a contiguous bf16 CUDA tensor");
  check_i32_cuda(dst_rank, "ep_combine_push: dst_rank");
  check_i32_cuda(dst_row, "ep_combine_push: dst_row");
  const c10::cuda::OptionalCUDAGuard guard(expert_out.device());
  TORCH_CHECK(dst_rank.numel() <= expert_out.size(0), "ep_combine_push: more plan rows than outputs");
  TORCH_CHECK(row_lo.has_value() == row_hi.has_value(), "ep_combine_push: give both row bounds or none");
  const int32_t* lo = nullptr;
  const int32_t* hi = nullptr;
  if (row_lo.has_value()) {
    check_i32_cuda(*row_lo, "ep_combine_push: row_lo");
    check_i32_cuda(*row_hi, "ep_combine_push: row_hi");
    lo = row_lo->data_ptr<int32_t>();
    hi = row_hi->data_ptr<int32_t>();
  }
  check_status(lsek_ep_combine_push(domain_of(h), expert_out.data_ptr(),
                                    dst_rank.data_ptr<int32_t>(), dst_row.data_ptr<int32_t>(),
                                    dst_w.data_ptr<float>(), to_i32(dst_rank.numel(), "rows"), lo,
                                    hi, publish ? 1 : 0, static_cast<uint32_t>(epoch),
                                    stream_of(expert_out)));
}

// lsek_ep_combine_plan_chunks: [dst_rank, dst_row, dst_w, order [chunks *
// valid_slots], order_count [chunks]].
std::vector<torch::Tensor> ep_combine_plan_chunks(int64_t h, torch::Tensor s2d,
                                                  torch::Tensor slot_row, torch::Tensor counts,
                                                  int64_t recv_rows, int64_t valid_slots,
                                                  int64_t chunk_tokens, int64_t chunks) {
  check_counts(counts);
  check_i32_cuda(s2d, "ep_combine_plan_chunks: s2d");
  check_i32_cuda(slot_row, "ep_combine_plan_chunks: slot_row");
  TORCH_CHECK(chunks >= 1 && chunks <= 16, "ep_combine_plan_chunks: chunks must be in [1, 16]");
  const c10::cuda::OptionalCUDAGuard guard(s2d.device());
  auto dst_rank = torch::empty({valid_slots}, s2d.options());
  auto dst_row = torch::empty({valid_slots}, s2d.options());
  auto dst_w = torch::empty({valid_slots}, s2d.options().dtype(at::kFloat));
  auto order = torch::empty({chunks * valid_slots}, s2d.options());
  auto order_count = torch::empty({chunks}, s2d.options());
  check_status(lsek_ep_combine_plan_chunks(
      domain_of(h), dst_rank.data_ptr<int32_t>(), dst_row.data_ptr<int32_t>(),
      dst_w.data_ptr<float>(), order.data_ptr<int32_t>(), order_count.data_ptr<int32_t>(),
      s2d.data_ptr<int32_t>(), slot_row.data_ptr<int32_t>(), counts.data_ptr<int32_t>(),
      to_i32(recv_rows, "recv_rows"), to_i32(valid_slots, "valid_slots"),
      to_i32(chunk_tokens, "chunk_tokens"), to_i32(chunks, "chunks"), stream_of(s2d)));
  return {dst_rank, dst_row, dst_w, order, order_count};
}

void ep_combine_push_chunk(int64_t h, torch::Tensor expert_out, torch::Tensor dst_rank,
                           torch::Tensor dst_row, torch::Tensor dst_w, torch::Tensor order,
                           torch::Tensor order_count, int64_t chunk, int64_t epoch,
                           c10::optional<torch::Tensor> row_lo,
                           c10::optional<torch::Tensor> row_hi) {
  TORCH_CHECK(expert_out.is_cuda() && expert_out.is_contiguous() &&
                  expert_out.scalar_type() == at::kBFloat16,
              "ep_combine_push_chunk: expert_out must be a contiguous bf16 CUDA tensor");
  check_i32_cuda(dst_rank, "ep_combine_push_chunk: dst_rank");
  check_i32_cuda(dst_row, "ep_combine_push_chunk: dst_row");
  check_i32_cuda(order, "ep_combine_push_chunk: order");
  check_i32_cuda(order_count, "ep_combine_push_chunk: order_count");
  const c10::cuda::OptionalCUDAGuard guard(expert_out.device());
  TORCH_CHECK(chunk >= 0 && order_count.numel() > chunk, "ep_combine_push_chunk: chunk out of range");
  TORCH_CHECK(dst_rank.numel() <= expert_out.size(0) &&
                  order.numel() >= (chunk + 1) * dst_rank.numel(),
              "ep_combine_push_chunk: plan rows, chunk lists and outputs disagree");
  TORCH_CHECK(row_lo.has_value() == row_hi.has_value(),
              "ep_combine_push_chunk: give both row bounds or none");
  const int32_t* lo = nullptr;
  const int32_t* hi = nullptr;
  if (row_lo.has_value()) {
    check_i32_cuda(*row_lo, "ep_combine_push_chunk: row_lo");
    check_i32_cuda(*row_hi, "ep_combine_push_chunk: row_hi");
    lo = row_lo->data_ptr<int32_t>();
    hi = row_hi->data_ptr<int32_t>();
  }
  check_status(lsek_ep_combine_push_chunk(
      domain_of(h), expert_out.data_ptr(), dst_rank.data_ptr<int32_t>(),
      dst_row.data_ptr<int32_t>(), dst_w.data_ptr<float>(), to_i32(dst_rank.numel(), "rows"), lo,
      hi, order.data_ptr<int32_t>(), order_count.data_ptr<int32_t>(), to_i32(chunk, "chunk"),
      static_cast<uint32_t>(epoch),
      stream_of(expert_out)));
}

void ep_down_gemm_combine(int64_t h, torch::Tensor hact, torch::Tensor w_down,
                          torch::Tensor expert_offsets, torch::Tensor dst_rank,
                          torch::Tensor dst_row, torch::Tensor dst_w, int64_t epoch) {
  TORCH_CHECK(hact.is_cuda() && hact.is_contiguous() && hact.scalar_type() == at::kBFloat16 &&
                  hact.dim() == 2,
              "ep_down_gemm_combine: h must be a contiguous bf16 CUDA tensor [rows, I]");
  TORCH_CHECK(w_down.is_cuda() && w_down.is_contiguous() && w_down.scalar_type() == at::kBFloat16 &&
                  w_down.dim() == 3,
              "ep_down_gemm_combine: W_down must be a contiguous bf16 CUDA tensor [E, H, I]");
  check_i32_cuda(expert_offsets, "ep_down_gemm_combine: expert_offsets");
  const c10::cuda::OptionalCUDAGuard guard(hact.device());
  TORCH_CHECK(dst_rank.numel() >= hact.size(0), "ep_down_gemm_combine: plan shorter than rows");
  auto ws = torch::empty({LSEK_GEMM_WORKSPACE_BYTES}, hact.options().dtype(at::kByte));
  check_status(lsek_ep_down_gemm_combine(
      domain_of(h), hact.data_ptr(), w_down.data_ptr(), expert_offsets.data_ptr<int32_t>(),
      to_i32(w_down.size(0), "local_experts"), to_i32(hact.size(0), "rows"),
      to_i32(hact.size(1), "I"), dst_rank.data_ptr<int32_t>(), dst_row.data_ptr<int32_t>(),
      dst_w.data_ptr<float>(), static_cast<uint32_t>(epoch), ws.data_ptr(), LSEK_GEMM_WORKSPACE_BYTES,
      stream_of(hact)));
}

// Timing events for lsek_moe_layer_forward's stage_events: created with
// timing enabled, recorded by the library on the layer's stream, read back
// as milliseconds between consecutive events.
std::vector<int64_t> events_create(int64_t n) {
  std::vector<int64_t> out;
  for (int64_t i = 0; i < n; ++i) {
    cudaEvent_t e = nullptr;
    TORCH_CHECK(cudaEventCreate(&e) == cudaSuccess, "events_create: cudaEventCreate failed");
    out.push_back(reinterpret_cast<int64_t>(e));
  }
  return out;
}

std::vector<double> events_elapsed_ms(std::vector<int64_t> handles) {
  std::vector<double> out;
  for (size_t i = 0; i + 1 < handles.size(); ++i) {
    auto a = reinterpret_cast<cudaEvent_t>(handles[i]);
    auto b = reinterpret_cast<cudaEvent_t>(handles[i + 1]);
    TORCH_CHECK(cudaEventSynchronize(b) == cudaSuccess, "events_elapsed_ms: synchronize failed");
    float ms = 0.0f;
    TORCH_CHECK(cudaEventElapsedTime(&ms, a, b) == cudaSuccess,
                "events_elapsed_ms: event not recorded");
    out.push_back(ms);
  }
  return out;
}

void events_destroy(std::vector<int64_t> handles) {
  for (auto h : handles) cudaEventDestroy(reinterpret_cast<cudaEvent_t>(h));
}

int64_t device_error() {
  int32_t code = 0;
  check_status(lsek_device_error(&code, static_cast<void*>(at::cuda::getCurrentCUDAStream().stream())));
  return code;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "B200 (sm_100a) MoE expert kernels behind the sm120_expert_kernels operator surface";
  namespace py = pybind11;

  m.def("fused_swiglu", &fused_swiglu, py::arg("input"), py::arg("swiglu_limit") = 0.0,
        "Fused SwiGLU: SiLU(gate) * up with optional clamp. Input [N, 2*d] -> output [N, d].");
  m.def("moe_permute", &moe_permute, py::arg("hidden_states"), py::arg("topk_indices"),
        py::arg("num_experts"),
        "MoE permute: sort tokens by expert. Returns (permuted, offsets, s2d_map, perm_idx).");
  m.def("moe_route", &moe_route, py::arg("topk_indices"), py::arg("num_experts"),
        "routing maps of moe_permute without the row copy: [expert_offsets, src_to_dest_map, "
        "permuted_idx]");
  m.def("moe_unpermute", &moe_unpermute, py::arg("permuted_output"), py::arg("topk_weights"),
        py::arg("src_to_dest_map"), py::arg("num_tokens"), py::arg("topk"),
        "MoE unpermute: weighted reduction back to original order.");
  m.def("moe_unpermute_fp32", &moe_unpermute_fp32, py::arg("permuted_output"),
        py::arg("topk_weights"), py::arg("src_to_dest_map"), py::arg("num_tokens"),
        py::arg("topk"), "Per-slot fp32 contributions [num_tokens, topk, hidden].");
  m.def("moe_combine_reduce_slots_fp32_to_bf16", &moe_combine_reduce_slots_fp32_to_bf16,
        py::arg("input_perslot_fp32"),
        "Fixed-order slot reduce of [num_tokens, topk, hidden] fp32 -> [num_tokens, hidden] bf16.");
  m.def("moe_unpermute_bf16_perslot", &moe_unpermute_bf16_perslot, py::arg("permuted_output"),
        py::arg("topk_weights"), py::arg("src_to_dest_map"), py::arg("num_tokens"),
        py::arg("topk"), "Per-slot 16-bit contributions [num_tokens, topk, hidden].");
  m.def("moe_combine_reduce_slots_bf16_to_bf16", &moe_combine_reduce_slots_bf16_to_bf16,
        py::arg("input_perslot_bf16"),
        "Fixed-order slot reduce of [num_tokens, topk, hidden] bf16 -> [num_tokens, hidden] bf16.");
  m.def("adaptive_gating", &adaptive_gating, py::arg("in_weights"), py::arg("in_indices"),
        py::arg("threshold"),
        "Adaptive gating: threshold-based expert pruning. Returns (weights, indices, counts).");
  m.def("topk_gating", &topk_gating, py::arg("logits"), py::arg("bias"), py::arg("topk"),
        py::arg("n_group"), py::arg("topk_group"), py::arg("routed_scaling_factor"),
        py::arg("renormalize"), py::arg("scoring_func") = "sigmoid",
        "Top-K gating with configurable scoring. Returns (weights, indices).");

  m.def("grouped_gemm_bf16", &grouped_gemm_bf16, py::arg("A"), py::arg("B"),
        py::arg("expert_offsets"),
        "Grouped bf16 GEMM: D[rows of e] = A[rows of e] @ B[e]^T, B [E, N, K].");
  m.def("grouped_gemm_swiglu_bf16", &grouped_gemm_swiglu_bf16, py::arg("A"), py::arg("W_gu"),
        py::arg("expert_offsets"), py::arg("swiglu_limit") = 0.0,
        "Gate/up grouped GEMM with fused SwiGLU: W_gu [E, 2I, K] -> [rows, I].");
  m.def("moe_layer_workspace_size", &moe_layer_workspace_size, py::arg("num_tokens"),
        py::arg("hidden_dim"), py::arg("inter_dim"), py::arg("num_experts"), py::arg("topk"));
  m.def("moe_layer_forward_out", &moe_layer_forward_out, py::arg("out"), py::arg("hidden"),
        py::arg("logits"), py::arg("bias"), py::arg("w_gu"), py::arg("w_down"), py::arg("topk"),
        py::arg("n_group"), py::arg("topk_group"), py::arg("routed_scaling_factor"),
        py::arg("renormalize"), py::arg("scoring_func"), py::arg("swiglu_limit"),
        py::arg("workspace"), py::arg("topk_weights") = py::none(),
        py::arg("topk_indices") = py::none(), py::arg("stage_events") = std::vector<int64_t>{});
  m.def("ep_plan", &ep_plan, py::arg("topk_indices"), py::arg("num_experts"),
        py::arg("world_size"));
  m.def("ep_dispatch_pack", &ep_dispatch_pack, py::arg("hidden"), py::arg("topk_indices"),
        py::arg("topk_weights"), py::arg("pair_row"), py::arg("send_off"), py::arg("rows"),
        py::arg("num_experts"), py::arg("world_size"));
  m.def("ep_slot_scan", &ep_slot_scan, py::arg("ids"));
  m.def("ep_expert_permute", &ep_expert_permute, py::arg("rows"), py::arg("local_ids"),
        py::arg("local_experts"), py::arg("valid_slots"));
  m.def("ep_combine_pack", &ep_combine_pack, py::arg("expert_out"), py::arg("s2d"), py::arg("ids"),
        py::arg("weights"), py::arg("slot_row"), py::arg("comb_rows"));
  m.def("ep_combine_reduce", &ep_combine_reduce, py::arg("comb_rows"), py::arg("topk_indices"),
        py::arg("pair_row"), py::arg("slot_row"), py::arg("num_experts"), py::arg("world_size"),
        py::arg("out") = py::none());
  m.def("ep_combine_plan_chunks", &ep_combine_plan_chunks, py::arg("domain"), py::arg("s2d"),
        py::arg("slot_row"), py::arg("counts"), py::arg("recv_rows"), py::arg("valid_slots"),
        py::arg("chunk_tokens"), py::arg("chunks"));
  m.def("ep_combine_push_chunk", &ep_combine_push_chunk, py::arg("domain"), py::arg("expert_out"),
        py::arg("dst_rank"), py::arg("dst_row"), py::arg("dst_w"), py::arg("order"),
        py::arg("order_count"), py::arg("chunk"), py::arg("epoch"), py::arg("row_lo") = py::none(),
        py::arg("row_hi") = py::none());
  m.def("ep_domain_create", &ep_domain_create, py::arg("rank"), py::arg("world_size"),
        py::arg("max_tokens"), py::arg("hidden_dim"), py::arg("topk"));
  m.def("ep_domain_export", &ep_domain_export, py::arg("domain"));
  m.def("ep_domain_import", &ep_domain_import, py::arg("domain"), py::arg("peer"),
        py::arg("handle"));
  m.def("ep_domain_buffers", &ep_domain_buffers, py::arg("domain"), py::arg("hidden_dim"),
        py::arg("topk"));
  m.def("ep_domain_destroy", &ep_domain_destroy, py::arg("domain"));
  m.def("ep_dispatch_push", &ep_dispatch_push, py::arg("domain"), py::arg("counts"),
        py::arg("hidden"), py::arg("topk_indices"), py::arg("topk_weights"), py::arg("pair_row"),
        py::arg("send_off"), py::arg("rows"), py::arg("num_experts"), py::arg("epoch"));
  m.def("copy_to_mapped_host", &copy_to_mapped_host, py::arg("host_dst"), py::arg("src"));
  m.def("ep_wait", &ep_wait, py::arg("domain"), py::arg("what"), py::arg("epoch"),
        py::arg("timeout_ns") = 0);
  m.def("ep_combine_plan", &ep_combine_plan, py::arg("domain"), py::arg("s2d"),
        py::arg("slot_row"), py::arg("counts"), py::arg("recv_rows"), py::arg("valid_slots"));
  m.def("ep_combine_push", &ep_combine_push, py::arg("domain"), py::arg("expert_out"),
        py::arg("dst_rank"), py::arg("dst_row"), py::arg("dst_w"), py::arg("epoch"),
        py::arg("row_lo") = py::none(), py::arg("row_hi") = py::none(), py::arg("publish") = true);
  m.def("grouped_gemm_bf16_out", &grouped_gemm_bf16_out, py::arg("D"), py::arg("A"), py::arg("B"),
        py::arg("expert_offsets"));
  m.def("ep_down_gemm_combine", &ep_down_gemm_combine, py::arg("domain"), py::arg("h"),
        py::arg("w_down"), py::arg("expert_offsets"), py::arg("dst_rank"), py::arg("dst_row"),
        py::arg("dst_w"), py::arg("epoch"));
  m.def("events_create", &events_create, py::arg("n"));
  m.def("events_elapsed_ms", &events_elapsed_ms, py::arg("handles"));
  m.def("events_destroy", &events_destroy, py::arg("handles"));
  m.def("device_error", &device_error,
        "Reads and clears the device-side error word (synchronises the current stream).");
  m.def("version", [] { return std::string(lsek_version()); });
}
