/*
 * lsek.h — C ABI of the B200 (sm_100a) MoE expert-kernel library (liblsek.so).
 *
 * Every entry point takes plain device pointers, sizes and a `void* stream`
 * (a cudaStream_t), launches asynchronously on that stream and returns an
 * lsek_status.  Nothing here allocates device memory: outputs and scratch
 * ("workspace") buffers are owned by the caller, with a size-query function
 * for each entry point that needs scratch.  The library keeps no per-call
 * state, so entry points are safe to call from several host threads on
 * different streams.
 *
 * Each entry point replaces one launcher of the reference library
 * (kkontosis/LayerStoRmExpertKernels, namespace layerstorm::compute); the
 * replaced interface is cited as file:line beside each declaration.  Shapes
 * and argument meanings are the reference's.  Three differences, all
 * deliberate:
 *   - errors come back as status codes (the reference throws C++ exceptions
 *     and never checks launch errors);
 *   - limits the reference leaves unchecked (topk <= 8 in unpermute, topk
 *     within the kept groups, experts per lane) are validated;
 *   - fp16 is computed as fp16 (the reference runs its bf16 kernel on fp16
 *     data).
 */
#ifndef LSEK_H_
#define LSEK_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LSEK_ABI_VERSION 1

/* Entry points are the only symbols liblsek.so exports. */
#if defined(__GNUC__)
#define LSEK_API __attribute__((visibility("default")))
#else
#define LSEK_API
#endif

/* Status codes.  INVALID_ARG maps to Python ValueError in the torch binding,
 * the rest to RuntimeError. */
typedef enum lsek_status {
  LSEK_OK = 0,
  LSEK_ERR_INVALID_ARG = 1, /* bad shape / parameter (reference: std::invalid_argument) */
  LSEK_ERR_UNSUPPORTED = 2, /* valid request this build does not implement (dtype, size) */
  LSEK_ERR_CUDA = 3,        /* a CUDA runtime call or kernel launch failed */
  LSEK_ERR_DEVICE = 4       /* a kernel reported a device-side error (bounded wait expired) */
} lsek_status;

/* Element types of activation tensors. */
typedef enum lsek_dtype {
  LSEK_BF16 = 0,
  LSEK_FP16 = 1,
  LSEK_FP32 = 2
} lsek_dtype;

/* Scoring functions (reference: sm120/gating/topk_gating.h:19 ScoringFunc). */
typedef enum lsek_scoring_func {
  LSEK_SCORING_SIGMOID = 0,
  LSEK_SCORING_SQRTSOFTPLUS = 1
} lsek_scoring_func;

/* Top-k gating parameters (reference: sm120/gating/topk_gating.h:22-31
 * TopkGatingParams). */
typedef struct lsek_topk_gating_params {
  int32_t num_tokens;
  int32_t num_experts;
  int32_t topk;                 /* experts selected per token */
  int32_t n_group;              /* expert groups; 1 = flat top-k */
  int32_t topk_group;           /* groups kept before the expert top-k (n_group > 1) */
  float routed_scaling_factor;  /* weights scaled so they sum to this (renormalize) */
  int32_t renormalize;          /* nonzero: w *= routed_scaling_factor / sum(w) */
  int32_t scoring_func;         /* lsek_scoring_func */
} lsek_topk_gating_params;

/* ---- library info ------------------------------------------------------ */

/* Message describing the last non-OK status returned on the calling thread. */
LSEK_API const char* lsek_last_error(void);
/* Version string, e.g. "lsek 0.1.0 sm_100a". */
LSEK_API const char* lsek_version(void);
/* Reads and clears the device-side error word that kernels set when a
 * bounded wait expires (synchronises `stream`).  *code receives 0 when no
 * kernel reported an error since the last call. */
LSEK_API lsek_status lsek_device_error(int32_t* code, void* stream);

/* ---- gating -------------------------------------------------------------- */

/* Top-k gating (grouped when n_group > 1).  logits [T,E] f32 row-major,
 * bias [E] f32 or NULL (selection only), outputs [T,topk] f32 / int32 in
 * selection order (descending biased score, ties to the lower expert id).
 * Limits: E <= 1024, topk <= 32, n_group <= 32, E % n_group == 0,
 * topk <= topk_group * (E / n_group).
 * Replaces launch_topk_gating (sm120/gating/topk_gating.h:43-46,
 * sm120/gating/topk_gating.cu:391-443). */
LSEK_API lsek_status lsek_topk_gating(float* topk_weights, int32_t* topk_indices,
                             const float* logits, const float* bias,
                             const lsek_topk_gating_params* params,
                             void* stream);

/* Adaptive gating: per token, sort (weight, index) by weight descending
 * (stable), keep the shortest prefix whose cumulative weight reaches
 * threshold * total, pad the rest with (0.0, -1).  topk in [1, 32],
 * threshold in [0, 1].  Replaces launch_adaptive_gating
 * (smxx/gating/adaptive_gating.h:34-39, adaptive_gating.cu:94-118). */
LSEK_API lsek_status lsek_adaptive_gating(float* out_weights, int32_t* out_indices,
                                 int32_t* expert_counts,
                                 const float* in_weights,
                                 const int32_t* in_indices, int32_t num_tokens,
                                 int32_t topk, double threshold, void* stream);

/* ---- permute / unpermute -------------------------------------------------- */

/* Scratch bytes lsek_moe_permute needs for these sizes.  Replaces
 * query_moe_permute_workspace_size (smxx/permute/moe_permute.h:25-26). */
LSEK_API size_t lsek_moe_permute_workspace_size(int32_t max_tokens, int32_t max_topk,
                                       int32_t num_experts);

/* Stable counting-sort permute.  topk_indices [T,topk] int32; an index
 * outside [0,E) (the adaptive-gating sentinel -1) is treated as expert E and
 * sorts last.  Outputs: permuted [T*topk, H] (rows grouped by expert, within
 * an expert in ascending t*topk+slot order), expert_offsets [E+1]
 * (offsets[E] = number of valid slots), src_to_dest_map [T*topk],
 * permuted_idx [T*topk].  elem_size_bytes is 2 or 4 (bitwise row copy).
 * E <= 1023.  Replaces launch_moe_permute (smxx/permute/moe_permute.h:42-55,
 * moe_permute.cu:518-600). */
LSEK_API lsek_status lsek_moe_permute(void* permuted_input, int32_t* expert_offsets,
                             int32_t* src_to_dest_map, int32_t* permuted_idx,
                             const void* hidden_states,
                             const int32_t* topk_indices, int32_t num_tokens,
                             int32_t topk, int32_t hidden_dim,
                             int32_t num_experts, int32_t elem_size_bytes,
                             void* workspace, size_t workspace_bytes,
                             void* stream);

/* The routing half of lsek_moe_permute alone: expert_offsets [E+1],
 * src_to_dest_map [T*topk] and permuted_idx [T*topk], identical to what
 * lsek_moe_permute writes for the same topk_indices (same stable order, same
 * sentinel handling), with no row copy and no workspace, in one launch.  For
 * callers that gather the token rows themselves (the layer forward folds the
 * gather into its GEMM or into its own copy).  E <= 1023.  Corresponds to
 * steps 1-3 of launch_moe_permute (remap, CUB sort, offsets;
 * smxx/permute/moe_permute.cu:47-92,553-575) without step 4
 * (expand_input_rows). */
LSEK_API lsek_status lsek_moe_route(int32_t* expert_offsets, int32_t* src_to_dest_map,
                           int32_t* permuted_idx, const int32_t* topk_indices,
                           int32_t num_tokens, int32_t topk, int32_t num_experts,
                           void* stream);

/* Size of the fixed device buffer behind lsek_moe_permute_noalloc (1 MiB). */
#define LSEK_NOALLOC_PERMUTE_SCRATCH_BYTES (1u << 20)

/* lsek_moe_permute without a workspace argument and without allocating.
 * No counterpart in the reference: it exists for callers that cannot
 * allocate device memory around this call, such as plugin hosts that are
 * handed their input and output buffers by another runtime and own no
 * allocator, or runtimes that plan all device memory at start-up and treat
 * any later cudaMalloc as an error.
 * Same arguments, results and limits as lsek_moe_permute.  Its scratch is a
 * static 1 MiB device buffer inside liblsek (one per GPU that loads the
 * library, held until the process exits), which bounds the problem size:
 * ceil(num_tokens * topk / 2048) * (num_experts + 1) * 4 bytes must not
 * exceed LSEK_NOALLOC_PERMUTE_SCRATCH_BYTES (with 256 experts: up to about
 * 2.09 M slots, e.g. 261120 tokens at top-8); larger requests return
 * LSEK_ERR_INVALID_ARG without launching anything.  The first call on a
 * device looks up the buffer's device address with that device current;
 * make that first call before any stream capture on the device.  Every call
 * reuses the same buffer and needs nothing in it cleared (each call's count
 * pass overwrites every entry its later passes read), but two calls that
 * overlap on the GPU, e.g. on two streams, race on it. */
LSEK_API lsek_status lsek_moe_permute_noalloc(void* permuted_input, int32_t* expert_offsets,
                                     int32_t* src_to_dest_map, int32_t* permuted_idx,
                                     const void* hidden_states,
                                     const int32_t* topk_indices, int32_t num_tokens,
                                     int32_t topk, int32_t hidden_dim,
                                     int32_t num_experts, int32_t elem_size_bytes,
                                     void* stream);

/* Weighted unpermute.  fp32_output == 0: out [T,H] (dtype) =
 * round(sum_k fma(w[t,k], x[s2d[t,k]], acc)), fp32 accumulation in slot order.
 * fp32_output != 0: out is f32 [T,topk,H], out[t,k,:] = w[t,k]*x[s2d[t,k]]
 * (no cross-slot sum).  topk <= 32.  Replaces launch_moe_unpermute
 * (smxx/permute/moe_permute.h:79-89, moe_permute.cu:602-642). */
LSEK_API lsek_status lsek_moe_unpermute(void* output, const void* permuted_output,
                               const float* topk_weights,
                               const int32_t* src_to_dest_map,
                               int32_t num_tokens, int32_t topk,
                               int32_t hidden_dim, int32_t dtype,
                               int32_t fp32_output, void* stream);

/* Per-slot unpermute with a 16-bit payload: out [T,topk,H] (dtype),
 * out[t,k,:] = round(w[t,k] * x[s2d[t,k]]).  Replaces
 * launch_moe_unpermute_bf16_perslot (smxx/permute/moe_permute.h:100-109,
 * moe_permute.cu:644-672). */
LSEK_API lsek_status lsek_moe_unpermute_perslot(void* output,
                                       const void* permuted_output,
                                       const float* topk_weights,
                                       const int32_t* src_to_dest_map,
                                       int32_t num_tokens, int32_t topk,
                                       int32_t hidden_dim, int32_t dtype,
                                       void* stream);

/* Fixed-order slot reduce: out[t,h] = round_bf16(sum_{k=0..topk-1} in[t,k,h])
 * with the sum taken in fp32 from 0.0f in slot order.  in_dtype is
 * LSEK_FP32 or LSEK_BF16; out is bf16.  Replaces
 * launch_moe_combine_reduce_slots_fp32_to_bf16 and
 * launch_moe_combine_reduce_slots_bf16_to_bf16
 * (smxx/permute/moe_permute.h:116-134, moe_permute.cu:674-710). */
LSEK_API lsek_status lsek_moe_combine_reduce_slots(void* output_bf16,
                                          const void* input_perslot,
                                          int32_t num_tokens, int32_t topk,
                                          int32_t hidden_dim, int32_t in_dtype,
                                          void* stream);

/* ---- activation ----------------------------------------------------------- */

/* Fused SwiGLU: out [N,d] = silu(g) * u with g = in[:, :d], u = in[:, d:],
 * computed in fp32, stored in dtype.  swiglu_limit > 0 clamps
 * g = min(g, L), u = clamp(u, -L, L) first.  Replaces launch_fused_swiglu
 * (smxx/activation/fused_swiglu.h:22-27, fused_swiglu.cu:156-183). */
LSEK_API lsek_status lsek_fused_swiglu(void* output, const void* input,
                              int32_t num_tokens, int32_t d,
                              float swiglu_limit, int32_t dtype, void* stream);

/* ---- expert contraction (tcgen05 / TMEM / TMA) -------------------------- */

/* Scratch for the grouped GEMMs' work-unit counter.  With it the persistent
 * CTAs take work units dynamically, which keeps the CTAs that share a weight
 * tile in step (L2 reuse); with workspace == NULL they take a static stride.
 * The entry point zeroes the counter on the stream before the launch. */
#define LSEK_GEMM_WORKSPACE_BYTES 256

/* Grouped bf16 GEMM over experts: for each expert e,
 *   D[r, :] = A[r, :] . B[e]^T   for r in [offsets[e], offsets[e+1])
 * A [rows, K] bf16 row-major, B [E, N, K] bf16 (row-major per expert),
 * D [rows, N] bf16, fp32 accumulation.  Rows outside every expert range are
 * not written.  K % 8 == 0, N % 32 == 0, A/B/D 16-byte aligned.
 * workspace: NULL or LSEK_GEMM_WORKSPACE_BYTES of device scratch (see above).
 * The reference documents this contraction (USAGE.md:40-57) and tests it
 * with ref_grouped_gemm (tests/test_reference.py:228-254) but ships the
 * kernel in a separate library; argument order follows USAGE.md:122-126. */
LSEK_API lsek_status lsek_grouped_gemm_bf16(void* D, const void* A, const void* B,
                                   const int32_t* expert_offsets,
                                   int32_t num_experts, int32_t rows,
                                   int32_t N, int32_t K, void* workspace,
                                   size_t workspace_bytes, void* stream);

/* Gate/up grouped GEMM with the SwiGLU in its epilogue.  W_gu [E, 2I, K]
 * holds gate rows 0..I-1 and up rows I..2I-1 per expert.  For each row r of
 * expert e: g = bf16(A[r].Wg^T), u = bf16(A[r].Wu^T) and
 * Hout[r, :] = swiglu(g, u, swiglu_limit) as in lsek_fused_swiglu, so the
 * result equals lsek_grouped_gemm_bf16 followed by lsek_fused_swiglu.
 * Hout [rows, I] bf16.  I % 32 == 0. */
LSEK_API lsek_status lsek_grouped_gemm_swiglu_bf16(void* Hout, const void* A,
                                          const void* W_gu,
                                          const int32_t* expert_offsets,
                                          int32_t num_experts, int32_t rows,
                                          int32_t I, int32_t K,
                                          float swiglu_limit, void* workspace,
                                          size_t workspace_bytes, void* stream);

/* ---- expert-parallel dispatch / combine ----------------------------------- */
/* Experts are sharded over world_size ranks, rank g owning experts
 * [g*E/G, (g+1)*E/G).  These kernels prepare and consume the two all-to-all
 * exchanges (issued by the host over NCCL) of an expert-parallel layer; the
 * result equals lsek_moe_unpermute_perslot followed by
 * lsek_moe_combine_reduce_slots(bf16) on one GPU, bit for bit, for every
 * world size.  The reference specifies this canonical per-slot combine
 * (smxx/permute/moe_permute.h:67-99) and leaves the exchange to its consumer. */

/* Scratch bytes for lsek_ep_plan. */
LSEK_API size_t lsek_ep_plan_workspace_size(int32_t num_tokens, int32_t world_size);

/* Send plan: send_off [G+1] (rank g's send rows are [send_off[g],
 * send_off[g+1])), send_counts [G][2] (rows sent to rank g, and the
 * (token, slot) pairs rank g serves), pair_row [T*G] (send row of token t
 * for rank g; >= send_off[G] when t has no expert on g), row_pair [T*G]
 * (inverse map).  Rows for a rank are in token order. */
LSEK_API lsek_status lsek_ep_plan(int32_t* send_off, int32_t* send_counts, int32_t* pair_row,
                         int32_t* row_pair, const int32_t* topk_indices,
                         int32_t num_tokens, int32_t topk, int32_t num_experts,
                         int32_t world_size, void* workspace, size_t workspace_bytes,
                         void* stream);

/* Fills the send rows [send_off[G], H] bf16 with each token's hidden row,
 * and per row and slot the expert's index on the target rank (-1 when the
 * slot's expert is on another rank) and the routing weight (0 there).  The
 * buffers hold send_capacity rows (send_off[G]; rows past it are skipped). */
LSEK_API lsek_status lsek_ep_dispatch_pack(void* send_rows, int32_t* send_ids, float* send_w,
                                  int32_t send_capacity, const void* hidden, const int32_t* topk_indices,
                                  const float* topk_weights, const int32_t* pair_row,
                                  const int32_t* send_off, int32_t num_tokens,
                                  int32_t topk, int32_t hidden_dim, int32_t num_experts,
                                  int32_t world_size, void* stream);

/* slot_row [rows+1]: exclusive scan of the number of ids >= 0 per row of
 * ids [rows, topk]; slot_row[rows] = total. */
LSEK_API lsek_status lsek_ep_slot_scan(int32_t* slot_row, const int32_t* ids, int32_t rows,
                              int32_t topk, void* stream);

/* Expert-side permute of the received rows by their local expert ids: as
 * lsek_moe_permute with ids of -1 sorting last, except that rows of -1
 * slots are not copied.  permuted holds permuted_rows rows (the number of
 * valid slots; rows past it are never written). */
LSEK_API lsek_status lsek_ep_expert_permute(void* permuted, int32_t permuted_rows,
                                   int32_t* expert_offsets,
                                   int32_t* src_to_dest_map, int32_t* permuted_idx,
                                   const void* rows_in, const int32_t* local_ids,
                                   int32_t rows, int32_t topk, int32_t hidden_dim,
                                   int32_t local_experts, void* workspace,
                                   size_t workspace_bytes, void* stream);

/* Combine rows, one per valid (received row i, slot j) in received-row and
 * slot order, at slot_row[i] + (valid slots of i before j):
 * bf16(w[i,j] * expert_out[src_to_dest_map[i*topk + j]]).  comb_rows holds
 * comb_capacity rows (slot_row[rows]; rows past it are skipped). */
LSEK_API lsek_status lsek_ep_combine_pack(void* comb_rows, int32_t comb_capacity,
                                 const void* expert_out,
                                 const int32_t* src_to_dest_map, const int32_t* ids,
                                 const float* weights, const int32_t* slot_row,
                                 int32_t rows, int32_t topk, int32_t hidden_dim,
                                 void* stream);

/* Sender side: out[t] = bf16(sum over slots j in order of the returned
 * combine row of (t, j)), fp32 accumulation from 0; comb_rows holds the
 * comb_count rows returned by all ranks in send-row order (never read past
 * them), slot_row the scan of the sent ids. */
LSEK_API lsek_status lsek_ep_combine_reduce(void* out, const void* comb_rows,
                                   int32_t comb_count, const int32_t* topk_indices, const int32_t* pair_row,
                                   const int32_t* slot_row, int32_t num_tokens,
                                   int32_t topk, int32_t hidden_dim, int32_t num_experts,
                                   int32_t world_size, void* stream);

/* ---- expert-parallel over peer memory (NVLink) ---------------------------- */
/* The same dispatch and combine with the exchanges done by the kernels
 * themselves: every rank of one node allocates a symmetric buffer (a domain),
 * the ranks swap its CUDA IPC handle once, and from then on the dispatch
 * kernel stores token rows straight into the owner ranks' buffers and the
 * down-projection GEMM stores each weighted per-slot row straight into the
 * source rank's buffer, so the NVLink transfer overlaps the math.  Kernels
 * publish with an epoch flag per rank; the waits are bounded (an expired wait
 * records a device error, see lsek_device_error).  No counterpart in the
 * reference (its consumer models the exchange as an all-reduce,
 * tests/test_kernels.py:131-142, 187-200). */

typedef struct lsek_ep_domain lsek_ep_domain;
#define LSEK_EP_MAX_RANKS 16
#define LSEK_EP_HANDLE_BYTES 64

/* Bytes of one rank's symmetric buffer. */
LSEK_API size_t lsek_ep_domain_bytes(int32_t max_tokens, int32_t hidden_dim, int32_t topk,
                            int32_t world_size);
/* Allocates this rank's buffer on the current device (zeroed). */
LSEK_API lsek_status lsek_ep_domain_create(lsek_ep_domain** out, int32_t rank, int32_t world_size,
                                  int32_t max_tokens, int32_t hidden_dim, int32_t topk);
/* The CUDA IPC handle of this rank's buffer (LSEK_EP_HANDLE_BYTES). */
LSEK_API lsek_status lsek_ep_domain_export(const lsek_ep_domain* d, void* handle,
                                  size_t handle_bytes);
/* Maps rank `peer`'s buffer from its exported handle. */
LSEK_API lsek_status lsek_ep_domain_import(lsek_ep_domain* d, int32_t peer, const void* handle,
                                  size_t handle_bytes);
/* This rank's receive views: rows [cap_rows, H] bf16, ids / weights
 * [cap_rows, topk], and the combine rows [cap_slots, H] bf16. */
LSEK_API lsek_status lsek_ep_domain_buffers(const lsek_ep_domain* d, void** recv_rows,
                                   int32_t** recv_ids, float** recv_w, void** back,
                                   int64_t* cap_rows, int64_t* cap_slots);
/* Synchronises the device, unmaps the peers and frees the buffer. */
LSEK_API void lsek_ep_domain_destroy(lsek_ep_domain* d);

/* Dispatch: stores each token row (and its per-slot local ids and weights)
 * into the receive buffer of every rank owning one of its experts, writes
 * the ids of the send rows to the local send_ids [send_capacity, topk], and
 * publishes dispatch epoch `epoch` to every rank.  counts [G][G][2] (host)
 * holds every rank's send_counts from lsek_ep_plan. */
LSEK_API lsek_status lsek_ep_dispatch_push(lsek_ep_domain* d, int32_t* send_ids,
                                  int32_t send_capacity, const int32_t* counts,
                                  const void* hidden, const int32_t* topk_indices,
                                  const float* topk_weights, const int32_t* pair_row,
                                  const int32_t* send_off, int32_t num_tokens,
                                  int32_t num_experts, uint32_t epoch, void* stream);
/* Copies `bytes` (a multiple of 4) of device memory into page-locked host
 * memory with a kernel that stores through the host buffer's device mapping,
 * so the copy never queues behind a large device-to-host transfer on another
 * stream (the copy engine serves those in order).  Used to read the
 * expert-parallel counts while the previous batch's output is being copied
 * out.  host_dst must be page-locked (cudaHostAlloc or cudaHostRegister);
 * the data is in place once the stream has passed this call.  No
 * counterpart in the reference (its host reads go through torch copies). */
LSEK_API lsek_status lsek_copy_to_mapped_host(void* host_dst, const void* dev_src, size_t bytes,
                                              void* stream);
/* Waits on the stream until every rank has published `epoch` for the
 * dispatch (what = 0), the combine (what = 1) or chunk c of a token-chunked
 * combine (what = 2 + c, c < 16); gives up after timeout_ns (<= 0: 2 s) and
 * records a device error. */
LSEK_API lsek_status lsek_ep_wait(lsek_ep_domain* d, int32_t what, uint32_t epoch,
                         int64_t timeout_ns, void* stream);
/* Per permuted row of the received slots: the source rank, the row of its
 * combine buffer and the weight (from the domain's recv ids / weights and
 * the expert permute's src_to_dest_map; slot_row = lsek_ep_slot_scan of the
 * received ids). */
LSEK_API lsek_status lsek_ep_combine_plan(lsek_ep_domain* d, int32_t* dst_rank, int32_t* dst_row,
                                 float* dst_w, const int32_t* src_to_dest_map,
                                 const int32_t* slot_row, const int32_t* counts,
                                 int32_t recv_rows, int32_t valid_slots, void* stream);
/* The combine of expert outputs already in memory (no GEMM in front):
 * bf16(dst_w[p] * expert_out[p]) to row dst_row[p] of rank dst_rank[p]'s
 * combine buffer for p < rows (or for *row_lo <= p < *row_hi when both
 * device pointers are given, e.g. two entries of the expert offsets, so the
 * rows of some experts can go while the GEMM computes the others); then,
 * if `publish`, publishes combine epoch `epoch` (the last of a series of
 * calls publishes once every row has been stored). */
LSEK_API lsek_status lsek_ep_combine_push(lsek_ep_domain* d, const void* expert_out,
                                 const int32_t* dst_rank, const int32_t* dst_row,
                                 const float* dst_w, int32_t rows, const int32_t* row_lo,
                                 const int32_t* row_hi, int32_t publish, uint32_t epoch,
                                 void* stream);
/* Token-chunked combine, step 1: lsek_ep_combine_plan that also lists the
 * rows of every token chunk.  Chunk c holds the permuted rows p whose source
 * token t (the token's index on the rank that sent it) has
 * t / chunk_tokens == c (capped at chunks - 1).  List c is
 * order[c * valid_slots ...], order_count[c] entries long, in no particular
 * order; order has chunks * valid_slots entries, order_count chunks.  Every
 * rank must use the same chunk_tokens and chunks (e.g. from the domain's
 * max_tokens), so chunk c of every source covers the same token range.
 * chunks in [1, 16].  No counterpart in the reference. */
LSEK_API lsek_status lsek_ep_combine_plan_chunks(lsek_ep_domain* d, int32_t* dst_rank,
                                        int32_t* dst_row, float* dst_w, int32_t* order,
                                        int32_t* order_count, const int32_t* src_to_dest_map,
                                        const int32_t* slot_row, const int32_t* counts,
                                        int32_t recv_rows, int32_t valid_slots,
                                        int32_t chunk_tokens, int32_t chunks, void* stream);
/* Token-chunked combine, step 2: lsek_ep_combine_push restricted to the rows
 * of chunk `chunk`'s list from lsek_ep_combine_plan_chunks (rows =
 * valid_slots there; with *row_lo <= p < *row_hi also when given), which
 * then publishes combine-chunk epoch `epoch` (lsek_ep_wait what = 2 + chunk).
 * A source can reduce chunk c's tokens (lsek_ep_combine_reduce on that token
 * range) once every rank has published chunk c, while later chunks are still
 * in flight.  Rows of earlier non-publishing pushes on the same stream are
 * ordered before the flag.  No counterpart in the reference. */
LSEK_API lsek_status lsek_ep_combine_push_chunk(lsek_ep_domain* d, const void* expert_out,
                                       const int32_t* dst_rank, const int32_t* dst_row,
                                       const float* dst_w, int32_t rows, const int32_t* row_lo,
                                       const int32_t* row_hi, const int32_t* order,
                                       const int32_t* order_count, int32_t chunk, uint32_t epoch,
                                       void* stream);
/* Down-projection GEMM with the combine fused into its epilogue: for each
 * permuted row p, bf16(dst_w[p] * bf16(H[p] . W_down[e]^T)) goes to row
 * dst_row[p] of rank dst_rank[p]'s combine buffer; then publishes combine
 * epoch `epoch` to every rank.  H [rows, I] bf16, W_down [E_local, hidden, I]. */
LSEK_API lsek_status lsek_ep_down_gemm_combine(lsek_ep_domain* d, const void* h, const void* w_down,
                                      const int32_t* expert_offsets, int32_t local_experts,
                                      int32_t rows, int32_t inter, const int32_t* dst_rank,
                                      const int32_t* dst_row, const float* dst_w,
                                      uint32_t epoch, void* workspace, size_t workspace_bytes,
                                      void* stream);

/* ---- whole MoE layer ------------------------------------------------------ */

/* Scratch bytes for lsek_moe_layer_forward. */
LSEK_API size_t lsek_moe_layer_workspace_size(int32_t num_tokens, int32_t hidden_dim,
                                     int32_t inter_dim, int32_t num_experts,
                                     int32_t topk);

/* Number of stages of lsek_moe_layer_forward, for stage_events. */
#define LSEK_LAYER_STAGES 6

/* DeepSeek-V3-style routed-expert layer, all on `stream`:
 *   topk_gating -> route -> row copy -> gate/up GEMM + SwiGLU ->
 *   down GEMM -> weighted unpermute.
 * hidden [T,H] bf16, logits [T,E] f32, bias [E] f32 or NULL,
 * W_gu [E, 2I, H] bf16, W_down [E, H, I] bf16, out [T,H] bf16.
 * topk_weights/topk_indices ([T,topk]) may be NULL; when given they receive
 * the routing.  stage_events is NULL or an array of LSEK_LAYER_STAGES + 1
 * cudaEvent_t that are recorded on `stream` before each stage and after the
 * last, for per-stage timing.  The composition follows the reference's
 * documented flow (USAGE.md:40-57) with the oracle ref_expert_forward
 * (tests/test_reference.py:257-276) generalised to top-k. */
LSEK_API lsek_status lsek_moe_layer_forward(
    void* out, const void* hidden, const float* logits, const float* bias,
    const void* W_gu, const void* W_down, const lsek_topk_gating_params* gp,
    int32_t hidden_dim, int32_t inter_dim, float swiglu_limit,
    float* topk_weights, int32_t* topk_indices, void* workspace,
    size_t workspace_bytes, void* const* stage_events, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* LSEK_H_ */
