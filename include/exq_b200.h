/*
 * exq_b200.h -- C ABI of the B200-native quantized MoE expert path.
 *
 * Drop-in replacement for the GPU hot path of alityb/exq: the
 * `exq_dispatch_cuda` extension (exq/kernels/cuda_src/exq_dispatch.cu), the
 * sgl_kernel steps the SGLang backend calls (`moe_align_block_size`,
 * `silu_and_mul`, exq/runtime/sglang_backend.py:79,:108-109,:140) and the
 * Triton INT4/FP16 grouped GEMMs of exq/kernels (moe_int4_kernel.py,
 * moe_grouped_gemm.py).
 *
 * Conventions
 *  - Every entry point takes plain device pointers, sizes and dtype tags and a
 *    `stream` (a cudaStream_t passed as void*; NULL = legacy default stream).
 *  - Work is only enqueued: nothing synchronises, nothing allocates, and every
 *    launch is capturable in a CUDA graph.  Temporary storage is a
 *    caller-provided workspace sized by the matching *_workspace_bytes query.
 *  - Outputs are caller-preallocated, as in the reference.
 *  - Return value: EXQ_OK (0) or a negative EXQ_ERR_* code;
 *    exq_last_error() gives a message (thread-local).  Argument errors are
 *    detected on the host before anything is enqueued.  Conditions that can
 *    only be seen on the device (an expert id out of range) are recorded in
 *    the device status word, read with exq_read_device_status().
 */
#ifndef EXQ_B200_H_
#define EXQ_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define EXQ_API __attribute__((visibility("default")))
#else
#define EXQ_API
#endif

#define EXQ_ABI_VERSION 1

/* status codes */
#define EXQ_OK 0
#define EXQ_ERR_INVALID -1     /* bad argument (shape, dtype, null pointer) */
#define EXQ_ERR_UNSUPPORTED -2 /* valid but not implemented (e.g. group size) */
#define EXQ_ERR_CUDA -3        /* a CUDA runtime call or launch failed */
#define EXQ_ERR_WORKSPACE -4   /* workspace missing or too small */

/* dtype tags */
#define EXQ_F16 0
#define EXQ_BF16 1
#define EXQ_F32 2
#define EXQ_I32 3
#define EXQ_I64 4
#define EXQ_U8 5
#define EXQ_I8 6

/* weight tiers, numbered as exq/kernels/exq_artifact.py:25 PRECISION_TO_INT */
#define EXQ_TIER_BF16 0 /* 16-bit weights in the activation dtype */
#define EXQ_TIER_INT8 1 /* int8 [N,K] + fp16 per-row scale [N] */
#define EXQ_TIER_INT4 2 /* u8 [N,K/2] (q+8 nibbles, even k low) + fp16 [N,K/128] */
#define EXQ_TIER_NONE -1

/* device status bits (exq_read_device_status) */
#define EXQ_DEV_BAD_EXPERT_ID 1u /* an id outside [0, n_experts) was dropped */
#define EXQ_DEV_BAD_SLOT 2u      /* a sort_order / slot entry was out of range */
#define EXQ_DEV_BAD_TIER 4u      /* an expert descriptor had an unknown tier */
#define EXQ_DEV_TIMEOUT 8u       /* a pipeline wait gave up (the kernel unwound) */

EXQ_API int exq_abi_version(void);
EXQ_API const char* exq_last_error(void);
EXQ_API const char* exq_status_string(int status);

/* Reads (synchronously, on `stream`) and optionally clears the device status
 * word that kernels OR their EXQ_DEV_* bits into.  Debug/validation helper,
 * not for hot paths. */
EXQ_API int exq_read_device_status(uint32_t* status_out, int clear, void* stream);

/* ---------------------------------------------------------------- routing */

/* sgl_kernel.moe_align_block_size (called at exq/runtime/sglang_backend.py:102-109).
 * Counts the flat top-k ids over `num_experts` buckets, pads each count to a
 * multiple of `block_size`, writes every slot index into its expert's range
 * (ascending slot order within an expert), pads with `numel`, writes the
 * owner expert of every block (-1 beyond num_tokens_post_pad/block_size), the
 * padded total and the exclusive padded prefix `cumsum_buffer[num_experts+1]`.
 * With pad_sorted_token_ids = 0 the positions not holding a slot are left
 * untouched (the caller pre-fills them). */
EXQ_API int exq_moe_align_block_size(const void* topk_ids, int ids_dtype, int64_t numel,
                             int32_t num_experts, int32_t block_size,
                             int32_t* sorted_token_ids, int64_t sorted_cap,
                             int32_t* expert_ids, int64_t expert_ids_cap,
                             int32_t* num_tokens_post_pad, int32_t* cumsum_buffer,
                             int32_t pad_sorted_token_ids, void* stream);

/* exq_dispatch_cuda.build_ends_from_slots (exq/kernels/cuda_src/exq_dispatch.cu:181-229).
 * From align output `sorted_slot_ids[em]` (entries >= n_active are padding) and
 * `flat_router[n_active]` (expert of each flat slot): expert_ends[E+1]
 * (exclusive prefix of per-expert counts) and sort_order[n_active] (int64,
 * valid slots compacted per expert in order of appearance).  One launch. */
EXQ_API int exq_build_ends_from_slots(const int32_t* sorted_slot_ids, int64_t em,
                              const int32_t* flat_router, int64_t n_active,
                              int32_t n_experts, int32_t* expert_ends,
                              int64_t* sort_order, void* stream);

/* exq_dispatch_cuda.dispatch (exq_dispatch.cu:99-149): stable sort of the flat
 * top-k ids by expert.  sort_order[n] and sorted_expert_ids[n] are int64,
 * expert_ends[E+1] int32.  One launch, no temporary storage. */
EXQ_API int exq_dispatch(const void* router_indices, int ids_dtype, int64_t n, int32_t n_experts,
                 int64_t* sort_order, int64_t* sorted_expert_ids, int32_t* expert_ends,
                 void* stream);

/* exq_dispatch_cuda.gather_hidden (exq_dispatch.cu:234-260):
 * out[i, :] = hidden[sort_order[i] / top_k, :].  fp16 and bf16 (the reference
 * takes fp16 only).  `row_stride` is hidden's row stride in elements. */
EXQ_API int exq_gather_hidden(const void* hidden, int dtype, int64_t n_tokens, int64_t hidden_size,
                      int64_t row_stride, const int64_t* sort_order, int64_t n_active,
                      int32_t top_k, void* out, void* stream);

/* exq_dispatch_cuda.combine (exq_dispatch.cu:263-310):
 * result[t, :] = sum_j w[t, j] * down_out[pos(t*k + j), :] with pos the
 * inverse of sort_order; fp32 products and sum in top-k order, one rounding
 * to the output dtype.  Deterministic (the reference uses fp32 atomics).
 * Weights may be fp32, fp16 or bf16 (the reference reads fp16 only). */
EXQ_API size_t exq_combine_workspace_bytes(int64_t n_active);
EXQ_API int exq_combine(const void* down_out, int dtype, int64_t n_active, int64_t hidden_size,
                const int64_t* sort_order, const void* router_weights, int w_dtype,
                int64_t n_tokens, int32_t top_k, void* result, int out_dtype,
                void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- expert parallelism */

/* No counterpart in the reference (its layer runs whole on one GPU,
 * exq/runtime/sglang_backend.py:65-158).  The send side of the NCCL
 * expert-parallel exchange of exq_b200/ep.py: the T*k slots of topk_ids
 * [T, k], grouped by destination rank d = expert / experts_per_rank in
 * ascending slot order, become send_rows [T*k, hidden_size] (the hidden row
 * of each slot, same dtype), send_ids[r] (the expert index local to the
 * destination), slot_row[slot] (send row of the slot, -1 if its expert id is
 * out of range: dropped and flagged in the device status) and
 * counts[n_ranks] (rows per destination).  At most 4096 slots and 64 ranks;
 * hidden_size % 8 == 0. */
EXQ_API int exq_ep_pack(const void* topk_ids, int ids_dtype, int64_t n_tokens, int32_t top_k,
                        int32_t experts_per_rank, int32_t n_ranks, const void* hidden, int dtype,
                        int64_t hidden_size, void* send_rows, int32_t* send_ids,
                        int32_t* slot_row, int32_t* counts, void* stream);

/* No counterpart in the reference.  The receive side of the exchange:
 * out[t, :] = base[t, :] + sum_j weights[t, j] * rows[slot_row[t*k + j], :]
 * (fp32 in slot order, one rounding; base may be NULL; slot_row < 0 skipped).
 * rows, base and out share dtype (fp16/bf16); weights fp32/fp16/bf16. */
EXQ_API int exq_ep_combine(const void* rows, int dtype, const int32_t* slot_row,
                           const void* weights, int w_dtype, int64_t n_tokens, int32_t top_k,
                           int64_t hidden_size, const void* base, void* out, void* stream);

/* No counterpart in the reference.  exq_combine without a workspace argument:
 * the inverse-permutation scratch is a static device array of
 * EXQ_COMBINE_NOALLOC_MAX_ACTIVE int32 slots (1 MiB per device) inside this
 * library, so the call allocates no memory (no cudaMalloc, no allocating
 * library).  For callers that hold only the input and output pointers and no
 * device allocator, e.g. a plain C binding of the reference's combine.
 * - n_active above the maximum returns EXQ_ERR_INVALID with a message.
 * - The scratch is one per device and shared: calls on the same device that
 *   overlap in time (different streams or host threads) race on it.
 * - The first call on each device looks the scratch address up (and may load
 *   the module); make it before any stream capture begins.
 * - Nothing has to start zeroed: each call fills what it uses on `stream`.
 * Results are identical to exq_combine. */
#define EXQ_COMBINE_NOALLOC_MAX_ACTIVE 262144
EXQ_API int exq_combine_noalloc(const void* down_out, int dtype, int64_t n_active,
                                int64_t hidden_size, const int64_t* sort_order,
                                const void* router_weights, int w_dtype, int64_t n_tokens,
                                int32_t top_k, void* result, int out_dtype, void* stream);

/* Router top-k, the step before the expert path: the reference's generated
 * MoE layers compute it as softmax -> torch.topk -> divide by the sum
 * (exq/codegen/triton_emitter.py:273-276), and SGLang hands the result to
 * _exq_forward_cuda as topk_output (exq/runtime/sglang_backend.py:88-90).
 * Per token: p = softmax(logits) in fp32, the top_k largest p in descending
 * order (equal p: the lower expert id first), and with renormalize != 0 the
 * selected p divided by their sum (summed in that order).
 * logits [n_tokens, n_experts] fp32/fp16/bf16, row stride n_experts;
 * 1 <= n_experts <= 1024; 1 <= top_k <= min(32, n_experts).
 * Out: topk_ids int32 [n_tokens, top_k], topk_weights fp32 [n_tokens, top_k]
 * (the ids/weights arguments of exq_moe_layer_forward). */
EXQ_API int exq_router_topk(const void* logits, int logits_dtype, int64_t n_tokens,
                            int32_t n_experts, int32_t top_k, int32_t renormalize,
                            int32_t* topk_ids, float* topk_weights, void* stream);

/* sgl_kernel.silu_and_mul (exq/runtime/sglang_backend.py:138-140):
 * out[m, i] = silu(x[m, i]) * x[m, I + i], fp32 math. */
EXQ_API int exq_silu_and_mul(const void* input, void* out, int dtype, int64_t m, int64_t inter,
                     void* stream);

/* ---------------------------------------------------------------- packing */

/* pack_int4_weights / pack_experts_int4 (exq/kernels/moe_int4_kernel.py:37-119),
 * on the GPU, bit-exact: rows x k matrix (fp16/bf16/fp32) -> packed u8
 * [rows, k/2] + fp16 scales [rows, k/group]; group = k when k < group_size. */
EXQ_API int exq_pack_int4(const void* w, int dtype, int64_t rows, int64_t k, int32_t group_size,
                  uint8_t* packed, void* scales_f16, void* stream);

/* The INT8 tier of a quant plan (exq/eval/quant_shim.py:84-96 semantics, scale
 * stored as fp16): int8 [rows, k] + fp16 per-row scale [rows]. */
EXQ_API int exq_quant_int8(const void* w, int dtype, int64_t rows, int64_t k, int8_t* q,
                   void* scales_f16, void* stream);

/* ------------------------------------------------------ grouped expert GEMMs */

/* One expert's weights in one of the three tiers.  Pointers are device
 * pointers; the array of descriptors itself lives in device memory. */
typedef struct exq_expert_desc {
  int32_t tier;           /* EXQ_TIER_* ; EXQ_TIER_NONE = expert absent */
  int32_t reserved;
  const void* w13;        /* gate_up [2I, H] in the tier's format */
  const void* w13_scales; /* INT4: f16 [2I, H/128]; INT8: f16 [2I]; BF16: NULL */
  const void* w2;         /* down [H, I] */
  const void* w2_scales;  /* INT4: f16 [H, I/128]; INT8: f16 [H]; BF16: NULL */
} exq_expert_desc;

/* The Triton `_moe_gemm_int4_kernel` / `_moe_gemm_kernel` launches of
 * moe_int4_forward (moe_int4_kernel.py:245-327) and moe_grouped_gemm
 * (moe_grouped_gemm.py:173-227), with the token sort and the hidden-state
 * gather fused in: out[i, :] = hidden[sort_order[i] / top_k] . W[e_i]^T in
 * expert-sorted (stable) order, fp32 accumulation.
 * `experts` is a device array of n_experts descriptors; only `w13` /
 * `w13_scales` are read, as a single [n_rows, k] projection.  The output
 * dtype is fp16 or bf16.  Optional `sort_order_out` (int64 [n]) and
 * `expert_ends_out` (int32 [E+1]) receive the routing metadata. */
EXQ_API size_t exq_moe_gemm_workspace_bytes(int64_t n_tokens, int32_t top_k, int32_t n_experts);
EXQ_API int exq_moe_gemm(const exq_expert_desc* experts, int32_t n_experts, int64_t n_rows,
                 int64_t k, const void* hidden, int act_dtype, int64_t n_tokens,
                 const void* topk_ids, int ids_dtype, int32_t top_k, void* out,
                 int out_dtype, int64_t* sort_order_out, int32_t* expert_ends_out,
                 void* workspace, size_t workspace_bytes, void* stream);

/* Packed weights of one MoE layer for the tcgen05 path, one contiguous
 * storage per tier.  Experts [0, n_routed) are routed; [n_routed,
 * n_routed + n_shared) are shared experts applied to every token with weight 1.
 * expert_slot (device, int32 [n_routed + n_shared]) = tier << 24 | index of
 * the expert inside its tier storage.  Layouts (H = hidden, I = inter; inside
 * each 8-element octet of k the "permuted" order is [0,4,1,5,2,6,3,7]):
 *   INT4: w13 u8 [n, 2I, H/2] and w2 u8 [n, H, I/2] in the reference nibble
 *         format (moe_int4_kernel.py:37-93); scales f16 group-major
 *         w13_scales [n, H/128, 2I], w2_scales [n, I/128, H]
 *   INT8: w13 i8 [n, 2I, H], w2 i8 [n, H, I], bytes octet-permuted; per-row f16
 *         scales w13_scales [n, 2I], w2_scales [n, H]
 *   BF16: w13 f16 [n, 2I, H], w2 f16 [n, H, I], octet-permuted; no scales
 * Requirements: H % 128 == 0, I % 128 == 0, every storage pointer 16-byte
 * aligned. */
typedef struct exq_moe_weights {
  int32_t n_routed;
  int32_t n_shared;
  int64_t hidden;
  int64_t inter;
  int32_t n_tier[3];            /* experts per tier storage, indexed by EXQ_TIER_* */
  int32_t reserved;
  const void* w13[3];
  const void* w13_scales[3];
  const void* w2[3];
  const void* w2_scales[3];
  const int32_t* expert_slot;
} exq_moe_weights;

/* The whole MoE layer of exq/runtime/sglang_backend.py:65-158 (and
 * moe_int4_full_forward, moe_int4_kernel.py:330-426): route -> activation
 * prep (gather + fp16 + octet permutation) -> one tcgen05 grouped-GEMM launch
 * that runs gate_up with fused SiLU*mul, then down (each down tile starts when
 * its gate_up row blocks are stored), and the deterministic router-weighted
 * top-k combine.  The experts may mix the three tiers.
 * hidden_states/out: [n_tokens, hidden] (fp16 or bf16; the matrix products
 * run on fp16 operands with fp32 accumulation, as the reference's kernel
 * does); topk_ids [n_tokens, top_k] int32/int64, where a negative id marks an
 * unused slot (no expert) and an id >= n_routed is dropped and flagged
 * (EXQ_DEV_BAD_EXPERT_ID); topk_weights [n_tokens, top_k] f32/f16/bf16.  Up
 * to 16384 slots and 1024 experts: two launches (route fused with prep; the
 * GEMM launch with the combine at its end); above: route, prep, GEMM, and
 * the combine apart when the GEMM launch cannot stage it.  No host
 * synchronisation. */
EXQ_API size_t exq_moe_layer_workspace_bytes(int64_t n_tokens, int32_t top_k, int32_t n_shared,
                                             int32_t n_experts_total, int64_t hidden,
                                             int64_t inter);
EXQ_API int exq_moe_layer_forward(const exq_moe_weights* weights, const void* hidden_states,
                                  int act_dtype, int64_t n_tokens, const void* topk_ids,
                                  int ids_dtype, const void* topk_weights, int w_dtype,
                                  int32_t top_k, void* out, void* workspace,
                                  size_t workspace_bytes, void* stream);

/* The same layer, launching only its stages [first_stage, end_stage):
 * 0 = route (sort + tile list), 1 = activation prep, 2 = gate_up GEMM,
 * 3 = down GEMM, 4 = top-k combine.  Stages communicate through `workspace`,
 * so a caller may run them separately on one stream (per-kernel timing) with
 * identical arguments, each stage once and in order after stage 0;
 * exq_moe_layer_forward = stages [0, 5).  Stages 2 and 3 in one range are one
 * launch; with stage 4 too (up to 16384 slots), the combine runs in it. */
#define EXQ_LAYER_STAGES 5
EXQ_API int exq_moe_layer_forward_range(const exq_moe_weights* weights,
                                        const void* hidden_states, int act_dtype,
                                        int64_t n_tokens, const void* topk_ids, int ids_dtype,
                                        const void* topk_weights, int w_dtype, int32_t top_k,
                                        void* out, void* workspace, size_t workspace_bytes,
                                        void* stream, int32_t first_stage, int32_t end_stage);

/* The layer from router logits: exq_router_topk (softmax -> top_k -> optional
 * renormalisation over the n_routed experts; the step SGLang performs before
 * _exq_forward_cuda, exq/runtime/sglang_backend.py:88-90) feeding
 * exq_moe_layer_forward, in one call.  logits [n_tokens, n_routed]
 * fp32/fp16/bf16.  The router's int32 ids and fp32 weights live in the
 * workspace (exq_moe_layer_from_logits_workspace_bytes), after the layer's
 * own.  The routing launch is chained programmatically to the router. */
EXQ_API size_t exq_moe_layer_from_logits_workspace_bytes(int64_t n_tokens, int32_t top_k,
                                                         int32_t n_shared,
                                                         int32_t n_experts_total, int64_t hidden,
                                                         int64_t inter);
EXQ_API int exq_moe_layer_forward_from_logits(const exq_moe_weights* weights,
                                              const void* hidden_states, int act_dtype,
                                              int64_t n_tokens, const void* router_logits,
                                              int logits_dtype, int32_t top_k,
                                              int32_t renormalize, void* out, void* workspace,
                                              size_t workspace_bytes, void* stream);

/* ------------------------------------------------ expert parallelism over peer memory
 *
 * No counterpart in the reference.  The exchange without NCCL or a host sync:
 * every rank holds one "EP buffer" (exq_ep_buffer_bytes), shared with the
 * other ranks of one node through CUDA IPC, and `peers` is a DEVICE array of
 * the n_ranks buffer addresses as mapped in this process (peers[rank] = own).
 * One buffer: a header of arrival flags, then, for n_ranks * capacity rows,
 * the received local expert ids (int32, -1 = unused), a column of 1.0f, the
 * received hidden rows and the returned expert output rows.  Block s of
 * `capacity` rows belongs to source rank s.  A step is, in stream order on
 * every rank: exq_ep_dispatch -> (shared experts) -> exq_ep_expert_forward
 * -> exq_ep_combine_peer.  Every rank must make the same calls in the same
 * order.  Waits on other ranks are bounded (5 s unless exq_ep_set_wait_timeout
 * says otherwise): on expiry the kernel sets EXQ_DEV_TIMEOUT in the device
 * status and marks the buffer failed, after which this rank's kernels neither
 * read the rows of that step nor send any back, so the peers' waits run out
 * too.  The caller reads the status (exq_read_device_status) and, after a
 * timeout, re-initialises every rank's buffer (exq_ep_buffer_init, with the
 * same barrier as at set-up) before the next step. */
#define EXQ_IPC_HANDLE_BYTES 64

/* The limit of every wait on another rank in the EP kernels launched after
 * this call, in nanoseconds (0: the default of 5 s).  Process-wide; a CUDA
 * graph keeps the limit it was captured with.  No counterpart in the
 * reference (its layer has no expert parallelism). */
EXQ_API int exq_ep_set_wait_timeout(uint64_t ns);

/* Bytes of one rank's EP buffer; 0 for invalid sizes. */
EXQ_API size_t exq_ep_buffer_bytes(int32_t n_ranks, int64_t capacity, int64_t hidden_size);

/* Clears the flags, the step counter, the failed mark and the ids and writes
 * the 1.0f column of a fresh buffer (or of one whose exchange timed out).
 * Every rank must finish it (stream synchronised, then a group barrier)
 * before any rank's next exq_ep_dispatch. */
EXQ_API int exq_ep_buffer_init(void* buffer, int32_t n_ranks, int64_t capacity,
                               int64_t hidden_size, void* stream);

/* cudaMalloc of `bytes` plus its IPC handle (EXQ_IPC_HANDLE_BYTES bytes
 * written to handle_out); exq_ep_ipc_free releases it. */
EXQ_API int exq_ep_ipc_alloc(size_t bytes, void** ptr_out, void* handle_out);
EXQ_API int exq_ep_ipc_free(void* ptr);
/* Maps another process's buffer on the current device (peer access enabled
 * lazily); exq_ep_ipc_close unmaps it. */
EXQ_API int exq_ep_ipc_open(const void* handle, void** ptr_out);
EXQ_API int exq_ep_ipc_close(void* ptr);

/* One launch: groups this rank's T*k slots by destination rank (as
 * exq_ep_pack) and writes each slot's hidden row and local expert id straight
 * into block `rank` of the destination's buffer (NVLink stores), fills the
 * rest of every block's ids with -1, then raises this rank's arrival flag in
 * every destination.  slot_row[slot] = d * capacity + q, the row of this
 * rank's return area that rank d fills for the slot (-1: dropped id).
 * n_tokens <= capacity / top_k is the caller's contract; a destination past
 * its capacity is flagged EXQ_DEV_BAD_SLOT and its extra rows dropped.
 * At most 4096 slots and 64 ranks; hidden_size % 8 == 0. */
EXQ_API int exq_ep_dispatch(const void* topk_ids, int ids_dtype, int64_t n_tokens, int32_t top_k,
                            int32_t experts_per_rank, int32_t n_ranks, int32_t rank,
                            const void* hidden, int dtype, int64_t hidden_size, int64_t capacity,
                            void* const* peers, int32_t* slot_row, void* stream);

/* Waits for every rank's arrival flag, runs this rank's routed experts
 * (`weights`, no shared experts) on all n_ranks * capacity received rows
 * (the layer of exq_moe_layer_forward with top_k 1 and weight 1; unused rows
 * carry id -1 and cost nothing in the GEMMs), then writes each output row,
 * rounded to `dtype`, into its source rank's return area (NVLink stores) and
 * raises this rank's return flag there.  workspace: exq_moe_layer_workspace_bytes(
 * n_ranks * capacity, 1, 0, n_routed, hidden, inter). */
EXQ_API int exq_ep_expert_forward(const exq_moe_weights* weights, int dtype, int32_t n_ranks,
                                  int32_t rank, int64_t capacity, void* buffer,
                                  void* const* peers, void* workspace, size_t workspace_bytes,
                                  void* stream);

/* exq_ep_expert_forward with the shared experts folded in.  `weights` holds
 * this rank's routed experts followed by the n_shared shared experts, all as
 * routed experts (n_shared field 0).  This rank's n_tokens rows of `hidden`
 * go into its own block of the receive area (block n_ranks), one row per
 * (token, shared expert), and the layer runs once on the received rows and
 * that block; the received rows' outputs return to their sources as in
 * exq_ep_expert_forward, and shared_out [n_tokens, hidden] (`dtype`) receives
 * the shared experts' summed output, rounded once (the `base` of
 * exq_ep_combine_peer).  n_tokens * n_shared <= capacity.  workspace:
 * exq_moe_layer_workspace_bytes((n_ranks + 1) * capacity, 1, 0, n_routed,
 * hidden, inter). */
EXQ_API int exq_ep_expert_forward_shared(const exq_moe_weights* weights, int dtype,
                                         int32_t n_ranks, int32_t rank, int64_t capacity,
                                         void* buffer, void* const* peers, const void* hidden,
                                         int64_t n_tokens, int32_t n_shared, void* shared_out,
                                         void* workspace, size_t workspace_bytes, void* stream);

/* Waits for every rank's return flag, then
 * out[t] = base[t] + sum_j weights[t, j] * returned[slot_row[t*k + j]]
 * as exq_ep_combine (base may be NULL). */
EXQ_API int exq_ep_combine_peer(const void* buffer, int32_t n_ranks, int64_t capacity,
                                int64_t hidden_size, int dtype, const int32_t* slot_row,
                                const void* weights, int w_dtype, int64_t n_tokens,
                                int32_t top_k, const void* base, void* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* EXQ_B200_H_ */
