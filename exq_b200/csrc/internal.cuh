// Internal kernel parameter blocks and launchers shared by the .cu files.
#pragma once

#include "common.cuh"

namespace exq {

// Programmatic dependent launch.  A kernel launched with launch_pdl(true, ...)
// may start while its predecessor in the stream is still running: it must call
// pdl_wait() before touching anything the predecessor writes, and calls
// pdl_trigger() to let its own successor launch early.  Both are no-ops for
// ordinary launches (launch_pdl(false, ...)).  Only a kernel whose stream
// predecessor is another kernel of the same call is launched programmatically:
// the first kernel of a call may follow a copy or a wait on another stream's
// event (an NCCL collective), which griddepcontrol.wait does not cover.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(bool pdl, void (*kernel)(KArgs...), dim3 grid, dim3 block,
                              size_t smem, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}


// ----------------------------------------------------------------- routing
enum RouteMode : int {
  kRouteAlign = 0,      // sgl_kernel moe_align_block_size
  kRouteEndsFromSlots,  // exq_build_ends_from_slots
  kRouteDispatch,       // exq_dispatch
  kRouteLayer,          // GEMM tile list (optionally with shared experts)
};

struct RouteParams {
  // inputs
  const void* ids;  // ALIGN / DISPATCH / LAYER: flat top-k ids
  int ids_dtype;
  const int32_t* slot_ids;     // ENDS_FROM_SLOTS: align output
  const int32_t* flat_router;  // ENDS_FROM_SLOTS
  int64_t n;                   // number of elements walked
  int64_t n_active;            // ENDS_FROM_SLOTS: valid slot bound
  int n_buckets;               // buckets counted (experts incl. shared)
  int n_routed;                // LAYER: ids must be < n_routed
  int top_k;                   // LAYER: ids row length
  int slots_per_token;         // LAYER: top_k + n_shared
  int block_size;              // ALIGN padding
  int mt;                      // LAYER: max rows per GEMM tile
  // outputs
  int32_t* sorted_i32;         // ALIGN: sorted_token_ids; LAYER: slot at each sorted position
  int64_t sorted_cap;          // ALIGN
  int pad_sorted;              // ALIGN
  int32_t* block_expert;       // ALIGN: expert_ids
  int64_t block_cap;           // ALIGN
  int32_t* ntpp;               // ALIGN
  int32_t* cumsum;             // ALIGN: [n_buckets + 1]
  int32_t* ends;               // ENDS/DISPATCH/LAYER: [n_buckets + 1]
  int64_t* order_i64;          // ENDS/DISPATCH (and LAYER if set): sort_order
  int64_t* sorted_expert_i64;  // DISPATCH
  int32_t* pos_of_slot;        // LAYER: sorted position of every slot, -1 if dropped
  float* sorted_w;             // LAYER: router weight of the slot at each sorted position
  const void* topk_w;          // LAYER: router weights [T, top_k] (shared slots weigh 1)
  int w_dtype;
  int32_t* tile_info;          // LAYER: [max_tiles][3] = expert, first row, rows
  int32_t* n_tiles;            // LAYER: [1]
  int64_t max_tiles;
  int32_t* counters;           // LAYER: zeroed (the GEMM's tile and work counters)
  int64_t n_counters;
  uint32_t* status;
};

// `pdl`: launch as a programmatic dependent of the previous kernel in the
// stream (the kernel waits on griddepcontrol before reading its inputs).
int launch_route(RouteParams& p, int mode, cudaStream_t stream, bool pdl = false);

// ------------------------------------------------------------ route + gather
// One layer call's routing fused with the activation gather (route_gather.cu).
constexpr int kRouteGatherMaxBuckets = 1024;
constexpr int64_t kRouteGatherMaxSlots = 4096;
// Layer calls up to this many slots route and gather in one multi-CTA kernel
// (its shared memory holds two ints per slot: 131 KB at the limit).  Above
// kRouteGatherMaxSlots only calls averaging at most
// kRouteGatherFusedMaxRowsPerBucket rows per expert take it: with a few deep
// experts (Mixtral prefill, 1024 rows each) the separate routing and gather
// kernels are faster.
constexpr int64_t kRouteGatherFusedMaxSlots = 16384;
constexpr int64_t kRouteGatherFusedMaxRowsPerBucket = 512;

struct RouteGatherParams {
  const void* ids;      // [T, top_k] expert ids
  int ids_dtype;
  const void* topk_w;   // [T, top_k] router weights
  int w_dtype;
  const void* hidden;   // [T, hidden_size] activations
  int act_dtype;
  int64_t hidden_size;
  int top_k, spt, n_routed, n_buckets, mt;
  int64_t n;            // slots = T * spt
  __half* act;          // [n, hidden_size] gathered, fp16, octet-permuted
  int32_t* pos_of_slot; // [n]
  float* sorted_w;      // [n]
  int32_t* ends;        // [n_buckets + 1] or null
  int32_t* tile_info;   // [max_tiles][3]
  int32_t* n_tiles;     // [1]
  int64_t max_tiles;
  int32_t* sorted_slot; // [n] slot at every sorted position (or null)
  int32_t* counters;    // [n_counters] zeroed (the GEMM's tile and work counters)
  int64_t n_counters;
  uint32_t* status;
};

int launch_route_gather(RouteGatherParams& p, cudaStream_t stream, bool pdl);

// ------------------------------------------------------------ grouped GEMM
constexpr int kGmMTHost = 32;   // max token rows per GEMM tile
constexpr int kGmRBHost = 128;  // weight rows per work item

enum GemmMode : int { kGemmModePlain = 0, kGemmModeGateUp = 1, kGemmModeDown = 2 };

struct GemmParams {
  const exq_expert_desc* experts;
  int proj;         // 0: w13 / w13_scales, 1: w2 / w2_scales
  int mode;
  int n_rows;       // output rows of the projection: PLAIN N, GATE_UP 2I, DOWN H
  int k;            // reduction length
  int inter;        // GATE_UP: I
  int nblocks;      // row blocks per tile
  const void* act;  // PLAIN/GATE_UP: hidden [T, k]; DOWN: mid [n_pos, k]
  int64_t act_stride;
  int gather;       // 1: activation row = token of the sorted slot
  int spt;          // slots per token (top_k + shared)
  int top_k;
  const int32_t* sorted_slot;
  const int32_t* tile_info;
  const int32_t* n_tiles_ptr;
  int max_tiles;
  void* out;
  int out_dtype;
  int64_t out_stride;
  const void* topk_w;
  int w_dtype;
  uint32_t* status;
};

int launch_gemm(const GemmParams& p, int act_dtype, int max_items, cudaStream_t stream);

// ------------------------------------------------------------- elementwise
// y[t] = sum_j w[t, j] * partial[pos_of_slot[t * spt + j]] (w = 1 past top_k).
int launch_combine_partials(const float* partial, int64_t H, const int32_t* pos_of_slot,
                            const void* topk_w, int w_dtype, int top_k, int64_t n_tokens, int spt,
                            void* out, int dtype, cudaStream_t stream, bool pdl);

uint32_t* device_status_ptr();

// Views into a layer workspace (exq_moe_layer_forward_range) for a caller that
// replaces the combine stage: the fp32 down partials [n_slots, hidden] by
// sorted position and the slot -> sorted position map (-1: no expert).
// Router top-k (router.cu): argument check and launch (an ordinary launch;
// the kernel lets a programmatic successor launch early).
int check_router_args(int logits_dtype, int64_t n_tokens, int32_t n_experts, int32_t top_k);
cudaError_t launch_router_topk(const void* logits, int dtype, int64_t n_tokens, int n_experts,
                               int top_k, int renormalize, int32_t* ids, float* weights,
                               cudaStream_t s);

void layer_partials(void* workspace, int64_t n_slots, int64_t n_tokens, int n_buckets,
                    int64_t hidden, int64_t inter, const float** partial,
                    const int32_t** pos_of_slot);

}  // namespace exq
