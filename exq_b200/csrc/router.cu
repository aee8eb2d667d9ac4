// Router top-k: softmax over a token's expert logits, the top_k largest
// probabilities, optionally renormalised over the selected ones.  This is the
// routing the reference's generated MoE layers compute before dispatch
// (exq/codegen/triton_emitter.py:273-276) and the `topk_output` SGLang hands to
// the expert path (exq/runtime/sglang_backend.py:88-90).
//
// One warp per token.  Expert e lives in lane e % 32, register e / 32, so the
// logit loads of a warp are coalesced.  Integer/compare work only besides the
// exponentials and two divisions per expert; the kernel is bound by reading
// the logits (T x E x 2-4 bytes).
#include "internal.cuh"

namespace exq {
namespace {

constexpr int kRouterMaxExperts = 1024;
constexpr int kRouterMaxTopK = 32;
constexpr int kRouterWarps = 8;

// (value, expert) pairs ordered by value, then by the lower expert id.
__device__ __forceinline__ bool better(float v, int e, float bv, int be) {
  return v > bv || (v == bv && e < be);
}

template <int PER>
__global__ void __launch_bounds__(32 * kRouterWarps)
    router_topk_kernel(const void* __restrict__ logits, int dtype, int64_t n_tokens, int n_experts,
                       int top_k, int renormalize, int32_t* __restrict__ ids,
                       float* __restrict__ weights) {
  const int lane = threadIdx.x & 31;
  // a routing kernel chained after this one may launch now: it waits for
  // this grid's completion (griddepcontrol.wait) before it reads the ids
  pdl_trigger();
  const int64_t warps = static_cast<int64_t>(gridDim.x) * kRouterWarps;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(kRouterWarps) + (threadIdx.x >> 5);
       t < n_tokens; t += warps) {
    const int64_t row = t * n_experts;
    float v[PER];
    float m = -INFINITY;
#pragma unroll
    for (int c = 0; c < PER; ++c) {
      const int e = c * 32 + lane;
      v[c] = e < n_experts ? load_as_f32(logits, dtype, row + e) : -INFINITY;
      m = fmaxf(m, v[c]);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    // softmax in fp32: exp(x - max) / sum; the sum is a fixed butterfly, so
    // every run gives the same bits
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < PER; ++c) {
      const int e = c * 32 + lane;
      v[c] = e < n_experts ? expf(v[c] - m) : 0.f;
      s += v[c];
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
#pragma unroll
    for (int c = 0; c < PER; ++c) v[c] = __fdiv_rn(v[c], s);

    // top_k rounds of a warp arg-max; lane j keeps the j-th pick
    uint32_t taken = 0;
    float my_p = 0.f;
    int my_e = -1;
    for (int r = 0; r < top_k; ++r) {
      float bv = -1.f;
      int be = INT32_MAX;
#pragma unroll
      for (int c = 0; c < PER; ++c) {
        const int e = c * 32 + lane;
        if (e < n_experts && !((taken >> c) & 1u) && better(v[c], e, bv, be)) {
          bv = v[c];
          be = e;
        }
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oe = __shfl_xor_sync(0xffffffffu, be, o);
        if (better(ov, oe, bv, be)) {
          bv = ov;
          be = oe;
        }
      }
      if ((be & 31) == lane) taken |= 1u << (be >> 5);
      if (lane == r) {
        my_p = bv;
        my_e = be;
      }
    }
    float w = my_p;
    if (renormalize) {
      // the selected probabilities summed in pick order (descending)
      float tot = 0.f;
      for (int j = 0; j < top_k; ++j) tot += __shfl_sync(0xffffffffu, my_p, j);
      w = __fdiv_rn(my_p, tot);
    }
    if (lane < top_k) {
      ids[t * top_k + lane] = my_e;
      weights[t * top_k + lane] = w;
    }
  }
}

template <int PER>
cudaError_t launch_router(const void* logits, int dtype, int64_t n_tokens, int n_experts,
                          int top_k, int renormalize, int32_t* ids, float* weights,
                          cudaStream_t s) {
  int64_t blocks = (n_tokens + kRouterWarps - 1) / kRouterWarps;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 16;
  if (blocks > cap) blocks = cap;
  router_topk_kernel<PER><<<static_cast<int>(blocks), 32 * kRouterWarps, 0, s>>>(
      logits, dtype, n_tokens, n_experts, top_k, renormalize, ids, weights);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_router_topk(const void* logits, int dtype, int64_t n_tokens, int n_experts,
                               int top_k, int renormalize, int32_t* ids, float* weights,
                               cudaStream_t s) {
  const int per = (n_experts + 31) / 32;
  if (per <= 1)
    return launch_router<1>(logits, dtype, n_tokens, n_experts, top_k, renormalize, ids, weights, s);
  if (per <= 2)
    return launch_router<2>(logits, dtype, n_tokens, n_experts, top_k, renormalize, ids, weights, s);
  if (per <= 4)
    return launch_router<4>(logits, dtype, n_tokens, n_experts, top_k, renormalize, ids, weights, s);
  if (per <= 8)
    return launch_router<8>(logits, dtype, n_tokens, n_experts, top_k, renormalize, ids, weights, s);
  if (per <= 16)
    return launch_router<16>(logits, dtype, n_tokens, n_experts, top_k, renormalize, ids, weights,
                             s);
  return launch_router<32>(logits, dtype, n_tokens, n_experts, top_k, renormalize, ids, weights, s);
}

int check_router_args(int logits_dtype, int64_t n_tokens, int32_t n_experts, int32_t top_k) {
  EXQ_CHECK_ARG(logits_dtype == EXQ_F32 || logits_dtype == EXQ_F16 || logits_dtype == EXQ_BF16,
                "router_topk: logits must be fp32, fp16 or bf16");
  EXQ_CHECK_ARG(n_tokens >= 0, "router_topk: n_tokens < 0");
  EXQ_CHECK_ARG(n_experts >= 1 && n_experts <= kRouterMaxExperts,
                "router_topk: n_experts=%d outside 1..%d", n_experts, kRouterMaxExperts);
  EXQ_CHECK_ARG(top_k >= 1 && top_k <= kRouterMaxTopK && top_k <= n_experts,
                "router_topk: top_k=%d outside 1..min(%d, n_experts)", top_k, kRouterMaxTopK);
  return EXQ_OK;
}

}  // namespace exq

using namespace exq;

extern "C" int exq_router_topk(const void* logits, int logits_dtype, int64_t n_tokens,
                               int32_t n_experts, int32_t top_k, int32_t renormalize,
                               int32_t* topk_ids, float* topk_weights, void* stream) {
  const int st = check_router_args(logits_dtype, n_tokens, n_experts, top_k);
  if (st != EXQ_OK) return st;
  if (n_tokens == 0) return EXQ_OK;
  EXQ_CHECK_ARG(logits && topk_ids && topk_weights, "router_topk: null pointer");
  const cudaError_t e = launch_router_topk(logits, logits_dtype, n_tokens, n_experts, top_k,
                                           renormalize, topk_ids, topk_weights,
                                           static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    set_error("router_topk_kernel: %s", cudaGetErrorString(e));
    return EXQ_ERR_CUDA;
  }
  return EXQ_OK;
}
