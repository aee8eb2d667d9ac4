// Row gather, top-k combine, SiLU*mul and the GPU weight packers.
#include <atomic>

#include "internal.cuh"

namespace exq {

// ---------------------------------------------------------------- gather
// out[i, :] = hidden[sort_order[i] / top_k, :]   (exq_dispatch.cu:234-260)
template <bool kVec>
__global__ void gather_rows_kernel(const uint8_t* __restrict__ hidden, int64_t row_bytes,
                                   int64_t src_stride_bytes, const int64_t* __restrict__ order,
                                   int64_t n_active, int64_t n_tokens, int top_k,
                                   uint8_t* __restrict__ out, uint32_t* status) {
  for (int64_t i = blockIdx.x; i < n_active; i += gridDim.x) {
    const int64_t slot = order[i];
    const int64_t tok = slot / top_k;
    uint8_t* dst = out + i * row_bytes;
    if (slot < 0 || tok >= n_tokens) {
      if (threadIdx.x == 0) atomicOr(status, EXQ_DEV_BAD_SLOT);
      continue;
    }
    const uint8_t* src = hidden + tok * src_stride_bytes;
    if (kVec) {
      const uint4* s4 = reinterpret_cast<const uint4*>(src);
      uint4* d4 = reinterpret_cast<uint4*>(dst);
      for (int64_t c = threadIdx.x; c < row_bytes / 16; c += blockDim.x) d4[c] = s4[c];
    } else {
      const uint16_t* s2 = reinterpret_cast<const uint16_t*>(src);
      uint16_t* d2 = reinterpret_cast<uint16_t*>(dst);
      for (int64_t c = threadIdx.x; c < row_bytes / 2; c += blockDim.x) d2[c] = s2[c];
    }
  }
}

// ---------------------------------------------------------------- combine
__global__ void inverse_perm_kernel(const int64_t* __restrict__ order, int64_t n,
                                    int32_t* __restrict__ inv, uint32_t* status) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t s = order[i];
    if (s < 0 || s >= n) {
      atomicOr(status, EXQ_DEV_BAD_SLOT);
      continue;
    }
    inv[s] = static_cast<int32_t>(i);
  }
}

// result[t, h] = cast(sum_j w[t, j] * down[inv[t*k+j], h])  (exq_dispatch.cu:263-310)
template <typename Tin, typename Tout>
__global__ void combine_kernel(const Tin* __restrict__ down, int64_t H,
                               const int32_t* __restrict__ inv, const void* __restrict__ w,
                               int w_dtype, int64_t n_tokens, int top_k,
                               Tout* __restrict__ result) {
  for (int64_t t = blockIdx.x; t < n_tokens; t += gridDim.x) {
    for (int64_t h = threadIdx.x; h < H; h += blockDim.x) {
      float acc = 0.f;
      for (int j = 0; j < top_k; ++j) {
        const int32_t r = inv[t * top_k + j];
        if (r < 0) continue;
        const float wj = load_as_f32(w, w_dtype, t * top_k + j);
        // separate rounding of product and sum (no FMA contraction)
        acc = __fadd_rn(acc, __fmul_rn(wj, to_f32<Tin>(down[(int64_t)r * H + h])));
      }
      result[t * H + h] = from_f32<Tout>(acc);
    }
  }
}

// Layer combine: y[t, h] = sum_j partial[pos(t, j), h] (partials already weighted,
// fp32, in sorted-position order; pos < 0 = slot dropped).
template <typename Tout>
__device__ __forceinline__ void store4(Tout* o, float4 a) {
  o[0] = from_f32<Tout>(a.x);
  o[1] = from_f32<Tout>(a.y);
  o[2] = from_f32<Tout>(a.z);
  o[3] = from_f32<Tout>(a.w);
}
template <>
__device__ __forceinline__ void store4<__half>(__half* o, float4 a) {
  __half2 lo = __floats2half2_rn(a.x, a.y), hi = __floats2half2_rn(a.z, a.w);
  uint2 v = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
  *reinterpret_cast<uint2*>(o) = v;
}
template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* o, float4 a) {
  __nv_bfloat162 lo = __floats2bfloat162_rn(a.x, a.y), hi = __floats2bfloat162_rn(a.z, a.w);
  uint2 v = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
  *reinterpret_cast<uint2*>(o) = v;
}

// y[t] = sum over the token's slots j, in slot order, of w[t, j] * partial[pos]
// (w = 1 for the always-on shared experts; product and sum rounded
// separately in fp32).  The token's slot positions and weights are staged in
// shared memory first so that the row loads of all its slots are independent
// and issue together.
template <typename Tout>
__global__ void combine_partials_kernel(const float* __restrict__ partial, int64_t H,
                                        const int32_t* __restrict__ pos_of_slot,
                                        const void* __restrict__ topk_w, int w_dtype, int top_k,
                                        int64_t n_tokens, int spt, Tout* __restrict__ out) {
  extern __shared__ int32_t spos[];  // [spt] positions, then [spt] weights
  float* sw = reinterpret_cast<float*>(spos + spt);
  pdl_wait();
  pdl_trigger();
  const int64_t hv = H / 4;
  for (int64_t t = blockIdx.x; t < n_tokens; t += gridDim.x) {
    for (int j = threadIdx.x; j < spt; j += blockDim.x) {
      spos[j] = pos_of_slot[t * spt + j];
      sw[j] = j < top_k ? load_as_f32(topk_w, w_dtype, t * top_k + j) : 1.0f;
    }
    __syncthreads();
    for (int64_t c = threadIdx.x; c < hv; c += blockDim.x) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int j0 = 0; j0 < spt; j0 += 8) {
        float4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int r = j0 + u < spt ? spos[j0 + u] : -1;
          v[u] = r >= 0 ? __ldg(reinterpret_cast<const float4*>(partial + (int64_t)r * H) + c)
                        : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {  // sum in slot order
          const float wj = j0 + u < spt ? sw[j0 + u] : 0.f;
          acc.x = __fadd_rn(acc.x, __fmul_rn(wj, v[u].x));
          acc.y = __fadd_rn(acc.y, __fmul_rn(wj, v[u].y));
          acc.z = __fadd_rn(acc.z, __fmul_rn(wj, v[u].z));
          acc.w = __fadd_rn(acc.w, __fmul_rn(wj, v[u].w));
        }
      }
      store4<Tout>(out + t * H + 4 * c, acc);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------- silu*mul
template <typename T>
__global__ void silu_and_mul_kernel(const T* __restrict__ in, T* __restrict__ out, int64_t m,
                                    int64_t inter) {
  const int64_t total = m * inter;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / inter, c = i - r * inter;
    const float g = to_f32<T>(in[r * 2 * inter + c]);
    const float u = to_f32<T>(in[r * 2 * inter + inter + c]);
    out[i] = from_f32<T>(g / (1.0f + expf(-g)) * u);
  }
}

// ---------------------------------------------------------------- packers
// One warp per (row, group).  Bit-exact restatement of pack_int4_weights
// (moe_int4_kernel.py:74-91): fp32 amax / 7 (IEEE division), clamp at
// FLT_EPSILON, round-half-even of w / scale (IEEE division), clamp [-8, 7],
// nibble q + 8 (even k low), scale rounded to fp16.
template <typename T>
__global__ void pack_int4_kernel(const T* __restrict__ w, int64_t rows, int64_t k, int gs,
                                 uint8_t* __restrict__ packed, __half* __restrict__ scales) {
  const int64_t ng = k / gs;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  const int lane = threadIdx.x & 31;
  for (int64_t wg = blockIdx.x * (int64_t)(blockDim.x / 32) + (threadIdx.x >> 5);
       wg < rows * ng; wg += warps) {
    const int64_t r = wg / ng, gi = wg - r * ng;
    const T* src = w + r * k + gi * gs;
    float amax = 0.f;
    for (int i = lane; i < gs; i += 32) amax = fmaxf(amax, fabsf(to_f32<T>(src[i])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    float scale = __fdiv_rn(amax, 7.0f);
    scale = fmaxf(scale, 1.1920928955078125e-07f);
    for (int i = 2 * lane; i < gs; i += 64) {
      const float q0 = fminf(fmaxf(rintf(__fdiv_rn(to_f32<T>(src[i]), scale)), -8.f), 7.f);
      const float q1 = fminf(fmaxf(rintf(__fdiv_rn(to_f32<T>(src[i + 1]), scale)), -8.f), 7.f);
      const uint32_t lo = static_cast<uint32_t>(static_cast<int>(q0) + 8);
      const uint32_t hi = static_cast<uint32_t>(static_cast<int>(q1) + 8);
      packed[r * (k / 2) + (gi * gs + i) / 2] = static_cast<uint8_t>(lo | (hi << 4));
    }
    if (lane == 0) scales[r * ng + gi] = __float2half_rn(scale);
  }
}

// One block per row: the INT8 tier (quant_shim.py:84-96; fp16 scale).
template <typename T>
__global__ void quant_int8_kernel(const T* __restrict__ w, int64_t rows, int64_t k,
                                  int8_t* __restrict__ q, __half* __restrict__ scales) {
  __shared__ float red[32];
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* src = w + r * k;
    float amax = 0.f;
    for (int64_t i = threadIdx.x; i < k; i += blockDim.x) amax = fmaxf(amax, fabsf(to_f32<T>(src[i])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    if (threadIdx.x < 32) {
      float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
      if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    float scale = fmaxf(__fdiv_rn(red[0], 127.0f), 1.1920928955078125e-07f);
    for (int64_t i = threadIdx.x; i < k; i += blockDim.x) {
      const float v = fminf(fmaxf(rintf(__fdiv_rn(to_f32<T>(src[i]), scale)), -128.f), 127.f);
      q[r * k + i] = static_cast<int8_t>(v);
    }
    if (threadIdx.x == 0) scales[r] = __float2half_rn(scale);
    __syncthreads();
  }
}

inline int grid_for(int64_t work, int threads, int max_blocks_per_sm = 8) {
  int64_t g = (work + threads - 1) / threads;
  const int64_t cap = (int64_t)num_sms() * max_blocks_per_sm;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return static_cast<int>(g);
}

int launch_combine_partials(const float* partial, int64_t H, const int32_t* pos_of_slot,
                            const void* topk_w, int w_dtype, int top_k, int64_t n_tokens, int spt,
                            void* out, int dtype, cudaStream_t stream, bool pdl) {
  if (n_tokens == 0) return EXQ_OK;
  const int threads = static_cast<int>(H / 4 < 256 ? (H / 4 < 32 ? 32 : H / 4) : 256);
  const int grid = static_cast<int>(n_tokens < 65535 ? n_tokens : 65535);
  cudaError_t e;
  if (dtype == EXQ_F16)
    e = launch_pdl(pdl, combine_partials_kernel<__half>, dim3(grid), dim3(threads),
                   2 * sizeof(int32_t) * spt, stream, partial, H, pos_of_slot, topk_w, w_dtype,
                   top_k, n_tokens, spt, static_cast<__half*>(out));
  else
    e = launch_pdl(pdl, combine_partials_kernel<__nv_bfloat16>, dim3(grid), dim3(threads),
                   2 * sizeof(int32_t) * spt, stream, partial, H, pos_of_slot, topk_w, w_dtype,
                   top_k, n_tokens, spt, static_cast<__nv_bfloat16*>(out));
  if (e != cudaSuccess) {
    set_error("combine_partials_kernel: %s", cudaGetErrorString(e));
    return EXQ_ERR_CUDA;
  }
  EXQ_CHECK_LAUNCH("combine_partials_kernel");
  return EXQ_OK;
}

}  // namespace exq

using namespace exq;

static bool is_act(int d) { return d == EXQ_F16 || d == EXQ_BF16; }

extern "C" int exq_gather_hidden(const void* hidden, int dtype, int64_t n_tokens,
                                 int64_t hidden_size, int64_t row_stride,
                                 const int64_t* sort_order, int64_t n_active, int32_t top_k,
                                 void* out, void* stream) {
  EXQ_CHECK_ARG(is_act(dtype), "gather_hidden: dtype must be fp16 or bf16");
  EXQ_CHECK_ARG(top_k > 0, "gather_hidden: top_k must be positive");
  EXQ_CHECK_ARG(n_active >= 0 && n_tokens >= 0 && hidden_size >= 0, "negative size");
  EXQ_CHECK_ARG(row_stride >= hidden_size, "row_stride < hidden_size");
  if (n_active == 0 || hidden_size == 0) return EXQ_OK;
  EXQ_CHECK_ARG(hidden && sort_order && out, "gather_hidden: null pointer");
  uint32_t* st = device_status_ptr();
  if (!st) return EXQ_ERR_CUDA;
  const int64_t row_bytes = hidden_size * 2;
  const bool vec = (row_bytes % 16 == 0) && ((row_stride * 2) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(hidden) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(out) % 16 == 0);
  const int threads = 128;
  const int grid = static_cast<int>(n_active < 65535 ? n_active : 65535);
  auto s = static_cast<cudaStream_t>(stream);
  if (vec)
    gather_rows_kernel<true><<<grid, threads, 0, s>>>(
        static_cast<const uint8_t*>(hidden), row_bytes, row_stride * 2, sort_order, n_active,
        n_tokens, top_k, static_cast<uint8_t*>(out), st);
  else
    gather_rows_kernel<false><<<grid, threads, 0, s>>>(
        static_cast<const uint8_t*>(hidden), row_bytes, row_stride * 2, sort_order, n_active,
        n_tokens, top_k, static_cast<uint8_t*>(out), st);
  EXQ_CHECK_LAUNCH("gather_rows_kernel");
  return EXQ_OK;
}

extern "C" size_t exq_combine_workspace_bytes(int64_t n_active) {
  return align_up(static_cast<size_t>(n_active > 0 ? n_active : 0) * sizeof(int32_t), 256);
}

extern "C" int exq_combine(const void* down_out, int dtype, int64_t n_active,
                           int64_t hidden_size, const int64_t* sort_order,
                           const void* router_weights, int w_dtype, int64_t n_tokens,
                           int32_t top_k, void* result, int out_dtype, void* workspace,
                           size_t workspace_bytes, void* stream) {
  EXQ_CHECK_ARG(is_act(dtype) || dtype == EXQ_F32, "combine: down_out dtype unsupported");
  EXQ_CHECK_ARG(is_act(out_dtype) || out_dtype == EXQ_F32, "combine: out dtype unsupported");
  EXQ_CHECK_ARG(w_dtype == EXQ_F32 || is_act(w_dtype), "combine: weight dtype unsupported");
  EXQ_CHECK_ARG(top_k > 0, "combine: top_k must be positive");
  EXQ_CHECK_ARG(n_active == n_tokens * top_k,
                "combine: sort_order has %lld entries, router_weights implies %lld",
                (long long)n_active, (long long)(n_tokens * top_k));
  if (n_tokens == 0 || hidden_size == 0) return EXQ_OK;
  EXQ_CHECK_ARG(down_out && sort_order && router_weights && result, "combine: null pointer");
  if (!workspace || workspace_bytes < exq_combine_workspace_bytes(n_active)) {
    set_error("combine: workspace of %zu bytes needed", exq_combine_workspace_bytes(n_active));
    return EXQ_ERR_WORKSPACE;
  }
  uint32_t* st = device_status_ptr();
  if (!st) return EXQ_ERR_CUDA;
  auto s = static_cast<cudaStream_t>(stream);
  int32_t* inv = static_cast<int32_t*>(workspace);
  if (cudaMemsetAsync(inv, 0xFF, n_active * sizeof(int32_t), s) != cudaSuccess) {
    set_error("combine: cudaMemsetAsync failed");
    return EXQ_ERR_CUDA;
  }
  inverse_perm_kernel<<<grid_for(n_active, 256), 256, 0, s>>>(sort_order, n_active, inv, st);
  EXQ_CHECK_LAUNCH("inverse_perm_kernel");
  const int threads = static_cast<int>(hidden_size < 256 ? hidden_size : 256);
  const int grid = static_cast<int>(n_tokens < 65535 ? n_tokens : 65535);
#define EXQ_COMBINE(TI, TO)                                                                   \
  combine_kernel<TI, TO><<<grid, threads, 0, s>>>(static_cast<const TI*>(down_out),          \
                                                   hidden_size, inv, router_weights, w_dtype, \
                                                   n_tokens, top_k, static_cast<TO*>(result))
  if (dtype == EXQ_F16) {
    if (out_dtype == EXQ_F16) EXQ_COMBINE(__half, __half);
    else if (out_dtype == EXQ_BF16) EXQ_COMBINE(__half, __nv_bfloat16);
    else EXQ_COMBINE(__half, float);
  } else if (dtype == EXQ_BF16) {
    if (out_dtype == EXQ_F16) EXQ_COMBINE(__nv_bfloat16, __half);
    else if (out_dtype == EXQ_BF16) EXQ_COMBINE(__nv_bfloat16, __nv_bfloat16);
    else EXQ_COMBINE(__nv_bfloat16, float);
  } else {
    if (out_dtype == EXQ_F16) EXQ_COMBINE(float, __half);
    else if (out_dtype == EXQ_BF16) EXQ_COMBINE(float, __nv_bfloat16);
    else EXQ_COMBINE(float, float);
  }
#undef EXQ_COMBINE
  EXQ_CHECK_LAUNCH("combine_kernel");
  return EXQ_OK;
}

// ---------------------------------------------------------------- combine, no allocation
// Scratch for exq_combine_noalloc: the inverse permutation of one call,
// EXQ_COMBINE_NOALLOC_MAX_ACTIVE int32 slots (1 MiB) per device, in the
// library's static device memory.  One copy per device, shared by every call
// on that device: calls that overlap in time race on it.
static __device__ __align__(256) int32_t g_combine_inv[EXQ_COMBINE_NOALLOC_MAX_ACTIVE];

// Address of g_combine_inv on the current device, looked up once per device.
// The first call on a device may load the module, so make it before any
// stream capture begins.
static int32_t* combine_scratch_ptr() {
  static std::atomic<int32_t*> ptrs[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    set_error("combine_noalloc: cudaGetDevice failed");
    return nullptr;
  }
  int32_t* p = ptrs[dev].load(std::memory_order_acquire);
  if (!p) {
    void* a = nullptr;
    e = cudaGetSymbolAddress(&a, g_combine_inv);
    if (e != cudaSuccess) {
      set_error("combine_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      return nullptr;
    }
    p = static_cast<int32_t*>(a);
    ptrs[dev].store(p, std::memory_order_release);
  }
  return p;
}

extern "C" int exq_combine_noalloc(const void* down_out, int dtype, int64_t n_active,
                                   int64_t hidden_size, const int64_t* sort_order,
                                   const void* router_weights, int w_dtype, int64_t n_tokens,
                                   int32_t top_k, void* result, int out_dtype, void* stream) {
  EXQ_CHECK_ARG(n_active >= 0 && n_active <= EXQ_COMBINE_NOALLOC_MAX_ACTIVE,
                "combine_noalloc: n_active %lld is outside the static scratch of %d slots "
                "(call exq_combine with a workspace instead)",
                (long long)n_active, EXQ_COMBINE_NOALLOC_MAX_ACTIVE);
  int32_t* inv = combine_scratch_ptr();
  if (!inv) return EXQ_ERR_CUDA;
  // exq_combine fills the first n_active slots with -1 on `stream` before use,
  // so nothing in the scratch has to start zeroed.
  return exq_combine(down_out, dtype, n_active, hidden_size, sort_order, router_weights, w_dtype,
                     n_tokens, top_k, result, out_dtype, inv,
                     sizeof(int32_t) * static_cast<size_t>(EXQ_COMBINE_NOALLOC_MAX_ACTIVE), stream);
}

extern "C" int exq_silu_and_mul(const void* input, void* out, int dtype, int64_t m,
                                int64_t inter, void* stream) {
  EXQ_CHECK_ARG(is_act(dtype), "silu_and_mul: dtype must be fp16 or bf16");
  EXQ_CHECK_ARG(m >= 0 && inter >= 0, "negative size");
  if (m == 0 || inter == 0) return EXQ_OK;
  EXQ_CHECK_ARG(input && out, "silu_and_mul: null pointer");
  auto s = static_cast<cudaStream_t>(stream);
  const int grid = grid_for(m * inter, 256);
  if (dtype == EXQ_F16)
    silu_and_mul_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(input),
                                                     static_cast<__half*>(out), m, inter);
  else
    silu_and_mul_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(input), static_cast<__nv_bfloat16*>(out), m, inter);
  EXQ_CHECK_LAUNCH("silu_and_mul_kernel");
  return EXQ_OK;
}

extern "C" int exq_pack_int4(const void* w, int dtype, int64_t rows, int64_t k,
                             int32_t group_size, uint8_t* packed, void* scales_f16,
                             void* stream) {
  EXQ_CHECK_ARG(is_act(dtype) || dtype == EXQ_F32, "pack_int4: dtype unsupported");
  EXQ_CHECK_ARG(rows >= 0, "rows < 0");
  EXQ_CHECK_ARG(k > 0 && k % 2 == 0, "K=%lld must be divisible by 2 for INT4 packing",
                (long long)k);
  EXQ_CHECK_ARG(group_size > 0, "group_size must be positive");
  int64_t gs = group_size;
  if (k < gs) gs = k;
  EXQ_CHECK_ARG(k % gs == 0, "K=%lld must be divisible by group_size=%lld", (long long)k,
                (long long)gs);
  EXQ_CHECK_ARG(gs % 2 == 0, "group_size must be even");
  if (rows == 0) return EXQ_OK;
  EXQ_CHECK_ARG(w && packed && scales_f16, "pack_int4: null pointer");
  auto s = static_cast<cudaStream_t>(stream);
  const int64_t work = rows * (k / gs) * 32;
  const int grid = grid_for(work, 256, 16);
#define EXQ_PACK(T)                                                                         \
  pack_int4_kernel<T><<<grid, 256, 0, s>>>(static_cast<const T*>(w), rows, k,              \
                                           static_cast<int>(gs), packed,                   \
                                           static_cast<__half*>(scales_f16))
  if (dtype == EXQ_F16) EXQ_PACK(__half);
  else if (dtype == EXQ_BF16) EXQ_PACK(__nv_bfloat16);
  else EXQ_PACK(float);
#undef EXQ_PACK
  EXQ_CHECK_LAUNCH("pack_int4_kernel");
  return EXQ_OK;
}

extern "C" int exq_quant_int8(const void* w, int dtype, int64_t rows, int64_t k, int8_t* q,
                              void* scales_f16, void* stream) {
  EXQ_CHECK_ARG(is_act(dtype) || dtype == EXQ_F32, "quant_int8: dtype unsupported");
  EXQ_CHECK_ARG(rows >= 0 && k > 0, "bad shape");
  if (rows == 0) return EXQ_OK;
  EXQ_CHECK_ARG(w && q && scales_f16, "quant_int8: null pointer");
  auto s = static_cast<cudaStream_t>(stream);
  const int grid = static_cast<int>(rows < 65535 ? rows : 65535);
#define EXQ_Q8(T)                                                                           \
  quant_int8_kernel<T><<<grid, 256, 0, s>>>(static_cast<const T*>(w), rows, k, q,          \
                                            static_cast<__half*>(scales_f16))
  if (dtype == EXQ_F16) EXQ_Q8(__half);
  else if (dtype == EXQ_BF16) EXQ_Q8(__nv_bfloat16);
  else EXQ_Q8(float);
#undef EXQ_Q8
  EXQ_CHECK_LAUNCH("quant_int8_kernel");
  return EXQ_OK;
}
