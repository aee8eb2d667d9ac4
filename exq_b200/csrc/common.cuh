// Shared device/host helpers for the exq_b200 CUDA library (sm_100a only).
//
// Everything here is plumbing for the kernels in this directory: the status
// codes of the C ABI, dtype tags, inline-PTX wrappers (cp.async, warp MMA,
// LOP3/PRMT dequantisation) and a thread-local error message.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include "exq_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "exq_b200 is built for sm_100a (B200) only"
#endif

namespace exq {

// ---------------------------------------------------------------------------
// Host-side error reporting
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);

#define EXQ_CHECK_ARG(cond, ...)                                   \
  do {                                                             \
    if (!(cond)) {                                                 \
      ::exq::set_error(__VA_ARGS__);                               \
      return EXQ_ERR_INVALID;                                      \
    }                                                              \
  } while (0)

#define EXQ_CHECK_LAUNCH(what)                                     \
  do {                                                             \
    cudaError_t _e = cudaGetLastError();                           \
    if (_e != cudaSuccess) {                                       \
      ::exq::set_error("%s: %s", what, cudaGetErrorString(_e));    \
      return EXQ_ERR_CUDA;                                         \
    }                                                              \
  } while (0)

inline int num_sms() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte global->shared async copy; src_bytes < 16 zero-fills the rest.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src),
               "r"(src_bytes));
}
// Same, with an L2 eviction-priority policy (weights are streamed once).
__device__ __forceinline__ void cp_async16_hint(uint32_t dst, const void* src, uint64_t pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;\n" ::"r"(dst),
               "l"(src), "l"(pol));
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;\n" : "=l"(p));
  return p;
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;\n" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
// d = (a & b) | c
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Warp MMA m16n8k16, fp32 accumulate.  A row-major 16x16, B col-major 16x8.
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1, __half) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1, __nv_bfloat16) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------------------
// Dequantisation to exact small integers (scales are applied in fp32 later).
//
// INT4 byte b of a packed word holds (k even: low nibble, k odd: high nibble),
// each stored as q + 8.  The result is the 16-bit pair (q_even, q_odd) with
// q_even in the low half, i.e. the natural k order of an activation pair.
// fp16: OR the nibble into the mantissa of 1024.0 (0x6400): low half
// 1024 + n, high half 1024 + 16 n; one HFMA2 with (1, 1/16) and
// (-1032, -72) turns both into n - 8 exactly.
// bf16: nibbles are first separated into bytes and ORed into 128.0 (0x4300);
// one HSUB2 of 136 gives n - 8 exactly.
// ---------------------------------------------------------------------------
template <typename T>
struct Dq;

template <>
struct Dq<__half> {
  // Pre-pass per 32-bit word (none needed for fp16).
  struct Word {
    uint32_t w;
  };
  static __device__ __forceinline__ Word prep(uint32_t w) { return Word{w}; }
  static __device__ __forceinline__ uint32_t int4_pair(Word w, int b) {
    // byte b -> bytes 0 and 2 (bytes 1, 3 from the zero operand)
    const uint32_t sel = 0x4040u | (uint32_t)b | ((uint32_t)b << 8);
    uint32_t x = prmt(w.w, 0u, sel);
    x = and_or(x, 0x00F0000Fu, 0x64006400u);
    const __half2 mul = __halves2half2(__float2half_rn(1.0f), __float2half_rn(0.0625f));
    const __half2 add = __halves2half2(__float2half_rn(-1032.0f), __float2half_rn(-72.0f));
    __half2 h = __hfma2(*reinterpret_cast<__half2*>(&x), mul, add);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  // INT8: word holds 4 signed bytes; returns the pair (byte 2p, byte 2p+1).
  static __device__ __forceinline__ uint32_t int8_pair(uint32_t w_xor80, int p) {
    // w_xor80 = w ^ 0x80808080 (unsigned offset); bytes -> mantissa of 1024.0
    const uint32_t sel = p == 0 ? 0x4140u : 0x4342u;
    uint32_t x = prmt(w_xor80, 0x64646464u, sel);
    __half2 h = __hsub2(*reinterpret_cast<__half2*>(&x),
                        __halves2half2(__float2half_rn(1152.0f), __float2half_rn(1152.0f)));
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

template <>
struct Dq<__nv_bfloat16> {
  struct Word {
    uint32_t lo, hi;  // nibbles separated: lo bytes = even k, hi bytes = odd k
  };
  static __device__ __forceinline__ Word prep(uint32_t w) {
    return Word{w & 0x0F0F0F0Fu, (w >> 4) & 0x0F0F0F0Fu};
  }
  static __device__ __forceinline__ uint32_t int4_pair(Word w, int b) {
    // byte0 <- lo.b, byte2 <- hi.b
    const uint32_t sel = (uint32_t)b | ((uint32_t)(4 + b) << 8);
    uint32_t x = prmt(w.lo, w.hi, sel);
    x = and_or(x, 0x000F000Fu, 0x43004300u);
    __nv_bfloat162 h = __hsub2(*reinterpret_cast<__nv_bfloat162*>(&x),
                               __floats2bfloat162_rn(136.0f, 136.0f));
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ uint32_t int8_pair(uint32_t w_xor80, int p) {
    // bytes -> fp32 mantissa of 2^23, subtract 2^23 + 128, pack to bf16x2
    const uint32_t s0 = p == 0 ? 0x7440u : 0x7442u;  // byte0 <- w.b(2p), bytes1-2 <- 0, byte3 <- 0x4B
    const uint32_t s1 = p == 0 ? 0x7441u : 0x7443u;
    uint32_t x0 = prmt(w_xor80, 0x4B000000u, s0);
    uint32_t x1 = prmt(w_xor80, 0x4B000000u, s1);
    float f0 = __uint_as_float(x0) - 8388736.0f;
    float f1 = __uint_as_float(x1) - 8388736.0f;
    __nv_bfloat162 h = __floats2bfloat162_rn(f0, f1);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float to_f32<float>(float v) {
  return v;
}
template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) {
  return __float2half_rn(v);
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ float from_f32<float>(float v) {
  return v;
}

__device__ __forceinline__ float load_as_f32(const void* p, int dtype, int64_t i) {
  if (dtype == EXQ_F32) return static_cast<const float*>(p)[i];
  if (dtype == EXQ_F16) return __half2float(static_cast<const __half*>(p)[i]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}

__device__ __forceinline__ int64_t load_index(const void* p, int dtype, int64_t i) {
  if (dtype == EXQ_I64) return static_cast<const int64_t*>(p)[i];
  return static_cast<const int32_t*>(p)[i];
}

}  // namespace exq
