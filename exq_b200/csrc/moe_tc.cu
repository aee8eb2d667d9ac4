// Warp-specialised tcgen05 grouped GEMM for the MoE expert layer (sm_100a).
//
// Replaces the reference's two Triton INT4 GEMM launches plus gather,
// silu_and_mul and the down half of the combine
// (exq/kernels/moe_int4_kernel.py:124-240, :374-426;
// exq/runtime/sglang_backend.py:117-156) for experts that mix BF16, INT8 and
// INT4 weight tiers.
//
// One persistent CTA per SM (480 threads, 15 warps):
//   warp 0       weight producer: TMA 2D loads of packed weights (+ INT4 group
//                scales) into a 12-slot ring of 4 KB slots
//   warp 1       activation producer: TMA 2D loads (128B swizzle) of the
//                item's token rows into a 3-slot ring (<= 256 rows x 64 k)
//   warp 2       MMA issuer: one thread issues tcgen05.mma (M=128, N=tokens,
//                K=16) into a double-buffered TMEM accumulator (2 x 256 cols)
//   warps 3-6    epilogue: tcgen05.ld of the accumulator, fused SiLU*mul
//                (gate_up) or router-weighted fp32 partials (down)
//   warps 7-14   dequantisers: packed weights -> fp16 (scale applied) written
//                into the 128B-swizzled K-major A tile the MMA reads
// A work item is (expert, 128-row block of the projection, up to 256 tokens
// of that expert): every weight byte is dequantised once per item and all the
// expert's tokens ride in the MMA's N dimension, so hot experts do not re-read
// or re-dequantise weights.
//
// K order.  Inside every 8-element octet the k order is permuted to
// [0,4,1,5,2,6,3,7] identically for weights and activations (a dot product
// does not depend on term order).  With it a packed INT4 word dequantises with
// the 1024.0 magic-number trick straight into K-adjacent fp16 pairs (4 LOP3 +
// 2 HSUB2 + 2 HFMA2 per 8 weights), the INT8 / 16-bit tiers are stored
// pre-permuted at pack time, and the activation prep kernel permutes rows.
#include <string.h>

#include <type_traits>

#include "tc_common.cuh"

namespace exq {
namespace tc {

constexpr int kWarps = 15;
constexpr int kThreads = kWarps * 32;
constexpr int kWarpW = 0, kWarpB = 1, kWarpMma = 2;
constexpr int kEpiWarp0 = 3, kNumEpiWarps = 4;
constexpr int kDqWarp0 = 7, kNumDqWarps = 8;
constexpr int kDqThreads = kNumDqWarps * 32;
constexpr int kWStages = 12, kAStages = 3, kBStages = 3;
constexpr int kWSlot = 4096, kSSlot = 256, kASlot = 16384, kBSlot = 32768;
constexpr int kMaxN = 256;
constexpr int kTmemCols = 512;
constexpr int kKS = 64;  // k per pipeline stage (one 128B swizzle atom of fp16)

constexpr int kOffA = 0;
constexpr int kOffB = kOffA + kAStages * kASlot;
constexpr int kOffW = kOffB + kBStages * kBSlot;
constexpr int kOffS = kOffW + kWStages * kWSlot;
constexpr int kOffBar = kOffS + kWStages * kSSlot;
constexpr int kNumBars = 2 * kWStages + 2 * kAStages + 2 * kBStages + 4;
constexpr int kOffMisc = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffMisc + 64 + 1024;  // + slack to align the base to 1024 B

enum : int { kTierBF16 = EXQ_TIER_BF16, kTierINT8 = EXQ_TIER_INT8, kTierINT4 = EXQ_TIER_INT4 };

struct TcParams {
  CUtensorMap tm_w[3];  // weights of this projection per tier storage
  CUtensorMap tm_s;     // INT4 group scales (group-major) of this projection
  CUtensorMap tm_b;     // activations [n_pos, k] fp16, octet-permuted
  const int32_t* expert_slot;  // tier << 24 | index inside the tier storage
  const int32_t* tile_info;
  const int32_t* n_tiles_ptr;
  int max_tiles;
  const float* sorted_w;  // down: router weight of every sorted position
  const __half* s8;       // INT8 per-row scales of this projection
  int gate_up;            // 1: gate_up (rows interleave gate/up), 0: down
  int n_rows;             // rows of the projection (2I or H)
  int inter;
  int k;
  int nblocks;
  void* out;
  int64_t out_stride;
  uint32_t* status;
};

struct Item {
  int e, m0, mc, nb, tier, idx, n, r0;
};

__device__ __forceinline__ bool decode_item(const TcParams& p, int item, int n_tiles, Item& it) {
  it.nb = item / n_tiles;
  const int tile = item - it.nb * n_tiles;
  it.e = __ldg(p.tile_info + 3 * tile);
  it.m0 = __ldg(p.tile_info + 3 * tile + 1);
  it.mc = __ldg(p.tile_info + 3 * tile + 2);
  const int code = __ldg(p.expert_slot + it.e);
  it.tier = code >> 24;
  it.idx = code & 0xFFFFFF;
  it.n = max(16, (it.mc + 15) & ~15);
  it.r0 = p.gate_up ? it.nb * 64 : it.nb * 128;
  return it.tier == kTierINT4 || it.tier == kTierINT8 || it.tier == kTierBF16;
}

__device__ __forceinline__ int wslots_of(int tier) {
  return tier == kTierINT4 ? 1 : (tier == kTierINT8 ? 2 : 4);
}

struct Ring {
  uint32_t idx = 0, phase = 0;
  __device__ __forceinline__ void next(int n) {
    if (++idx == static_cast<uint32_t>(n)) {
      idx = 0;
      phase ^= 1;
    }
  }
};

// Position of k-index `o` inside its permuted octet (inverse of [0,4,1,5,2,6,3,7]).
__device__ __forceinline__ int perm_pos(int o) {
  return (o & ~7) | (((o & 3) << 1) | ((o >> 2) & 1));
}

// INT4: one packed word (8 weights, reference nibble order) -> 4 fp16 pairs in
// permuted octet order, each multiplied by the group scale.
__device__ __forceinline__ uint4 dq_int4_word(uint32_t w, __half2 s) {
  const __half2 sub = __float2half2_rn(1032.0f);
  const __half2 mul16 = __float2half2_rn(0.0625f);
  const __half2 add72 = __float2half2_rn(-72.0f);
  uint32_t r0 = and_or(w, 0x000F000Fu, 0x64006400u);
  uint32_t r1 = and_or(w, 0x00F000F0u, 0x64006400u);
  const uint32_t w8 = w >> 8;
  uint32_t r2 = and_or(w8, 0x000F000Fu, 0x64006400u);
  uint32_t r3 = and_or(w8, 0x00F000F0u, 0x64006400u);
  __half2 h0 = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&r0), sub), s);
  __half2 h1 = __hmul2(__hfma2(*reinterpret_cast<__half2*>(&r1), mul16, add72), s);
  __half2 h2 = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&r2), sub), s);
  __half2 h3 = __hmul2(__hfma2(*reinterpret_cast<__half2*>(&r3), mul16, add72), s);
  uint4 o;
  o.x = *reinterpret_cast<uint32_t*>(&h0);
  o.y = *reinterpret_cast<uint32_t*>(&h1);
  o.z = *reinterpret_cast<uint32_t*>(&h2);
  o.w = *reinterpret_cast<uint32_t*>(&h3);
  return o;
}

// INT8 (bytes stored in permuted octet order): 4 weights -> 2 fp16 pairs.
__device__ __forceinline__ uint2 dq_int8_word(uint32_t w) {
  const uint32_t u = w ^ 0x80808080u;
  uint32_t a = prmt(u, 0x64646464u, 0x4140u);
  uint32_t b = prmt(u, 0x64646464u, 0x4342u);
  const __half2 sub = __float2half2_rn(1152.0f);
  __half2 ha = __hsub2(*reinterpret_cast<__half2*>(&a), sub);
  __half2 hb = __hsub2(*reinterpret_cast<__half2*>(&b), sub);
  return make_uint2(*reinterpret_cast<uint32_t*>(&ha), *reinterpret_cast<uint32_t*>(&hb));
}

__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};\n" ::"r"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint16_t lds16(uint32_t addr) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];\n" : "=h"(v) : "r"(addr));
  return v;
}

__global__ void __launch_bounds__(kThreads, 1) moe_tc_kernel(const __grid_constant__ TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t sA = base + kOffA, sB = base + kOffB, sW = base + kOffW, sS = base + kOffS;
  const uint32_t bar0 = base + kOffBar;
  auto W_full = [&](int i) { return bar0 + 8u * i; };
  auto W_empty = [&](int i) { return bar0 + 8u * (kWStages + i); };
  auto A_full = [&](int i) { return bar0 + 8u * (2 * kWStages + i); };
  auto A_empty = [&](int i) { return bar0 + 8u * (2 * kWStages + kAStages + i); };
  auto B_full = [&](int i) { return bar0 + 8u * (2 * kWStages + 2 * kAStages + i); };
  auto B_empty = [&](int i) { return bar0 + 8u * (2 * kWStages + 2 * kAStages + kBStages + i); };
  auto Acc_full = [&](int i) { return bar0 + 8u * (2 * kWStages + 2 * kAStages + 2 * kBStages + i); };
  auto Acc_empty = [&](int i) {
    return bar0 + 8u * (2 * kWStages + 2 * kAStages + 2 * kBStages + 2 + i);
  };
  volatile uint32_t* misc = reinterpret_cast<volatile uint32_t*>(gbase + kOffMisc);
  // misc[0] = TMEM base address, misc[1] = abort flag

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = min(*p.n_tiles_ptr, p.max_tiles);
  const int n_items = n_tiles * p.nblocks;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kWStages; ++i) {
      mbar_init(W_full(i), 1);
      mbar_init(W_empty(i), 1);
    }
    for (int i = 0; i < kAStages; ++i) {
      mbar_init(A_full(i), 1);
      mbar_init(A_empty(i), 1);
    }
    for (int i = 0; i < kBStages; ++i) {
      mbar_init(B_full(i), 1);
      mbar_init(B_empty(i), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(Acc_full(i), 1);
      mbar_init(Acc_empty(i), kNumEpiWarps);
    }
    misc[1] = 0;
    mbar_fence_init();
  }
  if (warp == kWarpMma) {
    tmem_alloc(base + kOffMisc, kTmemCols);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[0];
  auto aborted = [&]() { return misc[1] != 0; };
  auto do_abort = [&]() { misc[1] = 1; };

  if (warp == kWarpW) {
    // ---------------------------------------------------------- weights
    if (lane == 0) {
      Ring r;
      int issued = 0;
      const int G = p.k >> 7;
      for (int item = blockIdx.x; item < n_items && !aborted(); item += gridDim.x) {
        Item it;
        if (!decode_item(p, item, n_tiles, it)) {
          atomicOr(p.status, EXQ_DEV_BAD_TIER);
          continue;
        }
        const int nk = p.k / kKS;
        const int ns = wslots_of(it.tier);
        const int rows = p.n_rows;
        for (int kc = 0; kc < nk && !aborted(); ++kc) {
          for (int q = 0; q < ns; ++q) {
            if (!mbar_wait(W_empty(r.idx), r.phase ^ 1, p.status)) {
              do_abort();
              break;
            }
            const uint32_t dst = sW + r.idx * kWSlot, bar = W_full(r.idx);
            if (it.tier == kTierINT4) {
              mbar_arrive_tx(bar, kWSlot + kSSlot);
              const int ybase = it.idx * rows;
              const int y0 = ybase + (p.gate_up ? it.r0 : it.r0);
              const int y1 = ybase + (p.gate_up ? p.inter + it.r0 : it.r0 + 64);
              tma_load_2d(dst, &p.tm_w[kTierINT4], bar, kc * 32, y0);
              tma_load_2d(dst + 2048, &p.tm_w[kTierINT4], bar, kc * 32, y1);
              const int ys = it.idx * G + (kc >> 1);
              const int xs0 = it.r0;
              const int xs1 = p.gate_up ? p.inter + it.r0 : it.r0 + 64;
              tma_load_2d(sS + r.idx * kSSlot, &p.tm_s, bar, xs0, ys);
              tma_load_2d(sS + r.idx * kSSlot + 128, &p.tm_s, bar, xs1, ys);
            } else if (it.tier == kTierINT8) {
              mbar_arrive_tx(bar, kWSlot);
              const int y = it.idx * rows +
                            (p.gate_up ? (q ? p.inter : 0) + it.r0 : it.r0 + 64 * q);
              tma_load_2d(dst, &p.tm_w[kTierINT8], bar, kc * 64, y);
            } else {
              mbar_arrive_tx(bar, kWSlot);
              const int y = it.idx * rows +
                            (p.gate_up ? (q >= 2 ? p.inter : 0) + it.r0 + 32 * (q & 1)
                                       : it.r0 + 32 * q);
              tma_load_2d(dst, &p.tm_w[kTierBF16], bar, kc * 64, y);
            }
            r.next(kWStages);
            ++issued;
          }
        }
      }
      if (aborted()) {  // let in-flight copies land before the CTA exits
        Ring q = r;
        for (int i = 0; i < min(issued, kWStages); ++i) {
          if (q.idx == 0) q.phase ^= 1;
          q.idx = (q.idx + kWStages - 1) % kWStages;
          mbar_wait(W_full(q.idx), q.phase, p.status);
        }
      }
    }
  } else if (warp == kWarpB) {
    // ---------------------------------------------------------- activations
    if (lane == 0) {
      Ring r;
      int issued = 0;
      for (int item = blockIdx.x; item < n_items && !aborted(); item += gridDim.x) {
        Item it;
        if (!decode_item(p, item, n_tiles, it)) continue;
        const int nk = p.k / kKS;
        const int nbox = (it.mc + 31) >> 5;
        for (int kc = 0; kc < nk; ++kc) {
          if (!mbar_wait(B_empty(r.idx), r.phase ^ 1, p.status)) {
            do_abort();
            break;
          }
          const uint32_t bar = B_full(r.idx);
          mbar_arrive_tx(bar, nbox * 4096);
          for (int i = 0; i < nbox; ++i)
            tma_load_2d(sB + r.idx * kBSlot + i * 4096, &p.tm_b, bar, kc * kKS, it.m0 + 32 * i);
          r.next(kBStages);
          ++issued;
        }
      }
      if (aborted()) {
        Ring q = r;
        for (int i = 0; i < min(issued, kBStages); ++i) {
          if (q.idx == 0) q.phase ^= 1;
          q.idx = (q.idx + kBStages - 1) % kBStages;
          mbar_wait(B_full(q.idx), q.phase, p.status);
        }
      }
    }
  } else if (warp == kWarpMma) {
    // ---------------------------------------------------------- MMA issue
    if (lane == 0) {
      Ring ra, rb;
      int count = 0;
      for (int item = blockIdx.x; item < n_items && !aborted(); item += gridDim.x, ++count) {
        Item it;
        if (!decode_item(p, item, n_tiles, it)) {
          --count;
          continue;
        }
        const int ab = count & 1;
        const uint32_t acc_phase = (count >> 1) & 1;
        if (!mbar_wait(Acc_empty(ab), acc_phase ^ 1, p.status)) {
          do_abort();
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + ab * kMaxN;
        const uint32_t idesc = idesc_f16_m128(it.n);
        const int nk = p.k / kKS;
        bool ok = true;
        for (int kc = 0; kc < nk; ++kc) {
          if (!mbar_wait(A_full(ra.idx), ra.phase, p.status) ||
              !mbar_wait(B_full(rb.idx), rb.phase, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = sA + ra.idx * kASlot, b = sB + rb.idx * kBSlot;
#pragma unroll
          for (int k = 0; k < kKS / 16; ++k)
            tc_mma_f16(d, smem_desc_sw128(a + 32 * k), smem_desc_sw128(b + 32 * k), idesc,
                       (kc | k) != 0);
          tc_commit(A_empty(ra.idx));
          tc_commit(B_empty(rb.idx));
          ra.next(kAStages);
          rb.next(kBStages);
        }
        if (!ok) {
          do_abort();
          break;
        }
        tc_commit(Acc_full(ab));
      }
    }
  } else if (warp < kDqWarp0) {
    // ---------------------------------------------------------- epilogue
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
    const int row = 32 * quarter + lane;
    int count = 0;
    for (int item = blockIdx.x; item < n_items && !aborted(); item += gridDim.x, ++count) {
      Item it;
      if (!decode_item(p, item, n_tiles, it)) {
        --count;
        continue;
      }
      const int ab = count & 1;
      const uint32_t acc_phase = (count >> 1) & 1;
      const bool got = mbar_wait(Acc_full(ab), acc_phase, p.status);
      if (!__all_sync(0xffffffffu, got)) {  // keep the warp converged
        do_abort();
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem + (static_cast<uint32_t>(32 * quarter) << 16) + ab * kMaxN;
      if (p.gate_up) {
        // row 2j = gate g, row 2j+1 = up g, with g = r0 + row/2
        const int g = it.r0 + (row >> 1);
        const bool is_up = row & 1;
        float sg = 1.f, su = 1.f;
        if (it.tier == kTierINT8) {
          const int64_t rb = static_cast<int64_t>(it.idx) * p.n_rows;
          sg = __half2float(p.s8[rb + g]);
          su = __half2float(p.s8[rb + p.inter + g]);
        }
        __half* mid = static_cast<__half*>(p.out);
        const int col = perm_pos(g);
        for (int c = 0; c < it.n; c += 16) {
          uint32_t v[16];
          tmem_ld16(taddr + c, v);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float own = __uint_as_float(v[i]);
            const float other = __shfl_xor_sync(0xffffffffu, own, 1);
            const float gate = (is_up ? other : own) * sg;
            const float up = (is_up ? own : other) * su;
            // even lanes store tokens c..c+7, odd lanes c+8..c+15
            if ((i >> 3) == (is_up ? 1 : 0)) {
              const int tok = c + i;
              if (tok < it.mc) {
                const float m = gate / (1.0f + expf(-gate)) * up;
                mid[static_cast<int64_t>(it.m0 + tok) * p.out_stride + col] =
                    __float2half_rn(m);
              }
            }
          }
        }
      } else {
        const int h = it.r0 + row;
        float s = 1.f;
        if (it.tier == kTierINT8) s = __half2float(p.s8[static_cast<int64_t>(it.idx) * p.n_rows + h]);
        float* part = static_cast<float*>(p.out);
        for (int c = 0; c < it.n; c += 16) {
          uint32_t v[16];
          tmem_ld16(taddr + c, v);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int tok = c + i;
            if (tok < it.mc) {
              const int64_t pos = it.m0 + tok;
              part[pos * p.out_stride + h] = __uint_as_float(v[i]) * s * __ldg(p.sorted_w + pos);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(Acc_empty(ab));
    }
  } else {
    // ---------------------------------------------------------- dequant
    const int dt = threadIdx.x - kDqWarp0 * 32;
    const int r = dt >> 1, hh = dt & 1;  // A row, half of its 64 k
    const uint32_t arow_off = (r >> 3) * 1024 + (r & 7) * 128;
    const int sw = r & 7;
    Ring rw, ra;
    for (int item = blockIdx.x; item < n_items && !aborted(); item += gridDim.x) {
      Item it;
      if (!decode_item(p, item, n_tiles, it)) continue;
      const int lw = p.gate_up ? ((r & 1) ? 64 + (r >> 1) : (r >> 1)) : r;
      const int nk = p.k / kKS;
      const int ns = wslots_of(it.tier);
      bool ok = true;
      for (int kc = 0; kc < nk && ok; ++kc) {
        bool mine = mbar_wait(A_empty(ra.idx), ra.phase ^ 1, p.status);
        uint32_t slots[4];
        Ring rq = rw;
        for (int q = 0; q < ns; ++q) {
          slots[q] = rq.idx;
          if (mine && !mbar_wait(W_full(rq.idx), rq.phase, p.status)) mine = false;
          rq.next(kWStages);
        }
        // every dequant thread reaches this barrier; one failed wait stops all
        if (named_barrier_or(2, kDqThreads, !mine)) {
          ok = false;
          break;
        }
        const uint32_t adst = sA + ra.idx * kASlot + arow_off;
        if (it.tier == kTierINT4) {
          const uint32_t src = sW + slots[0] * kWSlot + lw * 32 + hh * 16;
          const uint4 wv = lds128(src);
          const uint16_t sraw = lds16(sS + slots[0] * kSSlot + lw * 2);
          const __half2 s2 = __halves2half2(__ushort_as_half(sraw), __ushort_as_half(sraw));
          sts128(adst + (((4 * hh + 0) ^ sw) << 4), dq_int4_word(wv.x, s2));
          sts128(adst + (((4 * hh + 1) ^ sw) << 4), dq_int4_word(wv.y, s2));
          sts128(adst + (((4 * hh + 2) ^ sw) << 4), dq_int4_word(wv.z, s2));
          sts128(adst + (((4 * hh + 3) ^ sw) << 4), dq_int4_word(wv.w, s2));
        } else if (it.tier == kTierINT8) {
          const uint32_t src = sW + slots[lw >> 6] * kWSlot + (lw & 63) * 64 + hh * 32;
          const uint4 w0 = lds128(src), w1 = lds128(src + 16);
          const uint32_t ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint2 a = dq_int8_word(ws[2 * j]), b = dq_int8_word(ws[2 * j + 1]);
            sts128(adst + (((4 * hh + j) ^ sw) << 4), make_uint4(a.x, a.y, b.x, b.y));
          }
        } else {
          // 16-bit rows arrive 128B-swizzled: chunk c of slot row t at c ^ (t & 7)
          const int t = lw & 31;
          const uint32_t src = sW + slots[lw >> 5] * kWSlot + t * 128;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int c = 4 * hh + j;
            sts128(adst + ((c ^ sw) << 4), lds128(src + ((c ^ (t & 7)) << 4)));
          }
        }
        fence_proxy_async_smem();
        named_barrier(1, kDqThreads);
        if (dt == 0) {
          for (int q = 0; q < ns; ++q) mbar_arrive(W_empty(slots[q]));
          mbar_arrive(A_full(ra.idx));
        }
        for (int q = 0; q < ns; ++q) rw.next(kWStages);
        ra.next(kAStages);
      }
      if (!ok) {
        do_abort();
        break;
      }
    }
  }

  // producer / MMA warps arrive here diverged (only lane 0 worked)
  cta_barrier_unaligned();
  if (warp == kWarpMma) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Activation prep: A[pos, :] = fp16(hidden[token(pos), :]) with every octet of
// k permuted to [0,4,1,5,2,6,3,7].
template <typename T>
__global__ void prep_act_kernel(const T* __restrict__ hidden, int64_t hid, const int32_t* sorted_slot,
                                int spt, int64_t n_pos, __half* __restrict__ out) {
  const int64_t octs = hid / 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n_pos * octs;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t pos = i / octs, o = i - pos * octs;
    const int64_t tok = sorted_slot[pos] / spt;
    const uint4 v = reinterpret_cast<const uint4*>(hidden + tok * hid)[o];
    uint32_t w[4] = {v.x, v.y, v.z, v.w};
    if (!std::is_same<T, __half>::value) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&w[j]);
        const float2 f = __bfloat1622float2(b);
        __half2 hf = __floats2half2_rn(f.x, f.y);
        w[j] = *reinterpret_cast<uint32_t*>(&hf);
      }
    }
    uint4 r;
    r.x = prmt(w[0], w[2], 0x5410u);  // (k0, k4)
    r.y = prmt(w[0], w[2], 0x7632u);  // (k1, k5)
    r.z = prmt(w[1], w[3], 0x5410u);  // (k2, k6)
    r.w = prmt(w[1], w[3], 0x7632u);  // (k3, k7)
    reinterpret_cast<uint4*>(out + pos * hid)[o] = r;
  }
}

}  // namespace tc
}  // namespace exq

// ============================================================== host side
namespace exq {
namespace tc {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// 2D row-major tensor [outer, inner] with `row_bytes` between rows.
static bool make_map(CUtensorMap* m, CUtensorMapDataType dt, const void* ptr, uint64_t inner,
                     uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                     CUtensorMapSwizzle sw, CUtensorMapL2promotion l2) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is unavailable from the driver");
    return false;
  }
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, l2, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) for a [%llu x %llu] tensor", (int)r,
              (unsigned long long)outer, (unsigned long long)inner);
    return false;
  }
  return true;
}

// Fill the per-projection maps.  proj 0 = w13 (rows 2I, k = H), 1 = w2 (rows H, k = I).
static int build_maps(const exq_moe_weights* w, int proj, const void* act, int64_t n_pos,
                      TcParams& p) {
  const int64_t rows = proj == 0 ? 2 * w->inter : w->hidden;
  const int64_t k = proj == 0 ? w->hidden : w->inter;
  memset(p.tm_w, 0, sizeof(p.tm_w));
  memset(&p.tm_s, 0, sizeof(p.tm_s));
  const int n4 = w->n_tier[EXQ_TIER_INT4], n8 = w->n_tier[EXQ_TIER_INT8],
            n16 = w->n_tier[EXQ_TIER_BF16];
  const void* const* wt = proj == 0 ? w->w13 : w->w2;
  const void* const* st = proj == 0 ? w->w13_scales : w->w2_scales;
  if (n4 > 0) {
    if (!make_map(&p.tm_w[EXQ_TIER_INT4], CU_TENSOR_MAP_DATA_TYPE_UINT8, wt[EXQ_TIER_INT4], k / 2,
                  (uint64_t)n4 * rows, k / 2, 32, 64, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B) ||
        !make_map(&p.tm_s, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, st[EXQ_TIER_INT4], rows,
                  (uint64_t)n4 * (k / 128), rows * 2, 64, 1, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B))
      return EXQ_ERR_CUDA;
  }
  if (n8 > 0) {
    if (!make_map(&p.tm_w[EXQ_TIER_INT8], CU_TENSOR_MAP_DATA_TYPE_UINT8, wt[EXQ_TIER_INT8], k,
                  (uint64_t)n8 * rows, k, 64, 64, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B))
      return EXQ_ERR_CUDA;
  }
  if (n16 > 0) {
    if (!make_map(&p.tm_w[EXQ_TIER_BF16], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, wt[EXQ_TIER_BF16], k,
                  (uint64_t)n16 * rows, 2 * k, 64, 32, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B))
      return EXQ_ERR_CUDA;
  }
  if (!make_map(&p.tm_b, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, act, k, (uint64_t)n_pos, 2 * k, 64, 32,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B))
    return EXQ_ERR_CUDA;
  p.s8 = static_cast<const __half*>(st[EXQ_TIER_INT8]);
  p.n_rows = static_cast<int>(rows);
  p.k = static_cast<int>(k);
  return EXQ_OK;
}

int launch_tc(const TcParams& p, int max_items, cudaStream_t stream) {
  static int attr_done[64] = {0};
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(moe_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSmemBytes);
    if (e != cudaSuccess) {
      set_error("moe_tc_kernel: cannot reserve %d B of shared memory: %s", kSmemBytes,
                cudaGetErrorString(e));
      return EXQ_ERR_CUDA;
    }
    sms[dev] = num_sms();
    attr_done[dev] = 1;
  }
  int grid = sms[dev];
  if (max_items < grid) grid = max_items;
  if (grid < 1) grid = 1;
  moe_tc_kernel<<<grid, kThreads, kSmemBytes, stream>>>(p);
  EXQ_CHECK_LAUNCH("moe_tc_kernel");
  return EXQ_OK;
}

int launch_prep(const void* hidden, int act_dtype, int64_t hid, const int32_t* sorted_slot,
                int spt, int64_t n_pos, __half* out, cudaStream_t stream) {
  if (n_pos == 0) return EXQ_OK;
  const int64_t work = n_pos * (hid / 8);
  int64_t grid = (work + 255) / 256;
  if (grid > 65535) grid = 65535;
  if (act_dtype == EXQ_F16)
    prep_act_kernel<__half><<<(int)grid, 256, 0, stream>>>(static_cast<const __half*>(hidden), hid,
                                                           sorted_slot, spt, n_pos, out);
  else
    prep_act_kernel<__nv_bfloat16><<<(int)grid, 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(hidden), hid, sorted_slot, spt, n_pos, out);
  EXQ_CHECK_LAUNCH("prep_act_kernel");
  return EXQ_OK;
}

}  // namespace tc
}  // namespace exq

// ============================================================== C ABI
using namespace exq;

namespace {

constexpr int kLayerMT = tc::kMaxN;  // tokens per GEMM tile (the MMA's N)

struct TcWs {
  int32_t* sorted_slot;
  int32_t* pos_of_slot;
  float* sorted_w;
  int32_t* ends;
  int32_t* tile_info;
  int32_t* n_tiles;
  __half* act;
  __half* mid;
  float* partial;
  int64_t max_tiles;
  size_t bytes;
};

TcWs carve_tc(void* base, int64_t n_slots, int n_buckets, int64_t hidden, int64_t inter) {
  TcWs w{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 256);
    return base ? static_cast<char*>(base) + o : nullptr;
  };
  w.max_tiles = n_slots / kLayerMT + (n_slots < n_buckets ? n_slots : n_buckets) + 1;
  w.sorted_slot = reinterpret_cast<int32_t*>(take(4 * n_slots));
  w.pos_of_slot = reinterpret_cast<int32_t*>(take(4 * n_slots));
  w.sorted_w = reinterpret_cast<float*>(take(4 * n_slots));
  w.ends = reinterpret_cast<int32_t*>(take(4 * (n_buckets + 1)));
  w.tile_info = reinterpret_cast<int32_t*>(take(12 * w.max_tiles));
  w.n_tiles = reinterpret_cast<int32_t*>(take(16));
  w.act = reinterpret_cast<__half*>(take(2 * n_slots * hidden));
  w.mid = reinterpret_cast<__half*>(take(2 * n_slots * inter));
  w.partial = reinterpret_cast<float*>(take(4 * n_slots * hidden));
  w.bytes = off;
  return w;
}

bool is_act(int d) { return d == EXQ_F16 || d == EXQ_BF16; }

}  // namespace

extern "C" size_t exq_moe_layer_workspace_bytes(int64_t n_tokens, int32_t top_k, int32_t n_shared,
                                                int32_t n_experts_total, int64_t hidden,
                                                int64_t inter) {
  if (n_tokens < 0 || top_k <= 0 || n_shared < 0 || n_experts_total <= 0) return 0;
  return carve_tc(nullptr, n_tokens * (top_k + n_shared), n_experts_total, hidden, inter).bytes;
}

extern "C" int exq_moe_layer_forward(const exq_moe_weights* weights, const void* hidden_states,
                                     int act_dtype, int64_t n_tokens, const void* topk_ids,
                                     int ids_dtype, const void* topk_weights, int w_dtype,
                                     int32_t top_k, void* out, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  return exq_moe_layer_forward_range(weights, hidden_states, act_dtype, n_tokens, topk_ids,
                                     ids_dtype, topk_weights, w_dtype, top_k, out, workspace,
                                     workspace_bytes, stream, 0, EXQ_LAYER_STAGES);
}

extern "C" int exq_moe_layer_forward_range(const exq_moe_weights* w, const void* hidden_states,
                                           int act_dtype, int64_t n_tokens, const void* topk_ids,
                                           int ids_dtype, const void* topk_weights, int w_dtype,
                                           int32_t top_k, void* out, void* workspace,
                                           size_t workspace_bytes, void* stream,
                                           int32_t first_stage, int32_t end_stage) {
  EXQ_CHECK_ARG(w, "moe_layer: weights is null");
  EXQ_CHECK_ARG(0 <= first_stage && first_stage <= end_stage && end_stage <= EXQ_LAYER_STAGES,
                "moe_layer: stage range [%d, %d) outside [0, %d)", first_stage, end_stage,
                EXQ_LAYER_STAGES);
  EXQ_CHECK_ARG(is_act(act_dtype), "moe_layer: activations must be fp16 or bf16");
  EXQ_CHECK_ARG(ids_dtype == EXQ_I32 || ids_dtype == EXQ_I64, "moe_layer: ids must be int32/int64");
  EXQ_CHECK_ARG(w_dtype == EXQ_F32 || is_act(w_dtype), "moe_layer: weights dtype unsupported");
  EXQ_CHECK_ARG(w->n_routed > 0 && w->n_shared >= 0 && top_k > 0 && n_tokens >= 0,
                "moe_layer: bad sizes");
  const int64_t H = w->hidden, I = w->inter;
  if (H <= 0 || H % 128 != 0 || I <= 0 || I % 128 != 0) {
    set_error("moe_layer: hidden=%lld and inter=%lld must be positive multiples of 128",
              (long long)H, (long long)I);
    return EXQ_ERR_UNSUPPORTED;
  }
  const int32_t n_total = w->n_routed + w->n_shared;
  int32_t tier_sum = 0;
  for (int t = 0; t < 3; ++t) {
    EXQ_CHECK_ARG(w->n_tier[t] >= 0, "moe_layer: negative tier count");
    tier_sum += w->n_tier[t];
    if (w->n_tier[t] > 0) {
      EXQ_CHECK_ARG(w->w13[t] && w->w2[t], "moe_layer: tier %d storage is null", t);
      EXQ_CHECK_ARG(t == EXQ_TIER_BF16 || (w->w13_scales[t] && w->w2_scales[t]),
                    "moe_layer: tier %d scales are null", t);
      EXQ_CHECK_ARG((reinterpret_cast<uintptr_t>(w->w13[t]) | reinterpret_cast<uintptr_t>(w->w2[t])) % 16 == 0,
                    "moe_layer: tier %d storage is not 16-byte aligned", t);
    }
  }
  EXQ_CHECK_ARG(tier_sum >= 1 && w->expert_slot, "moe_layer: no expert storage");
  const int spt = top_k + w->n_shared;
  const int64_t n_slots = n_tokens * spt;
  const size_t need = exq_moe_layer_workspace_bytes(n_tokens, top_k, w->n_shared, n_total, H, I);
  if (!workspace || workspace_bytes < need) {
    set_error("moe_layer: workspace of %zu bytes needed", need);
    return EXQ_ERR_WORKSPACE;
  }
  if (n_tokens == 0) return EXQ_OK;
  EXQ_CHECK_ARG(hidden_states && topk_ids && topk_weights && out, "moe_layer: null pointer");
  EXQ_CHECK_ARG(reinterpret_cast<uintptr_t>(hidden_states) % 16 == 0,
                "moe_layer: hidden_states must be 16-byte aligned");
  auto s = static_cast<cudaStream_t>(stream);
  TcWs ws = carve_tc(workspace, n_slots, n_total, H, I);
  uint32_t* status = device_status_ptr();
  if (!status) return EXQ_ERR_CUDA;
  int st = EXQ_OK;

  if (first_stage <= 0 && end_stage > 0) {
    RouteParams rp{};
    rp.ids = topk_ids;
    rp.ids_dtype = ids_dtype;
    rp.n = n_slots;
    rp.n_buckets = n_total;
    rp.n_routed = w->n_routed;
    rp.top_k = top_k;
    rp.slots_per_token = spt;
    rp.mt = kLayerMT;
    rp.sorted_i32 = ws.sorted_slot;
    rp.pos_of_slot = ws.pos_of_slot;
    rp.sorted_w = ws.sorted_w;
    rp.topk_w = topk_weights;
    rp.w_dtype = w_dtype;
    rp.ends = ws.ends;
    rp.tile_info = ws.tile_info;
    rp.n_tiles = ws.n_tiles;
    rp.max_tiles = ws.max_tiles;
    st = launch_route(rp, kRouteLayer, s);
    if (st != EXQ_OK) return st;
  }
  if (first_stage <= 1 && end_stage > 1) {
    st = tc::launch_prep(hidden_states, act_dtype, H, ws.sorted_slot, spt, n_slots, ws.act, s);
    if (st != EXQ_OK) return st;
  }
  for (int proj = 0; proj < 2; ++proj) {
    const int stage = 2 + proj;
    if (!(first_stage <= stage && end_stage > stage)) continue;
    tc::TcParams p;
    memset(&p, 0, sizeof(p));
    st = tc::build_maps(w, proj, proj == 0 ? ws.act : ws.mid, n_slots, p);
    if (st != EXQ_OK) return st;
    p.expert_slot = w->expert_slot;
    p.tile_info = ws.tile_info;
    p.n_tiles_ptr = ws.n_tiles;
    p.max_tiles = static_cast<int>(ws.max_tiles);
    p.sorted_w = ws.sorted_w;
    p.gate_up = proj == 0;
    p.inter = static_cast<int>(I);
    p.nblocks = static_cast<int>(proj == 0 ? I / 64 : H / 128);
    p.out = proj == 0 ? static_cast<void*>(ws.mid) : static_cast<void*>(ws.partial);
    p.out_stride = proj == 0 ? I : H;
    p.status = status;
    const int64_t max_items = ws.max_tiles * p.nblocks;
    st = tc::launch_tc(p, static_cast<int>(max_items < INT32_MAX ? max_items : INT32_MAX), s);
    if (st != EXQ_OK) return st;
  }
  if (first_stage <= 4 && end_stage > 4)
    return launch_combine_partials(ws.partial, H, ws.pos_of_slot, n_tokens, spt, out, act_dtype, s);
  return EXQ_OK;
}
