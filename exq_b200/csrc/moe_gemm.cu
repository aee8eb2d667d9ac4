// Grouped expert GEMMs for the decode-shaped MoE path (small rows per expert).
//
// Replaces the Triton `_moe_gemm_int4_kernel` (exq/kernels/moe_int4_kernel.py
// :124-240) and `_moe_gemm_kernel` (exq/kernels/moe_grouped_gemm.py:47-132),
// plus the gather (exq_dispatch.cu:234-260), SiLU*mul and the down-proj
// half of the combine, for experts that mix three weight tiers in one launch.
//
// Decomposition.  The route kernel lists GEMM tiles (expert, first sorted row,
// <= 32 rows).  A work item is (row block of the weight matrix, tile); items
// are numbered row-block-major so consecutive items are the m-tiles of one
// expert reading the same weight block (the second read hits L2).  The grid
// is persistent: each CTA walks items blockIdx.x, +gridDim.x, ...
//
// Data flow per item.  The weight matrix is streamed once, in k-chunks of 64
// bytes per row (128 INT4 / 64 INT8 / 32 16-bit values), 128 rows per CTA,
// through a 4-stage cp.async ring; the activation rows of the tile (gathered
// through the sorted slot list, never materialised) ride in the same stages.
// The load cursor runs 3 stages ahead of compute and crosses item boundaries,
// so the pipeline never drains between items.
//
// Math.  Swap-AB warp MMA m16n8k16: 16 weight rows x 8 token columns.  Lane
// (g = lane/4, q = lane%4) reads one 16-byte slab per weight row and chunk,
// the 1/4 of the chunk's k range that belongs to q; the k order inside an
// MMA is permuted identically for weights and activations (a dot product
// does not depend on the order of its terms), which lets both operands come
// from single 128-bit shared loads.  INT4/INT8 weights are dequantised to
// the exact integers q (fp16 and bf16 hold them exactly); INT4 group scales
// are applied in fp32 to each chunk's partial sum (chunk == group of 128),
// INT8 row scales in the epilogue.  Accumulation is fp32 throughout.
#include "internal.cuh"

namespace exq {

constexpr int kGmThreads = 128;  // 4 warps
constexpr int kGmWarps = 4;
constexpr int kGmR = 2;             // 16-row MMA tiles per warp
constexpr int kGmRB = kGmWarps * kGmR * 16;  // 128 weight rows per item
static_assert(kGmRB == kGmRBHost, "row block mismatch");
constexpr int kGmMT = kGmMTHost;     // max token rows per tile
constexpr int kGmNT = kGmMT / 8;    // max 8-column MMA tiles
constexpr int kGmS = 4;             // pipeline stages
constexpr int kStageW = kGmRB * 64;   // 8 KB of weights
constexpr int kStageA = kGmMT * 256;  // 8 KB of activations (<= 128 values of 2 B per row)
constexpr int kStageBytes = kStageW + kStageA;
constexpr int kGmSmem = kGmS * kStageBytes;

__host__ __device__ constexpr int tier_ks(int tier) {
  return tier == EXQ_TIER_INT4 ? 128 : (tier == EXQ_TIER_INT8 ? 64 : 32);
}

__device__ __forceinline__ int act_swizzle(int n, int c, int tier) {
  if (tier == EXQ_TIER_INT4) return c ^ ((n & 1) | (((c >> 3) & 1) << 1));
  if (tier == EXQ_TIER_INT8) return c ^ (n & 1);
  return c ^ ((n & 1) << 2);
}

// Weight row of local row lr (0..127) in row block nb; -1 when out of range.
__device__ __forceinline__ int weight_row(const GemmParams& p, int nb, int lr) {
  if (p.mode == kGemmModeGateUp) {
    const int g = nb * (kGmRB / 2) + (lr >> 4) * 8 + (lr & 7);
    if (g >= p.inter) return -1;
    return (lr & 8) ? p.inter + g : g;
  }
  const int r = nb * kGmRB + lr;
  return r < p.n_rows ? r : -1;
}

struct ItemInfo {
  int e, m0, mc, nb, tier, nk;
  const uint8_t* w;
  const __half* s;
  int64_t row_bytes;
};

__device__ __forceinline__ void decode_item(const GemmParams& p, int item, int n_tiles,
                                            ItemInfo& it) {
  it.nb = item / n_tiles;
  const int tile = item - it.nb * n_tiles;
  it.e = p.tile_info[tile * 3 + 0];
  it.m0 = p.tile_info[tile * 3 + 1];
  it.mc = p.tile_info[tile * 3 + 2];
  const exq_expert_desc& d = p.experts[it.e];
  it.tier = d.tier;
  it.w = static_cast<const uint8_t*>(p.proj ? d.w2 : d.w13);
  it.s = static_cast<const __half*>(p.proj ? d.w2_scales : d.w13_scales);
  if (it.tier != EXQ_TIER_INT4 && it.tier != EXQ_TIER_INT8 && it.tier != EXQ_TIER_BF16) {
    if (threadIdx.x == 0) atomicOr(p.status, EXQ_DEV_BAD_TIER);
    it.tier = -1;
    it.nk = 0;
    return;
  }
  it.row_bytes = it.tier == EXQ_TIER_INT4 ? p.k / 2 : (it.tier == EXQ_TIER_INT8 ? p.k : 2 * p.k);
  it.nk = p.k / tier_ks(it.tier);
}

// Per-thread loader state for one item: the activation rows this thread copies.
struct LoadCtx {
  ItemInfo it;
  const uint8_t* arow[4];
};

__device__ __forceinline__ void setup_load(const GemmParams& p, int item, int n_tiles,
                                           LoadCtx& L) {
  decode_item(p, item, n_tiles, L.it);
  if (L.it.tier < 0) return;
  const int cpr = tier_ks(L.it.tier) * 2 / 16;  // 16-byte chunks per activation row
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int idx = threadIdx.x + kGmThreads * i;
    const int n = idx / cpr;
    L.arow[i] = nullptr;
    if (idx < kGmMT * cpr && n < L.it.mc) {
      int64_t row;
      if (p.gather) {
        row = p.sorted_slot[L.it.m0 + n] / p.spt;
      } else {
        row = L.it.m0 + n;
      }
      L.arow[i] = static_cast<const uint8_t*>(p.act) + row * p.act_stride * 2;
    }
  }
}

__device__ __forceinline__ void issue_stage(const GemmParams& p, const LoadCtx& L, int kc,
                                            uint32_t sbase, uint64_t wpol) {
  const ItemInfo& it = L.it;
  const uint32_t sw = sbase, sa = sbase + kStageW;
  // weights: 128 rows x 4 chunks of 16 B
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int idx = threadIdx.x + kGmThreads * i;
    const int lr = idx >> 2, ch = idx & 3;
    const int row = weight_row(p, it.nb, lr);
    const uint32_t dst = sw + lr * 64 + ch * 16;
    if (row >= 0) {
      cp_async16_hint(dst, it.w + row * it.row_bytes + kc * 64 + ch * 16, wpol);
    } else {
      cp_async16(dst, it.w, 0);
    }
  }
  // activations: rows of the tile, chunk c of this k-chunk
  const int ks = tier_ks(it.tier);
  const int cpr = ks * 2 / 16;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int idx = threadIdx.x + kGmThreads * i;
    if (L.arow[i] != nullptr) {
      const int n = idx / cpr, c = idx - (idx / cpr) * cpr;
      const uint32_t dst = sa + n * 256 + (act_swizzle(n, c, it.tier) << 4);
      cp_async16(dst, L.arow[i] + (int64_t)kc * ks * 2 + c * 16, 16);
    }
  }
}

// Scale of weight row `row` for INT4 group kc (fp16 -> fp32).
__device__ __forceinline__ float int4_scale(const ItemInfo& it, int k, int row, int kc) {
  if (row < 0) return 0.f;
  return __half2float(it.s[(int64_t)row * (k >> 7) + kc]);
}

template <typename T>
struct Acc {
  float v[kGmR][kGmNT][4];
};

template <typename T>
__device__ __forceinline__ void compute_stage(const GemmParams& p, const ItemInfo& it, int kc,
                                              uint32_t sbase, int nt_used, int (&rows)[kGmR][2],
                                              Acc<T>& acc) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, q = lane & 3;
  const uint32_t sw = sbase, sa = sbase + kStageW;
  uint4 wr[kGmR][2];
#pragma unroll
  for (int rt = 0; rt < kGmR; ++rt) {
    const int lr = (warp * kGmR + rt) * 16 + g;
    wr[rt][0] = lds128(sw + lr * 64 + q * 16);
    wr[rt][1] = lds128(sw + (lr + 8) * 64 + q * 16);
  }
  const T tag{};
  if (it.tier == EXQ_TIER_INT4) {
    float sc[kGmR][2];
#pragma unroll
    for (int rt = 0; rt < kGmR; ++rt) {
      sc[rt][0] = int4_scale(it, p.k, rows[rt][0], kc);
      sc[rt][1] = int4_scale(it, p.k, rows[rt][1], kc);
    }
    float tmp[kGmR][kGmNT][4];
#pragma unroll
    for (int rt = 0; rt < kGmR; ++rt)
#pragma unroll
      for (int nt = 0; nt < kGmNT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) tmp[rt][nt][i] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint4 x[kGmNT];
#pragma unroll
      for (int nt = 0; nt < kGmNT; ++nt) {
        if (nt < nt_used) {
          const int n = nt * 8 + g;
          const int c = 4 * q + j;
          x[nt] = lds128(sa + n * 256 + (act_swizzle(n, c, EXQ_TIER_INT4) << 4));
        }
      }
      typename Dq<T>::Word w0[kGmR], w1[kGmR];
#pragma unroll
      for (int rt = 0; rt < kGmR; ++rt) {
        const uint32_t a0 = j == 0 ? wr[rt][0].x : j == 1 ? wr[rt][0].y : j == 2 ? wr[rt][0].z : wr[rt][0].w;
        const uint32_t a1 = j == 0 ? wr[rt][1].x : j == 1 ? wr[rt][1].y : j == 2 ? wr[rt][1].z : wr[rt][1].w;
        w0[rt] = Dq<T>::prep(a0);
        w1[rt] = Dq<T>::prep(a1);
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int rt = 0; rt < kGmR; ++rt) {
          uint32_t a[4];
          a[0] = Dq<T>::int4_pair(w0[rt], 2 * h);
          a[1] = Dq<T>::int4_pair(w1[rt], 2 * h);
          a[2] = Dq<T>::int4_pair(w0[rt], 2 * h + 1);
          a[3] = Dq<T>::int4_pair(w1[rt], 2 * h + 1);
#pragma unroll
          for (int nt = 0; nt < kGmNT; ++nt) {
            if (nt < nt_used) {
              const uint32_t b0 = h ? x[nt].z : x[nt].x;
              const uint32_t b1 = h ? x[nt].w : x[nt].y;
              mma16816(tmp[rt][nt], a, b0, b1, tag);
            }
          }
        }
      }
    }
#pragma unroll
    for (int rt = 0; rt < kGmR; ++rt)
#pragma unroll
      for (int nt = 0; nt < kGmNT; ++nt) {
        acc.v[rt][nt][0] = fmaf(sc[rt][0], tmp[rt][nt][0], acc.v[rt][nt][0]);
        acc.v[rt][nt][1] = fmaf(sc[rt][0], tmp[rt][nt][1], acc.v[rt][nt][1]);
        acc.v[rt][nt][2] = fmaf(sc[rt][1], tmp[rt][nt][2], acc.v[rt][nt][2]);
        acc.v[rt][nt][3] = fmaf(sc[rt][1], tmp[rt][nt][3], acc.v[rt][nt][3]);
      }
  } else if (it.tier == EXQ_TIER_INT8) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      uint4 x[kGmNT];
#pragma unroll
      for (int nt = 0; nt < kGmNT; ++nt) {
        if (nt < nt_used) {
          const int n = nt * 8 + g;
          const int c = 2 * q + j;
          x[nt] = lds128(sa + n * 256 + (act_swizzle(n, c, EXQ_TIER_INT8) << 4));
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int rt = 0; rt < kGmR; ++rt) {
          const int wi = 2 * j + h;
          const uint32_t r0 = (wi == 0 ? wr[rt][0].x : wi == 1 ? wr[rt][0].y : wi == 2 ? wr[rt][0].z : wr[rt][0].w) ^ 0x80808080u;
          const uint32_t r1 = (wi == 0 ? wr[rt][1].x : wi == 1 ? wr[rt][1].y : wi == 2 ? wr[rt][1].z : wr[rt][1].w) ^ 0x80808080u;
          uint32_t a[4];
          a[0] = Dq<T>::int8_pair(r0, 0);
          a[1] = Dq<T>::int8_pair(r1, 0);
          a[2] = Dq<T>::int8_pair(r0, 1);
          a[3] = Dq<T>::int8_pair(r1, 1);
#pragma unroll
          for (int nt = 0; nt < kGmNT; ++nt) {
            if (nt < nt_used) {
              const uint32_t b0 = h ? x[nt].z : x[nt].x;
              const uint32_t b1 = h ? x[nt].w : x[nt].y;
              mma16816(acc.v[rt][nt], a, b0, b1, tag);
            }
          }
        }
      }
    }
  } else {  // 16-bit weights
    uint4 x[kGmNT];
#pragma unroll
    for (int nt = 0; nt < kGmNT; ++nt) {
      if (nt < nt_used) {
        const int n = nt * 8 + g;
        x[nt] = lds128(sa + n * 256 + (act_swizzle(n, q, EXQ_TIER_BF16) << 4));
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int rt = 0; rt < kGmR; ++rt) {
        uint32_t a[4];
        a[0] = h ? wr[rt][0].z : wr[rt][0].x;
        a[1] = h ? wr[rt][1].z : wr[rt][1].x;
        a[2] = h ? wr[rt][0].w : wr[rt][0].y;
        a[3] = h ? wr[rt][1].w : wr[rt][1].y;
#pragma unroll
        for (int nt = 0; nt < kGmNT; ++nt) {
          if (nt < nt_used) {
            const uint32_t b0 = h ? x[nt].z : x[nt].x;
            const uint32_t b1 = h ? x[nt].w : x[nt].y;
            mma16816(acc.v[rt][nt], a, b0, b1, tag);
          }
        }
      }
    }
  }
}

__device__ __forceinline__ float slot_weight(const GemmParams& p, int slot) {
  const int t = slot / p.spt;
  const int j = slot - t * p.spt;
  if (j >= p.top_k) return 1.0f;
  return load_as_f32(p.topk_w, p.w_dtype, (int64_t)t * p.top_k + j);
}

__device__ __forceinline__ void store_out(void* out, int dtype, int64_t idx, float v) {
  if (dtype == EXQ_F16) {
    static_cast<__half*>(out)[idx] = __float2half_rn(v);
  } else if (dtype == EXQ_BF16) {
    static_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(v);
  } else {
    static_cast<float*>(out)[idx] = v;
  }
}

template <typename T>
__device__ __forceinline__ void epilogue(const GemmParams& p, const ItemInfo& it, int nt_used,
                                         const int (&rows)[kGmR][2], const Acc<T>& acc) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, q = lane & 3;
#pragma unroll
  for (int rt = 0; rt < kGmR; ++rt) {
    float rs0 = 1.f, rs1 = 1.f;
    if (it.tier == EXQ_TIER_INT8) {
      if (rows[rt][0] >= 0) rs0 = __half2float(it.s[rows[rt][0]]);
      if (rows[rt][1] >= 0) rs1 = __half2float(it.s[rows[rt][1]]);
    }
#pragma unroll
    for (int nt = 0; nt < kGmNT; ++nt) {
      if (nt >= nt_used) continue;
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int tk = nt * 8 + 2 * q + cc;
        if (tk >= it.mc) continue;
        const int64_t pos = it.m0 + tk;
        const float v0 = acc.v[rt][nt][cc] * rs0;      // row g
        const float v1 = acc.v[rt][nt][2 + cc] * rs1;  // row g + 8
        if (p.mode == kGemmModeGateUp) {
          if (rows[rt][0] < 0) continue;
          const int gi = rows[rt][0];  // gate row index == mid column
          const float silu = v0 / (1.0f + expf(-v0));
          store_out(p.out, p.out_dtype, pos * p.out_stride + gi, silu * v1);
        } else if (p.mode == kGemmModeDown) {
          const float w = slot_weight(p, p.sorted_slot[pos]);
          if (rows[rt][0] >= 0)
            static_cast<float*>(p.out)[pos * p.out_stride + rows[rt][0]] = v0 * w;
          if (rows[rt][1] >= 0)
            static_cast<float*>(p.out)[pos * p.out_stride + rows[rt][1]] = v1 * w;
        } else {
          if (rows[rt][0] >= 0) store_out(p.out, p.out_dtype, pos * p.out_stride + rows[rt][0], v0);
          if (rows[rt][1] >= 0) store_out(p.out, p.out_dtype, pos * p.out_stride + rows[rt][1], v1);
        }
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kGmThreads, 3) moe_gemm_kernel(const GemmParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int n_tiles = min(*p.n_tiles_ptr, p.max_tiles);
  const int n_items = n_tiles * p.nblocks;
  if (static_cast<int>(blockIdx.x) >= n_items) return;
  const uint32_t sbase = smem_u32(smem);
  const uint64_t wpol = policy_evict_first();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2;

  LoadCtx L;
  int l_item = blockIdx.x, l_kc = 0;
  setup_load(p, l_item, n_tiles, L);
  uint32_t issued = 0, consumed = 0;

  auto issue_next = [&]() {
    while (l_item < n_items && l_kc >= L.it.nk) {  // skip empty / bad items
      l_item += gridDim.x;
      l_kc = 0;
      if (l_item < n_items) setup_load(p, l_item, n_tiles, L);
    }
    if (l_item < n_items) {
      issue_stage(p, L, l_kc, sbase + (issued % kGmS) * kStageBytes, wpol);
      ++issued;
      if (++l_kc >= L.it.nk) {
        l_item += gridDim.x;
        l_kc = 0;
        if (l_item < n_items) setup_load(p, l_item, n_tiles, L);
      }
    }
    cp_async_commit();
  };

#pragma unroll 1
  for (int s = 0; s < kGmS - 1; ++s) issue_next();

#pragma unroll 1
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    ItemInfo it;
    decode_item(p, item, n_tiles, it);
    if (it.tier < 0) continue;
    const int nt_used = (it.mc + 7) >> 3;
    int rows[kGmR][2];
#pragma unroll
    for (int rt = 0; rt < kGmR; ++rt) {
      const int lr = (warp * kGmR + rt) * 16 + g;
      rows[rt][0] = weight_row(p, it.nb, lr);
      rows[rt][1] = weight_row(p, it.nb, lr + 8);
    }
    Acc<T> acc;
#pragma unroll
    for (int rt = 0; rt < kGmR; ++rt)
#pragma unroll
      for (int nt = 0; nt < kGmNT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc.v[rt][nt][i] = 0.f;

#pragma unroll 1
    for (int kc = 0; kc < it.nk; ++kc) {
      cp_async_wait<kGmS - 2>();
      __syncthreads();
      issue_next();
      compute_stage<T>(p, it, kc, sbase + (consumed % kGmS) * kStageBytes, nt_used, rows, acc);
      ++consumed;
    }
    epilogue<T>(p, it, nt_used, rows, acc);
  }
  cp_async_wait<0>();
}

template <typename T>
int launch_gemm_t(const GemmParams& p, int max_items, cudaStream_t stream) {
  static int g_gemm_occ[64] = {0};  // per device, per instantiation
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (g_gemm_occ[dev] == 0) {
    cudaFuncSetAttribute(moe_gemm_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kGmSmem);
    int occ = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, moe_gemm_kernel<T>, kGmThreads,
                                                  kGmSmem);
    g_gemm_occ[dev] = occ > 0 ? occ : 1;
  }
  int grid = num_sms() * g_gemm_occ[dev];
  if (max_items < grid) grid = max_items;
  if (grid < 1) grid = 1;
  moe_gemm_kernel<T><<<grid, kGmThreads, kGmSmem, stream>>>(p);
  EXQ_CHECK_LAUNCH("moe_gemm_kernel");
  return EXQ_OK;
}

int launch_gemm(const GemmParams& p, int act_dtype, int max_items, cudaStream_t stream) {
  if (act_dtype == EXQ_F16) return launch_gemm_t<__half>(p, max_items, stream);
  return launch_gemm_t<__nv_bfloat16>(p, max_items, stream);
}

}  // namespace exq
