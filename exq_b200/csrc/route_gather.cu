// Layer routing fused with the activation gather (decode-sized inputs).
//
// Replaces, for one MoE layer call, the sort/align step and the gather of
// exq/runtime/sglang_backend.py:102-131 (moe_align_block_size, then the
// hidden-state gather the Triton GEMM performs through sorted_token_ids).
//
// Every CTA reads all T*(top_k+shared) slots' expert ids (a few thousand, from
// L2) and computes the same bucket counts and bucket bases in shared memory,
// so all CTAs agree on the stable counting sort without a grid-wide barrier.
// The slots are split into contiguous chunks, one per CTA; a CTA places only
// its own chunk (position = bucket base + the bucket's slots before the chunk
// + the slot's rank among the chunk's slots of its bucket, by match_any on one
// warp) and, slot by slot,
//   - copies the hidden-state row into the fp16 activation buffer at the
//     slot's sorted position, converting bf16 and permuting every octet of k
//     to [0,4,1,5,2,6,3,7] (the k order of the dequantised weights),
//   - writes the slot -> position map and the router weight at the position.
// CTA 0 also writes the GEMM tile list and the expert ends; dropped slots
// (expert id out of range or negative) map to -1, and the positions past the
// routed total that the last GEMM tile reads get zero rows.
#include <type_traits>

#include "internal.cuh"

namespace exq {

constexpr int kRgThreads = 256;
constexpr int kRgWarps = kRgThreads / 32;

size_t route_gather_smem_bytes(int n_buckets, int64_t n) {
  return sizeof(int) * (static_cast<size_t>(4) * n_buckets + 34 + 2 * n);
}

namespace {

// (token, slot in token) of slot i; one slot per token (expert-parallel
// receive areas) needs no division
__device__ __forceinline__ void rg_split(int i, int spt, int* t, int* j) {
  if (spt == 1) {
    *t = i;
    *j = 0;
  } else {
    *t = i / spt;
    *j = i - *t * spt;
  }
}

__device__ __forceinline__ int rg_exclusive_scan(int v, int* tmp, int* excl) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) tmp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    const int w = lane < kRgWarps ? tmp[lane] : 0;
    int s = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < kRgWarps) tmp[lane] = s - w;
    if (lane == 31) tmp[32] = s;
  }
  __syncthreads();
  *excl = tmp[warp] + x - v;
  const int total = tmp[32];
  __syncthreads();
  return total;
}

// fp16 or bf16 octet -> fp16 octet in [0,4,1,5,2,6,3,7] order
template <typename T>
__device__ __forceinline__ uint4 permute_octet(uint4 v) {
  uint32_t w[4] = {v.x, v.y, v.z, v.w};
  if (!std::is_same<T, __half>::value) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&w[j]));
      __half2 h = __floats2half2_rn(f.x, f.y);
      w[j] = *reinterpret_cast<uint32_t*>(&h);
    }
  }
  uint4 r;
  r.x = prmt(w[0], w[2], 0x5410u);  // (k0, k4)
  r.y = prmt(w[0], w[2], 0x7632u);  // (k1, k5)
  r.z = prmt(w[1], w[3], 0x5410u);  // (k2, k6)
  r.w = prmt(w[1], w[3], 0x7632u);  // (k3, k7)
  return r;
}

template <typename T>
__global__ void __launch_bounds__(kRgThreads) route_gather_kernel(const RouteGatherParams p) {
  extern __shared__ int smem[];
  const int nb = p.n_buckets;
  const int n = static_cast<int>(p.n);
  int* cnt_all = smem;               // [nb] slots of every bucket
  int* cnt_pre = cnt_all + nb;       // [nb] of them before this CTA's chunk, then cursors
  int* base = cnt_pre + nb;          // [nb] first sorted position of every bucket
  int* tstart = base + nb;           // [nb] first tile of every bucket
  int* tmp = tstart + nb;            // [33] scan scratch, [33] routed total
  int* bkt = tmp + 34;               // [n] bucket of every slot (-1: dropped)
  int* slot_pos = bkt + n;           // [chunk] sorted position of this CTA's slots (-1: dropped)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

  pdl_wait();
  pdl_trigger();

  for (int i = threadIdx.x; i < 2 * nb; i += kRgThreads) cnt_all[i] = 0;
  // bucket of every slot; the id loads of 8 slots are issued before any is used
  for (int i0 = threadIdx.x; i0 < n; i0 += 8 * kRgThreads) {
    int64_t v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * kRgThreads;
      int t, j;
      rg_split(i, p.spt, &t, &j);
      const bool routed = i < n && j < p.top_k;
      const int64_t src = routed ? static_cast<int64_t>(t) * p.top_k + j : 0;
      v[u] = load_index(p.ids, p.ids_dtype, src);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * kRgThreads;
      if (i >= n) break;
      int t, j;
      rg_split(i, p.spt, &t, &j);
      int e;
      if (j >= p.top_k) {
        e = p.n_routed + (j - p.top_k);  // always-on shared expert
      } else {
        // negative: a padding slot (no expert); past the experts: dropped and flagged
        e = (v[u] >= 0 && v[u] < p.n_routed) ? static_cast<int>(v[u]) : -1;
        if (v[u] >= p.n_routed && blockIdx.x == 0) atomicOr(p.status, EXQ_DEV_BAD_EXPERT_ID);
      }
      bkt[i] = e;
    }
  }
  __syncthreads();

  // This CTA's slots [s0, s1).  A slot's sorted position is the first
  // position of its bucket, plus the slots of the same bucket before s0, plus
  // its rank among this chunk's slots of that bucket (a stable counting sort,
  // with only the chunk's own slots placed here).
  const int chunk = (n + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x);
  const int s0 = min(n, static_cast<int>(blockIdx.x) * chunk), s1 = min(n, s0 + chunk);

  // pass 1: bucket counts of all slots and of the slots before s0 (order-free).
  // With few buckets (large calls of a few experts) the lanes of a warp that
  // hold one bucket add their count once, instead of all contending for it.
  if (nb <= 32) {
    for (int i0 = 0; i0 < n; i0 += kRgThreads) {
      const int i = i0 + threadIdx.x;
      const int e = i < n ? bkt[i] : -1;
      const unsigned same = __match_any_sync(0xffffffffu, e);
      const unsigned pre = same & __ballot_sync(0xffffffffu, i < s0);
      if (e >= 0 && lane == __ffs(same) - 1) {
        atomicAdd(&cnt_all[e], __popc(same));
        if (pre) atomicAdd(&cnt_pre[e], __popc(pre));
      }
    }
  } else {
    for (int i = threadIdx.x; i < n; i += kRgThreads) {
      const int e = bkt[i];
      if (e >= 0) {
        atomicAdd(&cnt_all[e], 1);
        if (i < s0) atomicAdd(&cnt_pre[e], 1);
      }
    }
  }
  __syncthreads();

  // pass 2: bucket bases and tile starts (one scan of (tiles << 16 | rows):
  // both stay below 2^16, n <= 16384)
  int carry = 0, tile_carry = 0;
  for (int c0 = 0; c0 < nb; c0 += kRgThreads) {
    const int e = c0 + threadIdx.x;
    const int total = e < nb ? cnt_all[e] : 0;
    int packed_excl;
    const int packed = rg_exclusive_scan(((total + p.mt - 1) / p.mt) << 16 | total, tmp, &packed_excl);
    const int sum = packed & 0xFFFF, tsum = packed >> 16;
    const int excl = packed_excl & 0xFFFF, texcl = packed_excl >> 16;
    if (e < nb) {
      base[e] = carry + excl;
      tstart[e] = tile_carry + texcl;
    }
    carry += sum;
    tile_carry += tsum;
  }
  __syncthreads();

  // pass 3: the chunk's slots in order, 32 at a time, on warp 0
  if (warp == 0) {
    const unsigned lt_mask = (1u << lane) - 1u;
    for (int b0 = s0; b0 < s1; b0 += 32) {
      const int i = b0 + lane;
      const int e = i < s1 ? bkt[i] : -1;
      const unsigned peers = __match_any_sync(0xffffffffu, e);
      if (e >= 0) slot_pos[i - s0] = base[e] + cnt_pre[e] + __popc(peers & lt_mask);
      else if (i < s1) slot_pos[i - s0] = -1;
      __syncwarp();
      if (e >= 0 && lane == __ffs(peers) - 1) cnt_pre[e] += __popc(peers);
      __syncwarp();
    }
  }
  __syncthreads();

  if (blockIdx.x == 0) {
    for (int e = threadIdx.x; e < nb; e += kRgThreads) {
      const int c = cnt_all[e];
      if (p.ends) p.ends[e] = base[e];
      for (int t = 0; t * p.mt < c; ++t) {
        const int64_t ti = tstart[e] + t;
        if (ti < p.max_tiles) {
          p.tile_info[ti * 3 + 0] = e;
          p.tile_info[ti * 3 + 1] = base[e] + t * p.mt;
          p.tile_info[ti * 3 + 2] = min(p.mt, c - t * p.mt);
        }
      }
    }
    if (threadIdx.x == 0) {
      if (p.ends) p.ends[nb] = carry;
      p.n_tiles[0] = tile_carry;
    }
  }
  for (int i = s0 + threadIdx.x; i < s1; i += kRgThreads) {
    const int pos = slot_pos[i - s0];
    p.pos_of_slot[i] = pos;
    if (pos >= 0) {
      // the router weight of this CTA's slots only; shared experts weigh 1
      int t, j;
      rg_split(i, p.spt, &t, &j);
      p.sorted_w[pos] =
          j < p.top_k ? load_as_f32(p.topk_w, p.w_dtype, static_cast<int64_t>(t) * p.top_k + j)
                      : 1.0f;
      if (p.sorted_slot) p.sorted_slot[pos] = i;
    }
  }
  // the GEMM's tile and work counters start at zero
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kRgThreads + threadIdx.x; i < p.n_counters;
       i += static_cast<int64_t>(gridDim.x) * kRgThreads)
    p.counters[i] = 0;
  // row copies: threads take the 16-byte chunks of a row, kU rows at a time
  // (a thread's loads of the kU rows are in flight together); a dropped slot
  // has no row
  const int octs = static_cast<int>(p.hidden_size / 8);
  const T* hid = static_cast<const T*>(p.hidden);
  uint4* act = reinterpret_cast<uint4*>(p.act);
  constexpr int kU = 8;
  for (int r0 = 0; r0 < s1 - s0; r0 += kU) {
    const uint4* src[kU];
    int pos[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int r = r0 + u;
      pos[u] = r < s1 - s0 ? slot_pos[r] : -1;
      int t = 0, j = 0;
      if (pos[u] >= 0) rg_split(s0 + r, p.spt, &t, &j);
      src[u] = reinterpret_cast<const uint4*>(hid + static_cast<int64_t>(t) * p.hidden_size);
    }
    for (int o = threadIdx.x; o < octs; o += kRgThreads) {
      uint4 v[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) v[u] = pos[u] >= 0 ? __ldg(src[u] + o) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        // act is stage-major [H/64][n][64]
        if (pos[u] >= 0)
          act[(static_cast<int64_t>(o >> 3) * n + pos[u]) * 8 + (o & 7)] = permute_octet<T>(v[u]);
      }
    }
  }
  // positions past the routed total that the last GEMM tile reads (a tile
  // starts below the total and spans mt rows): zero rows
  const int zend = min(n, carry + p.mt);
  const int zc = (zend - carry + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x);
  const int z0 = carry + static_cast<int>(blockIdx.x) * zc, z1 = min(zend, z0 + zc);
  for (int idx = threadIdx.x; idx < max(0, z1 - z0) * octs; idx += kRgThreads) {
    const int pos = z0 + idx / octs, o = idx % octs;
    reinterpret_cast<uint4*>(p.act)[(static_cast<int64_t>(o >> 3) * n + pos) * 8 + (o & 7)] =
        make_uint4(0, 0, 0, 0);
  }
}

}  // namespace

int launch_route_gather(RouteGatherParams& p, cudaStream_t stream, bool pdl) {
  if (p.n_buckets < 1 || p.n_buckets > kRouteGatherMaxBuckets || p.n > kRouteGatherFusedMaxSlots) {
    set_error("route_gather: %d buckets / %lld slots outside the fused path", p.n_buckets,
              (long long)p.n);
    return EXQ_ERR_UNSUPPORTED;
  }
  if (p.n == 0) return EXQ_OK;
  p.status = device_status_ptr();
  if (!p.status) return EXQ_ERR_CUDA;
  const size_t smem = route_gather_smem_bytes(p.n_buckets, p.n);
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    const size_t mx = route_gather_smem_bytes(kRouteGatherMaxBuckets, kRouteGatherFusedMaxSlots);
    cudaFuncSetAttribute(route_gather_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(mx));
    cudaFuncSetAttribute(route_gather_kernel<__nv_bfloat16>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(mx));
    attr_set[dev] = true;
  }
  // at least one sorted position per CTA; two CTAs per SM while two fit in
  // shared memory, else one (no CTA waits for another, so more would only queue)
  int64_t grid = p.n;
  const int64_t cap = (smem > 110 * 1024 ? 1 : 2) * static_cast<int64_t>(num_sms());
  if (grid > cap) grid = cap;
  cudaError_t e;
  if (p.act_dtype == EXQ_F16)
    e = launch_pdl(pdl, route_gather_kernel<__half>, dim3(static_cast<int>(grid)),
                   dim3(kRgThreads), smem, stream, p);
  else
    e = launch_pdl(pdl, route_gather_kernel<__nv_bfloat16>, dim3(static_cast<int>(grid)),
                   dim3(kRgThreads), smem, stream, p);
  if (e != cudaSuccess) {
    set_error("route_gather_kernel: %s", cudaGetErrorString(e));
    return EXQ_ERR_CUDA;
  }
  EXQ_CHECK_LAUNCH("route_gather_kernel");
  return EXQ_OK;
}

}  // namespace exq
