// Token -> expert routing metadata: align, ends, stable sort, GEMM tile lists.
//
// One single-CTA kernel (1024 threads = 32 warps) does every variant.  The
// element range is cut into 32 contiguous warp segments.  Pass 1: each warp
// walks its segment 32 elements at a time, groups lanes with the same bucket
// with __match_any_sync and adds the group size to its own row of a
// [32 warps x n_buckets] shared-memory histogram (no atomics: a row belongs
// to one warp).  Pass 2: a column scan over warps plus a block-wide scan over
// buckets turns the table into per-(warp, bucket) write cursors and the
// bucket boundaries.  Pass 3: each warp re-walks its segment and writes every
// element at cursor + its rank inside the lane group.  Elements therefore land
// in ascending element order inside each bucket (a stable counting sort), and
// the result is deterministic, unlike the atomics of
// exq/kernels/cuda_src/exq_dispatch.cu:160-178.
#include "internal.cuh"

namespace exq {

constexpr int kRouteThreads = 1024;
constexpr int kRouteWarps = kRouteThreads / 32;
constexpr int kMaxBuckets = 1024;

// Token and slot of layer slot i = t * spt + j.  In 32 bits (launch_route
// keeps n below 2^30): a 64-bit division is a long software routine, and this
// runs for every slot on one CTA.  One slot per token (expert-parallel
// receive areas) needs no division.
__device__ __forceinline__ void split_slot(int64_t i, int spt, int64_t* t, int* j) {
  if (spt == 1) {
    *t = i;
    *j = 0;
    return;
  }
  const int ii = static_cast<int>(i);
  const int tt = ii / spt;
  *t = tt;
  *j = ii - tt * spt;
}

// Bucket and value of element i (bucket < 0: element skipped).
__device__ __forceinline__ int route_bucket(const RouteParams& p, int mode, int64_t i,
                                            int64_t* value) {
  if (mode == kRouteEndsFromSlots) {
    const int32_t slot = p.slot_ids[i];
    if (slot < 0 || slot >= p.n_active) return -1;  // padding
    *value = slot;
    const int e = p.flat_router[slot];
    if (e < 0 || e >= p.n_buckets) {
      atomicOr(p.status, EXQ_DEV_BAD_EXPERT_ID);
      return -1;
    }
    return e;
  }
  if (mode == kRouteLayer) {
    int64_t t;
    int j;
    split_slot(i, p.slots_per_token, &t, &j);
    *value = i;
    if (j >= p.top_k) return p.n_routed + (j - p.top_k);  // shared expert
    const int64_t e = load_index(p.ids, p.ids_dtype, t * p.top_k + j);
    if (e < 0) return -1;  // a padding slot: no expert
    if (e >= p.n_routed) {
      atomicOr(p.status, EXQ_DEV_BAD_EXPERT_ID);
      return -1;
    }
    return static_cast<int>(e);
  }
  const int64_t e = load_index(p.ids, p.ids_dtype, i);
  *value = i;
  if (e < 0 || e >= p.n_buckets) {
    atomicOr(p.status, EXQ_DEV_BAD_EXPERT_ID);
    return -1;
  }
  return static_cast<int>(e);
}

// Block-wide exclusive scan of v (one value per thread); returns the total.
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_tmp, int* excl) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tmp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = warp_tmp[lane];
    int s = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    warp_tmp[lane] = s - w;  // exclusive warp offsets
    if (lane == 31) warp_tmp[32] = s;
  }
  __syncthreads();
  *excl = warp_tmp[warp] + x - v;
  const int total = warp_tmp[32];
  __syncthreads();
  return total;
}

__global__ void __launch_bounds__(kRouteThreads, 1) route_kernel(RouteParams p, int mode) {
  extern __shared__ int smem[];
  int* cnt = smem;                                   // [32][n_buckets]
  int* base = cnt + kRouteWarps * p.n_buckets;       // [n_buckets] bucket start
  int* tstart = base + p.n_buckets;                  // [n_buckets] tile start (LAYER)
  int* warp_tmp = tstart + p.n_buckets;              // [33]
  const int nb = p.n_buckets;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  pdl_wait();
  pdl_trigger();

  for (int i = threadIdx.x; i < kRouteWarps * nb; i += kRouteThreads) cnt[i] = 0;
  if (mode == kRouteAlign && p.pad_sorted) {
    for (int64_t i = threadIdx.x; i < p.sorted_cap; i += kRouteThreads)
      p.sorted_i32[i] = static_cast<int32_t>(p.n);
  }
  __syncthreads();

  // warp segments (multiples of 32 elements)
  const int64_t per_warp = ((p.n + kRouteWarps - 1) / kRouteWarps + 31) / 32 * 32;
  const int64_t seg_lo = warp * per_warp;
  const int64_t seg_hi = min(p.n, seg_lo + per_warp);

  // pass 1: per-warp histogram rows
  for (int64_t b0 = seg_lo; b0 < seg_hi; b0 += 32) {
    const int64_t i = b0 + lane;
    int64_t val = 0;
    const int e = (i < seg_hi) ? route_bucket(p, mode, i, &val) : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    if (e >= 0 && lane == __ffs(peers) - 1) cnt[warp * nb + e] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();

  // pass 2a: column scan over warps -> per-warp offsets inside a bucket
  // pass 2b: block scan over buckets (padded for ALIGN) -> bucket bases
  int carry = 0, tile_carry = 0;
  for (int c0 = 0; c0 < nb; c0 += kRouteThreads) {
    const int e = c0 + threadIdx.x;
    int total = 0;
    if (e < nb) {
      for (int w = 0; w < kRouteWarps; ++w) {
        const int v = cnt[w * nb + e];
        cnt[w * nb + e] = total;
        total += v;
      }
    }
    int span = total;
    if (mode == kRouteAlign) span = (total + p.block_size - 1) / p.block_size * p.block_size;
    int excl;
    const int sum = block_exclusive_scan(span, warp_tmp, &excl);
    int tiles = 0;
    if (mode == kRouteLayer) tiles = (total + p.mt - 1) / p.mt;
    int texcl;
    const int tsum = block_exclusive_scan(tiles, warp_tmp, &texcl);
    if (e < nb) {
      base[e] = carry + excl;
      tstart[e] = tile_carry + texcl;
    }
    carry += sum;
    tile_carry += tsum;
    __syncthreads();
  }
  // bucket counts are base[e+1]-base[e] for non-ALIGN modes; for ALIGN keep
  // the padded prefix.
  if (threadIdx.x == 0) {
    if (mode == kRouteAlign) {
      p.ntpp[0] = carry;
      p.cumsum[nb] = carry;
    } else if (p.ends) {
      p.ends[nb] = carry;
    }
    if (mode == kRouteLayer) p.n_tiles[0] = tile_carry;
  }
  for (int e = threadIdx.x; e < nb; e += kRouteThreads) {
    if (mode == kRouteAlign) {
      p.cumsum[e] = base[e];
    } else if (p.ends) {
      p.ends[e] = base[e];
    }
  }
  __syncthreads();

  if (mode == kRouteAlign) {
    // expert_ids: owner of every block, -1 past the padded total
    const int64_t used_blocks = carry / p.block_size;
    for (int64_t b = threadIdx.x; b < p.block_cap; b += kRouteThreads) {
      int owner = -1;
      if (b < used_blocks) {
        const int pos = static_cast<int>(b * p.block_size);
        int lo = 0, hi = nb - 1;  // last e with base[e] <= pos
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (base[mid] <= pos) lo = mid; else hi = mid - 1;
        }
        owner = lo;
      }
      p.block_expert[b] = owner;
    }
  }
  if (mode == kRouteLayer) {
    // the GEMM's tile and work counters start at zero
    for (int64_t i = threadIdx.x; i < p.n_counters; i += kRouteThreads) p.counters[i] = 0;
    // positions past the routed total (slots dropped for a bad expert id) hold -1
    for (int64_t i = carry + threadIdx.x; i < p.n; i += kRouteThreads) {
      p.sorted_i32[i] = -1;
      if (p.order_i64) p.order_i64[i] = -1;
    }
    // tile list: (expert, first sorted row, rows) ; counts from the next base
    for (int e = threadIdx.x; e < nb; e += kRouteThreads) {
      const int c = ((e + 1 < nb) ? base[e + 1] : carry) - base[e];
      const int t0 = tstart[e];
      for (int t = 0; t * p.mt < c; ++t) {
        const int64_t ti = t0 + t;
        if (ti < p.max_tiles) {
          p.tile_info[ti * 3 + 0] = e;
          p.tile_info[ti * 3 + 1] = base[e] + t * p.mt;
          p.tile_info[ti * 3 + 2] = min(p.mt, c - t * p.mt);
        }
      }
    }
  }

  // pass 3: stable placement
  for (int e = threadIdx.x; e < nb; e += kRouteThreads) {
    for (int w = 0; w < kRouteWarps; ++w) cnt[w * nb + e] += base[e];
  }
  __syncthreads();
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int64_t b0 = seg_lo; b0 < seg_hi; b0 += 32) {
    const int64_t i = b0 + lane;
    int64_t val = 0;
    const int e = (i < seg_hi) ? route_bucket(p, mode, i, &val) : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    int pos = 0;
    if (e >= 0) pos = cnt[warp * nb + e] + __popc(peers & lt_mask);
    __syncwarp();
    if (e >= 0) {
      if (lane == __ffs(peers) - 1) cnt[warp * nb + e] += __popc(peers);
      switch (mode) {
        case kRouteAlign:
          if (pos < p.sorted_cap) p.sorted_i32[pos] = static_cast<int32_t>(val);
          break;
        case kRouteEndsFromSlots:
          // duplicated slot ids (invalid input) could overflow sort_order
          if (pos < p.n_active) p.order_i64[pos] = val;
          else atomicOr(p.status, EXQ_DEV_BAD_SLOT);
          break;
        case kRouteDispatch:
          p.order_i64[pos] = val;
          p.sorted_expert_i64[pos] = e;
          break;
        default:
          p.sorted_i32[pos] = static_cast<int32_t>(val);
          if (p.pos_of_slot) p.pos_of_slot[val] = pos;
          if (p.sorted_w) {
            int64_t t;
            int j;
            split_slot(val, p.slots_per_token, &t, &j);
            p.sorted_w[pos] =
                j < p.top_k ? load_as_f32(p.topk_w, p.w_dtype, t * p.top_k + j) : 1.0f;
          }
          if (p.order_i64) p.order_i64[pos] = val;
          break;
      }
    } else if (mode == kRouteLayer && i < seg_hi && p.pos_of_slot) {
      p.pos_of_slot[i] = -1;  // dropped (expert id out of range)
    }
    __syncwarp();
  }
}

size_t route_smem_bytes(int n_buckets) {
  return sizeof(int) * (static_cast<size_t>(kRouteWarps) * n_buckets + 2 * n_buckets + 33);
}

int launch_route(RouteParams& p, int mode, cudaStream_t stream, bool pdl) {
  if (p.n_buckets < 1 || p.n_buckets > kMaxBuckets) {
    set_error("route: number of experts %d outside [1, %d]", p.n_buckets, kMaxBuckets);
    return EXQ_ERR_UNSUPPORTED;
  }
  if (p.n > INT32_MAX / 2) {
    set_error("route: %lld elements exceeds the int32 index range", (long long)p.n);
    return EXQ_ERR_UNSUPPORTED;
  }
  p.status = device_status_ptr();
  if (!p.status) return EXQ_ERR_CUDA;
  const size_t smem = route_smem_bytes(p.n_buckets);
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaFuncSetAttribute(route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         route_smem_bytes(kMaxBuckets));
    attr_set[dev] = true;
  }
  if (pdl) {
    const cudaError_t e =
        launch_pdl(true, route_kernel, dim3(1), dim3(kRouteThreads), smem, stream, p, mode);
    if (e != cudaSuccess) {
      set_error("route_kernel: %s", cudaGetErrorString(e));
      return EXQ_ERR_CUDA;
    }
  } else {
    route_kernel<<<1, kRouteThreads, smem, stream>>>(p, mode);
  }
  EXQ_CHECK_LAUNCH("route_kernel");
  return EXQ_OK;
}

}  // namespace exq

using namespace exq;

extern "C" int exq_moe_align_block_size(const void* topk_ids, int ids_dtype, int64_t numel,
                                        int32_t num_experts, int32_t block_size,
                                        int32_t* sorted_token_ids, int64_t sorted_cap,
                                        int32_t* expert_ids, int64_t expert_ids_cap,
                                        int32_t* num_tokens_post_pad, int32_t* cumsum_buffer,
                                        int32_t pad_sorted_token_ids, void* stream) {
  EXQ_CHECK_ARG(ids_dtype == EXQ_I32 || ids_dtype == EXQ_I64, "topk_ids must be int32/int64");
  EXQ_CHECK_ARG(numel >= 0, "numel < 0");
  EXQ_CHECK_ARG(block_size > 0, "block_size must be positive");
  EXQ_CHECK_ARG(numel == 0 || topk_ids, "topk_ids is null");
  EXQ_CHECK_ARG(sorted_token_ids && expert_ids && num_tokens_post_pad && cumsum_buffer,
                "null output pointer");
  const int64_t max_padded = numel + static_cast<int64_t>(num_experts) * (block_size - 1);
  EXQ_CHECK_ARG(sorted_cap >= max_padded,
                "sorted_token_ids has %lld entries, needs numel + num_experts*(block_size-1)"
                " = %lld",
                (long long)sorted_cap, (long long)max_padded);
  EXQ_CHECK_ARG(expert_ids_cap * block_size >= max_padded,
                "expert_ids has %lld entries, needs ceil(%lld / %d)", (long long)expert_ids_cap,
                (long long)max_padded, block_size);
  RouteParams p{};
  p.ids = topk_ids;
  p.ids_dtype = ids_dtype;
  p.n = numel;
  p.n_buckets = num_experts;
  p.block_size = block_size;
  p.sorted_i32 = sorted_token_ids;
  p.sorted_cap = sorted_cap;
  p.pad_sorted = pad_sorted_token_ids;
  p.block_expert = expert_ids;
  p.block_cap = expert_ids_cap;
  p.ntpp = num_tokens_post_pad;
  p.cumsum = cumsum_buffer;
  return launch_route(p, kRouteAlign, static_cast<cudaStream_t>(stream));
}

extern "C" int exq_build_ends_from_slots(const int32_t* sorted_slot_ids, int64_t em,
                                         const int32_t* flat_router, int64_t n_active,
                                         int32_t n_experts, int32_t* expert_ends,
                                         int64_t* sort_order, void* stream) {
  EXQ_CHECK_ARG(em >= 0 && n_active >= 0, "negative size");
  EXQ_CHECK_ARG(em == 0 || sorted_slot_ids, "sorted_slot_ids is null");
  EXQ_CHECK_ARG(n_active == 0 || (flat_router && sort_order), "null flat_router/sort_order");
  EXQ_CHECK_ARG(expert_ends, "expert_ends is null");
  RouteParams p{};
  p.slot_ids = sorted_slot_ids;
  p.flat_router = flat_router;
  p.n = em;
  p.n_active = n_active;
  p.n_buckets = n_experts;
  p.ends = expert_ends;
  p.order_i64 = sort_order;
  return launch_route(p, kRouteEndsFromSlots, static_cast<cudaStream_t>(stream));
}

extern "C" int exq_dispatch(const void* router_indices, int ids_dtype, int64_t n,
                            int32_t n_experts, int64_t* sort_order, int64_t* sorted_expert_ids,
                            int32_t* expert_ends, void* stream) {
  EXQ_CHECK_ARG(ids_dtype == EXQ_I32 || ids_dtype == EXQ_I64,
                "router_indices must be int32/int64");
  EXQ_CHECK_ARG(n >= 0, "n < 0");
  EXQ_CHECK_ARG(n == 0 || (router_indices && sort_order && sorted_expert_ids),
                "null pointer");
  EXQ_CHECK_ARG(expert_ends, "expert_ends is null");
  RouteParams p{};
  p.ids = router_indices;
  p.ids_dtype = ids_dtype;
  p.n = n;
  p.n_buckets = n_experts;
  p.ends = expert_ends;
  p.order_i64 = sort_order;
  p.sorted_expert_i64 = sorted_expert_ids;
  return launch_route(p, kRouteDispatch, static_cast<cudaStream_t>(stream));
}
