// Expert-parallel dispatch packing and return combine (one launch each).
//
// The reference runs the layer on one GPU (exq/runtime/sglang_backend.py:65-158);
// these two kernels are the per-rank ends of the expert-parallel exchange that
// exq_b200/ep.py drives over NCCL.
//
// exq_ep_pack: the T*k slots of this rank's tokens, grouped by destination
// rank (expert / experts_per_rank) in ascending slot order, become the send
// buffer: row r holds the hidden row of the slot, send_ids[r] its expert index
// local to the destination, slot_row[slot] = r, counts[d] = rows for rank d.
// Every CTA recomputes the same stable grouping (a few thousand slots) in
// shared memory and copies its chunk of rows, as route_gather.cu does.
//
// exq_ep_combine: y[t] = base[t] + sum_j w[t, j] * rows[slot_row[t*k + j]],
// fp32 sum in slot order, one rounding to the output type.
#include "internal.cuh"

namespace exq {
namespace {

constexpr int kEpThreads = 256;
constexpr int kEpWarps = kEpThreads / 32;
constexpr int kEpMaxRanks = 64;

__global__ void __launch_bounds__(kEpThreads) ep_pack_kernel(
    const void* ids, int ids_dtype, int n, int top_k, int per_rank, int n_ranks,
    const uint8_t* __restrict__ hidden, int64_t row_bytes, uint8_t* __restrict__ send_rows,
    int32_t* __restrict__ send_ids, int32_t* __restrict__ slot_row, int32_t* __restrict__ counts,
    uint32_t* status) {
  extern __shared__ int sm[];
  int* cnt = sm;                             // [warps][n_ranks] counts, then cursors
  int* base = cnt + kEpWarps * n_ranks;      // [n_ranks + 1]
  int* dst = base + n_ranks + 1;             // [n] destination of every slot (-1: dropped)
  int* row_slot = dst + n;                   // [n] slot of every send row
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < kEpWarps * n_ranks; i += kEpThreads) cnt[i] = 0;
  for (int i = threadIdx.x; i < n; i += kEpThreads) {
    const int64_t e = load_index(ids, ids_dtype, i);
    int d = -1;
    if (e >= 0 && e < static_cast<int64_t>(per_rank) * n_ranks) d = static_cast<int>(e / per_rank);
    else if (blockIdx.x == 0) atomicOr(status, EXQ_DEV_BAD_EXPERT_ID);
    dst[i] = d;
  }
  __syncthreads();
  const int per_warp = ((n + kEpWarps - 1) / kEpWarps + 31) / 32 * 32;
  const int lo = warp * per_warp, hi = min(n, lo + per_warp);
  for (int i = lo + lane; i < hi; i += 32)
    if (dst[i] >= 0) atomicAdd(&cnt[warp * n_ranks + dst[i]], 1);
  __syncthreads();
  if (threadIdx.x == 0) {  // at most 64 ranks x 8 warps: one thread scans
    int run = 0;
    for (int d = 0; d < n_ranks; ++d) {
      base[d] = run;
      for (int w = 0; w < kEpWarps; ++w) {
        const int c = cnt[w * n_ranks + d];
        cnt[w * n_ranks + d] = run;
        run += c;
      }
    }
    base[n_ranks] = run;
  }
  __syncthreads();
  // stable placement: rank of a slot among the earlier slots of its warp segment
  const unsigned lt = (1u << lane) - 1u;
  for (int b0 = lo; b0 < hi; b0 += 32) {
    const int i = b0 + lane;
    const int d = i < hi ? dst[i] : -1;
    unsigned peers = __match_any_sync(0xffffffffu, d);
    if (d >= 0) {
      const int r = cnt[warp * n_ranks + d] + __popc(peers & lt);
      row_slot[r] = i;
      if (blockIdx.x == 0) slot_row[i] = r;
    } else if (i < hi && blockIdx.x == 0) {
      slot_row[i] = -1;
    }
    __syncwarp();
    if (d >= 0 && lane == __ffs(peers) - 1) cnt[warp * n_ranks + d] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  const int total = base[n_ranks];
  if (blockIdx.x == 0) {
    for (int d = threadIdx.x; d < n_ranks; d += kEpThreads) counts[d] = base[d + 1] - base[d];
  }
  // this CTA's chunk of send rows
  const int chunk = (total + gridDim.x - 1) / gridDim.x;
  const int r0 = blockIdx.x * chunk, r1 = min(total, r0 + chunk);
  for (int r = r0 + threadIdx.x; r < r1; r += kEpThreads) {
    const int slot = row_slot[r];
    const int64_t e = load_index(ids, ids_dtype, slot);
    send_ids[r] = static_cast<int32_t>(e - static_cast<int64_t>(e / per_rank) * per_rank);
  }
  const int64_t vecs = row_bytes / 16;
  for (int64_t idx = threadIdx.x; idx < (r1 - r0) * vecs; idx += kEpThreads) {
    const int r = r0 + static_cast<int>(idx / vecs);
    const int64_t v = idx - static_cast<int64_t>(r - r0) * vecs;
    const int tok = row_slot[r] / top_k;
    reinterpret_cast<uint4*>(send_rows + static_cast<int64_t>(r) * row_bytes)[v] =
        __ldg(reinterpret_cast<const uint4*>(hidden + static_cast<int64_t>(tok) * row_bytes) + v);
  }
}

template <typename T>
__global__ void ep_combine_kernel(const T* __restrict__ rows, const int32_t* __restrict__ slot_row,
                                  const void* __restrict__ w, int w_dtype, int64_t n_tokens,
                                  int top_k, int64_t H, const T* __restrict__ base,
                                  T* __restrict__ out) {
  for (int64_t t = blockIdx.x; t < n_tokens; t += gridDim.x) {
    for (int64_t h = threadIdx.x; h < H; h += blockDim.x) {
      float acc = base ? to_f32<T>(base[t * H + h]) : 0.f;
      for (int j = 0; j < top_k; ++j) {
        const int32_t r = slot_row[t * top_k + j];
        if (r < 0) continue;
        acc = __fadd_rn(acc, __fmul_rn(load_as_f32(w, w_dtype, t * top_k + j),
                                       to_f32<T>(rows[static_cast<int64_t>(r) * H + h])));
      }
      out[t * H + h] = from_f32<T>(acc);
    }
  }
}

bool is_act(int d) { return d == EXQ_F16 || d == EXQ_BF16; }

}  // namespace
}  // namespace exq

using namespace exq;

extern "C" int exq_ep_pack(const void* topk_ids, int ids_dtype, int64_t n_tokens, int32_t top_k,
                           int32_t experts_per_rank, int32_t n_ranks, const void* hidden,
                           int dtype, int64_t hidden_size, void* send_rows, int32_t* send_ids,
                           int32_t* slot_row, int32_t* counts, void* stream) {
  EXQ_CHECK_ARG(ids_dtype == EXQ_I32 || ids_dtype == EXQ_I64, "ep_pack: ids must be int32/int64");
  EXQ_CHECK_ARG(is_act(dtype), "ep_pack: hidden must be fp16 or bf16");
  EXQ_CHECK_ARG(top_k > 0 && experts_per_rank > 0 && n_ranks > 0 && n_ranks <= kEpMaxRanks,
                "ep_pack: bad sizes (top_k %d, experts per rank %d, ranks %d; at most %d ranks)",
                top_k, experts_per_rank, n_ranks, kEpMaxRanks);
  EXQ_CHECK_ARG(n_tokens >= 0 && hidden_size > 0 && hidden_size % 8 == 0,
                "ep_pack: hidden_size must be a positive multiple of 8");
  const int64_t n = n_tokens * top_k;
  if (n > kRouteGatherMaxSlots) {
    set_error("ep_pack: %lld slots exceed %lld per call", (long long)n,
              (long long)kRouteGatherMaxSlots);
    return EXQ_ERR_UNSUPPORTED;
  }
  EXQ_CHECK_ARG(counts, "ep_pack: counts is null");
  auto s = static_cast<cudaStream_t>(stream);
  if (n == 0) {
    if (cudaMemsetAsync(counts, 0, sizeof(int32_t) * n_ranks, s) != cudaSuccess) {
      set_error("ep_pack: cudaMemsetAsync failed");
      return EXQ_ERR_CUDA;
    }
    return EXQ_OK;
  }
  EXQ_CHECK_ARG(topk_ids && hidden && send_rows && send_ids && slot_row, "ep_pack: null pointer");
  EXQ_CHECK_ARG((reinterpret_cast<uintptr_t>(hidden) | reinterpret_cast<uintptr_t>(send_rows)) % 16 == 0,
                "ep_pack: hidden and send_rows must be 16-byte aligned");
  uint32_t* st = device_status_ptr();
  if (!st) return EXQ_ERR_CUDA;
  const size_t smem = sizeof(int) * (static_cast<size_t>(kEpWarps + 1) * n_ranks + 1 + 2 * n);
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaFuncSetAttribute(ep_pack_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(sizeof(int) * ((kEpWarps + 1) * kEpMaxRanks + 1 +
                                                         2 * kRouteGatherMaxSlots)));
    attr_set[dev] = true;
  }
  int64_t grid = n;
  if (grid > 2 * num_sms()) grid = 2 * num_sms();
  ep_pack_kernel<<<static_cast<int>(grid), kEpThreads, smem, s>>>(
      topk_ids, ids_dtype, static_cast<int>(n), top_k, experts_per_rank, n_ranks,
      static_cast<const uint8_t*>(hidden), hidden_size * 2, static_cast<uint8_t*>(send_rows),
      send_ids, slot_row, counts, st);
  EXQ_CHECK_LAUNCH("ep_pack_kernel");
  return EXQ_OK;
}

extern "C" int exq_ep_combine(const void* rows, int dtype, const int32_t* slot_row,
                              const void* weights, int w_dtype, int64_t n_tokens, int32_t top_k,
                              int64_t hidden_size, const void* base, void* out, void* stream) {
  EXQ_CHECK_ARG(is_act(dtype), "ep_combine: rows must be fp16 or bf16");
  EXQ_CHECK_ARG(w_dtype == EXQ_F32 || is_act(w_dtype), "ep_combine: weights dtype unsupported");
  EXQ_CHECK_ARG(top_k > 0 && n_tokens >= 0 && hidden_size > 0, "ep_combine: bad sizes");
  if (n_tokens == 0) return EXQ_OK;
  EXQ_CHECK_ARG(slot_row && weights && out, "ep_combine: null pointer");
  auto s = static_cast<cudaStream_t>(stream);
  const int threads = static_cast<int>(hidden_size < 256 ? hidden_size : 256);
  const int grid = static_cast<int>(n_tokens < 65535 ? n_tokens : 65535);
  if (dtype == EXQ_F16)
    ep_combine_kernel<__half><<<grid, threads, 0, s>>>(
        static_cast<const __half*>(rows), slot_row, weights, w_dtype, n_tokens, top_k,
        hidden_size, static_cast<const __half*>(base), static_cast<__half*>(out));
  else
    ep_combine_kernel<__nv_bfloat16><<<grid, threads, 0, s>>>(
        static_cast<const __nv_bfloat16*>(rows), slot_row, weights, w_dtype, n_tokens, top_k,
        hidden_size, static_cast<const __nv_bfloat16*>(base), static_cast<__nv_bfloat16*>(out));
  EXQ_CHECK_LAUNCH("ep_combine_kernel");
  return EXQ_OK;
}
