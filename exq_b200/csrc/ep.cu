// Expert-parallel exchange: packing, the peer-memory exchange and the return
// combine.
//
// The reference runs the layer on one GPU (exq/runtime/sglang_backend.py:65-158);
// these kernels are the per-rank ends of the expert-parallel exchange that
// exq_b200/ep.py drives.
//
// exq_ep_pack (NCCL exchange): the T*k slots of this rank's tokens, grouped by
// destination rank (expert / experts_per_rank) in ascending slot order, become
// the send buffer: row r holds the hidden row of the slot, send_ids[r] its
// expert index local to the destination, slot_row[slot] = r, counts[d] = rows
// for rank d.  Every CTA recomputes the same stable grouping (a few thousand
// slots) in shared memory and copies its chunk of rows, as route_gather.cu does.
//
// exq_ep_combine: y[t] = base[t] + sum_j w[t, j] * rows[slot_row[t*k + j]],
// fp32 sum in slot order, one rounding to the output type.
//
// Peer-memory exchange (no NCCL, no host sync).  Every rank owns one buffer,
// mapped into the other ranks of the node through CUDA IPC:
//   header  u32 flags: [0, 64) arrival flag of each source rank, [64, 128)
//           return flag of each expert rank, [128] this rank's step counter,
//           [129] / [130] grid tickets of the dispatch / return kernels
//   ids     int32 [P * cap]   local expert id of each received row (-1: none)
//   ones    f32   [P * cap]   1.0f, the router weight of a received row
//   recv    act   [P * cap, H] received hidden rows
//   back    act   [P * cap, H] expert outputs returned to this rank
// Block s (rows [s*cap, (s+1)*cap)) of ids/recv is written by source rank s,
// block d of back by expert rank d.  A flag holds the step counter of the
// last step whose data it covers, so nothing is ever reset between steps.
//   exq_ep_dispatch: the grouping above, with each row and id stored straight
//     into the destination's block (NVLink stores); the last CTA to finish
//     (grid ticket) fences, raises this rank's arrival flag in every
//     destination with a system-scope release store, and bumps the counter.
//   exq_ep_expert_forward: one thread per source waits (acquire, bounded) for
//     the arrival flags; the layer's route, gate_up and down stages run on the
//     P*cap received rows (unused rows have id -1 and no GEMM tile); a return
//     kernel rounds each real row's fp32 output and stores it into its source's
//     back block, then raises the return flags the same way.
//   exq_ep_combine_peer: every CTA waits for the return flags, then combines
//     as exq_ep_combine from the back area (loads bypass L1).
// A step on one rank cannot overwrite data a peer still reads: a rank reaches
// its next dispatch only after its combine saw every peer's return flag, which
// each peer raised after its expert stages finished reading their recv area;
// a peer writes this rank's back area only after this rank's next arrival flag.
#include "internal.cuh"

namespace exq {
namespace {

constexpr int kEpThreads = 256;
constexpr int kEpWarps = kEpThreads / 32;
constexpr int kEpMaxRanks = 64;

// header words (u32 index)
constexpr int kEpFlagArrive = 0;
constexpr int kEpFlagReturn = 64;
constexpr int kEpStep = 128;
constexpr int kEpTicketDispatch = 129;
constexpr int kEpTicketReturn = 130;
constexpr int kEpFailed = 131;  // nonzero once a wait of this rank's kernels ran out
constexpr int64_t kEpHeaderBytes = 1024;
// a wait on another rank gives up after this long (exq_ep_set_wait_timeout)
constexpr unsigned long long kEpWaitNsDefault = 5000000000ull;
unsigned long long g_ep_wait_ns = kEpWaitNsDefault;

struct EpLayout {
  int64_t ids, ones, recv, back, bytes;
};

// Receive side: n_ranks + 1 blocks of cap rows (ids, weights 1.0, rows):
// block s holds what source rank s sent, block n_ranks this rank's own tokens
// for its shared experts (exq_ep_expert_forward_shared).  Return side:
// n_ranks blocks, block d written by expert rank d.
__host__ __device__ inline EpLayout ep_layout(int n_ranks, int64_t cap, int64_t row_bytes) {
  const int64_t rows_in = static_cast<int64_t>(n_ranks + 1) * cap;
  const int64_t rows = static_cast<int64_t>(n_ranks) * cap;
  auto up = [](int64_t x) { return (x + 255) / 256 * 256; };
  EpLayout l;
  l.ids = kEpHeaderBytes;
  l.ones = l.ids + up(4 * rows_in);
  l.recv = l.ones + up(4 * rows_in);
  l.back = l.recv + up(rows_in * row_bytes);
  l.bytes = l.back + up(rows * row_bytes);
  return l;
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
  return t;
}

// Waits until *flag has reached `step` (wrap-safe).  Bounded by time
// (wait_ns) and by iterations; on expiry sets EXQ_DEV_TIMEOUT, marks the
// rank's buffer as failed (hdr[kEpFailed]) and returns false.  After that the
// exchange is out of step: the kernels of this rank stop reading and writing
// peer data, the peers' own waits run out in turn, and every rank must
// re-initialise its buffer (exq_ep_buffer_init) before the next step.
__device__ bool ep_wait_flag(const uint32_t* flag, uint32_t step, uint32_t* status,
                             uint32_t* hdr, unsigned long long wait_ns) {
  const unsigned long long t0 = global_ns();
  for (uint32_t it = 0; static_cast<int32_t>(ld_acquire_sys(flag) - step) < 0; ++it) {
    if (it > (1u << 27) || global_ns() - t0 > wait_ns) {
      atomicOr(status, EXQ_DEV_TIMEOUT);
      atomicExch(hdr + kEpFailed, 1u);
      return false;
    }
    __nanosleep(100);
  }
  return true;
}

// The last CTA of the grid to get here (all others have fenced their stores)
// returns true in every thread; the ticket is reset for the next launch.
__device__ bool ep_last_cta(uint32_t* ticket) {
  __shared__ bool last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    last = atomicAdd(ticket, 1u) == gridDim.x - 1;
    if (last) {
      *ticket = 0;
      __threadfence_system();
    }
  }
  __syncthreads();
  return last;
}

struct EpPackArgs {
  const void* ids;
  int ids_dtype, n, top_k, per_rank, n_ranks;
  const uint8_t* hidden;
  int64_t row_bytes;
  // NCCL exchange: packed send buffer
  uint8_t* send_rows;
  int32_t* send_ids;
  int32_t* counts;
  // peer exchange: buffer of every rank
  uint8_t* const* peers;
  int rank, cap;
  EpLayout lay;
  int32_t* slot_row;
  uint32_t* status;
};

template <bool kPeer>
__global__ void __launch_bounds__(kEpThreads) ep_pack_kernel(EpPackArgs a) {
  extern __shared__ int sm[];
  __shared__ uint8_t* peer[kEpMaxRanks];
  const int n = a.n, n_ranks = a.n_ranks, cap = a.cap;
  int* cnt = sm;                             // [warps][n_ranks] counts, then cursors
  int* base = cnt + kEpWarps * n_ranks;      // [n_ranks + 1]
  int* dst = base + n_ranks + 1;             // [n] destination of every slot (-1: dropped)
  int* row_slot = dst + n;                   // [n] slot of every grouped row
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (kPeer)
    for (int d = threadIdx.x; d < n_ranks; d += kEpThreads) peer[d] = a.peers[d];
  for (int i = threadIdx.x; i < kEpWarps * n_ranks; i += kEpThreads) cnt[i] = 0;
  for (int i = threadIdx.x; i < n; i += kEpThreads) {
    const int64_t e = load_index(a.ids, a.ids_dtype, i);
    int d = -1;
    if (e >= 0 && e < static_cast<int64_t>(a.per_rank) * n_ranks) d = static_cast<int>(e / a.per_rank);
    else if (blockIdx.x == 0) atomicOr(a.status, EXQ_DEV_BAD_EXPERT_ID);
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
      if (blockIdx.x == 0) {
        int sr = r;
        if (kPeer) {  // row of this rank's back area that rank d fills
          const int q = r - base[d];
          sr = q < cap ? d * cap + q : -1;
          if (q >= cap) atomicOr(a.status, EXQ_DEV_BAD_SLOT);
        }
        a.slot_row[i] = sr;
      }
    } else if (i < hi && blockIdx.x == 0) {
      a.slot_row[i] = -1;
    }
    __syncwarp();
    if (d >= 0 && lane == __ffs(peers) - 1) cnt[warp * n_ranks + d] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  const int total = base[n_ranks];
  if (!kPeer && blockIdx.x == 0)
    for (int d = threadIdx.x; d < n_ranks; d += kEpThreads) a.counts[d] = base[d + 1] - base[d];
  // where grouped row r goes: the packed send row, or row `rank*cap + q` of
  // destination d's receive block (nullptr past the capacity)
  auto ids_of = [&](int r, int d) -> int32_t* {
    if (!kPeer) return a.send_ids + r;
    const int q = r - base[d];
    return q < cap ? reinterpret_cast<int32_t*>(peer[d] + a.lay.ids) + (a.rank * cap + q) : nullptr;
  };
  auto row_of = [&](int r, int d) -> uint8_t* {
    if (!kPeer) return a.send_rows + static_cast<int64_t>(r) * a.row_bytes;
    const int q = r - base[d];
    return q < cap ? peer[d] + a.lay.recv + static_cast<int64_t>(a.rank * cap + q) * a.row_bytes
                   : nullptr;
  };
  // this CTA's chunk of grouped rows
  const int chunk = (total + gridDim.x - 1) / gridDim.x;
  const int r0 = blockIdx.x * chunk, r1 = min(total, r0 + chunk);
  for (int r = r0 + threadIdx.x; r < r1; r += kEpThreads) {
    const int slot = row_slot[r];
    if (slot < 0 || slot >= n) {  // cannot happen: every grouped row has a slot
      atomicOr(a.status, EXQ_DEV_BAD_SLOT);
      continue;
    }
    const int d = dst[slot];
    const int64_t e = load_index(a.ids, a.ids_dtype, slot);
    int32_t* p = ids_of(r, d);
    if (p) *p = static_cast<int32_t>(e - static_cast<int64_t>(d) * a.per_rank);
  }
  const int64_t vecs = a.row_bytes / 16;
  for (int64_t idx = threadIdx.x; idx < (r1 - r0) * vecs; idx += kEpThreads) {
    const int r = r0 + static_cast<int>(idx / vecs);
    const int64_t v = idx - static_cast<int64_t>(r - r0) * vecs;
    const int slot = row_slot[r];
    if (slot < 0 || slot >= n) continue;  // flagged above
    uint8_t* p = row_of(r, dst[slot]);
    if (!p) continue;
    const int tok = slot / a.top_k;
    reinterpret_cast<uint4*>(p)[v] =
        __ldg(reinterpret_cast<const uint4*>(a.hidden + static_cast<int64_t>(tok) * a.row_bytes) + v);
  }
  if (kPeer) {
    // the unused ids of this rank's block in every destination
    const int64_t fill = static_cast<int64_t>(n_ranks) * cap;
    for (int64_t idx = static_cast<int64_t>(blockIdx.x) * kEpThreads + threadIdx.x; idx < fill;
         idx += static_cast<int64_t>(gridDim.x) * kEpThreads) {
      const int d = static_cast<int>(idx / cap), q = static_cast<int>(idx - static_cast<int64_t>(d) * cap);
      if (q >= base[d + 1] - base[d])
        reinterpret_cast<int32_t*>(peer[d] + a.lay.ids)[a.rank * cap + q] = -1;
    }
    uint32_t* own = reinterpret_cast<uint32_t*>(peer[a.rank]);
    if (ep_last_cta(own + kEpTicketDispatch) && threadIdx.x == 0) {
      const uint32_t step = *reinterpret_cast<volatile uint32_t*>(own + kEpStep) + 1u;
      for (int d = 0; d < n_ranks; ++d)
        st_release_sys(reinterpret_cast<uint32_t*>(peer[d]) + kEpFlagArrive + a.rank, step);
      *reinterpret_cast<volatile uint32_t*>(own + kEpStep) = step;
    }
  }
}

template <typename T>
__global__ void ep_combine_kernel(const T* __restrict__ rows, const int32_t* __restrict__ slot_row,
                                  const void* __restrict__ w, int w_dtype, int64_t n_tokens,
                                  int top_k, int64_t H, const T* __restrict__ base,
                                  T* __restrict__ out, uint32_t* wait_hdr, int n_ranks,
                                  uint32_t* status, unsigned long long wait_ns) {
  if (wait_hdr) {  // peer exchange: every expert rank has returned this step's rows
    const uint32_t step = *reinterpret_cast<const volatile uint32_t*>(wait_hdr + kEpStep);
    bool ok = true;
    if (threadIdx.x < n_ranks)
      ok = ep_wait_flag(wait_hdr + kEpFlagReturn + threadIdx.x, step, status, wait_hdr, wait_ns);
    // a return that never came: the rows are not this step's, leave out untouched
    if (__syncthreads_or(!ok)) return;
  }
  for (int64_t t = blockIdx.x; t < n_tokens; t += gridDim.x) {
    for (int64_t h = threadIdx.x; h < H; h += blockDim.x) {
      float acc = base ? to_f32<T>(base[t * H + h]) : 0.f;
      for (int j = 0; j < top_k; ++j) {
        const int32_t r = slot_row[t * top_k + j];
        if (r < 0) continue;
        // rows written by other GPUs during this kernel's wait: L2, not L1
        const T v = wait_hdr ? __ldcg(rows + static_cast<int64_t>(r) * H + h)
                             : rows[static_cast<int64_t>(r) * H + h];
        acc = __fadd_rn(acc, __fmul_rn(load_as_f32(w, w_dtype, t * top_k + j), to_f32<T>(v)));
      }
      out[t * H + h] = from_f32<T>(acc);
    }
  }
}

// One thread per source rank waits for its arrival flag of the current step.
__global__ void ep_wait_arrivals_kernel(uint32_t* hdr, int n_ranks, uint32_t* status,
                                        unsigned long long wait_ns) {
  const uint32_t step = *reinterpret_cast<const volatile uint32_t*>(hdr + kEpStep);
  if (threadIdx.x < n_ranks)
    ep_wait_flag(hdr + kEpFlagArrive + threadIdx.x, step, status, hdr, wait_ns);
}

template <typename T>
__device__ __forceinline__ uint4 round8(float4 x, float4 y);
template <>
__device__ __forceinline__ uint4 round8<__half>(float4 x, float4 y) {
  __half2 h[4] = {__floats2half2_rn(x.x, x.y), __floats2half2_rn(x.z, x.w),
                  __floats2half2_rn(y.x, y.y), __floats2half2_rn(y.z, y.w)};
  return *reinterpret_cast<uint4*>(h);
}
template <>
__device__ __forceinline__ uint4 round8<__nv_bfloat16>(float4 x, float4 y) {
  __nv_bfloat162 h[4] = {__floats2bfloat162_rn(x.x, x.y), __floats2bfloat162_rn(x.z, x.w),
                         __floats2bfloat162_rn(y.x, y.y), __floats2bfloat162_rn(y.z, y.w)};
  return *reinterpret_cast<uint4*>(h);
}

// Received row q (source q / cap, entry q % cap) whose expert output sits at
// sorted position pos_of_slot[q] of the fp32 partials goes back, rounded, to
// row rank*cap + q % cap of the source's back area.  0 + v, as the layer's
// combine computes for one slot of weight 1.
template <typename T>
__global__ void __launch_bounds__(kEpThreads) ep_return_kernel(
    const float* __restrict__ partial, const int32_t* __restrict__ pos_of_slot, int64_t H,
    int rows, int cap, int n_ranks, int rank, uint8_t* const* peers, int64_t back_off) {
  __shared__ uint8_t* peer[kEpMaxRanks];
  for (int d = threadIdx.x; d < n_ranks; d += kEpThreads) peer[d] = peers[d];
  __syncthreads();
  // an arrival that never came (this step's rows are incomplete): send
  // nothing back and raise no return flag
  if (*reinterpret_cast<const volatile uint32_t*>(reinterpret_cast<uint32_t*>(peer[rank]) + kEpFailed))
    return;
  const int64_t oct = H / 8;
  for (int q = blockIdx.x; q < rows; q += gridDim.x) {
    const int pos = pos_of_slot[q];
    if (pos < 0) continue;
    const int src = q / cap;
    uint4* dstrow = reinterpret_cast<uint4*>(peer[src] + back_off) +
                    static_cast<int64_t>(rank * cap + (q - src * cap)) * oct;
    const float4* srow = reinterpret_cast<const float4*>(partial + static_cast<int64_t>(pos) * H);
    for (int64_t c = threadIdx.x; c < oct; c += kEpThreads) {
      float4 x = __ldg(srow + 2 * c), y = __ldg(srow + 2 * c + 1);
      x = make_float4(__fadd_rn(0.f, x.x), __fadd_rn(0.f, x.y), __fadd_rn(0.f, x.z), __fadd_rn(0.f, x.w));
      y = make_float4(__fadd_rn(0.f, y.x), __fadd_rn(0.f, y.y), __fadd_rn(0.f, y.z), __fadd_rn(0.f, y.w));
      dstrow[c] = round8<T>(x, y);
    }
  }
  uint32_t* own = reinterpret_cast<uint32_t*>(peer[rank]);
  if (ep_last_cta(own + kEpTicketReturn) && threadIdx.x == 0) {
    const uint32_t step = *reinterpret_cast<volatile uint32_t*>(own + kEpStep);
    for (int d = 0; d < n_ranks; ++d)
      st_release_sys(reinterpret_cast<uint32_t*>(peer[d]) + kEpFlagReturn + rank, step);
  }
}

// This rank's own block (block n_ranks of the receive area): token t's row
// for its shared expert s at entry n_shared * t + s, id n_local + s; the
// block's other entries get id -1 (no expert).
template <typename T>
__global__ void __launch_bounds__(kEpThreads) ep_own_block_kernel(
    const T* __restrict__ x, int64_t n_tokens, int n_shared, int n_local, int64_t H, int cap,
    T* __restrict__ rows, int32_t* __restrict__ ids) {
  const int64_t used = n_tokens * n_shared;
  const int64_t oct = H / 8;
  for (int64_t r = blockIdx.x; r < cap; r += gridDim.x) {
    if (r >= used) {
      if (threadIdx.x == 0) ids[r] = -1;
      continue;
    }
    const int64_t t = r / n_shared;
    const int s = static_cast<int>(r - t * n_shared);
    if (threadIdx.x == 0) ids[r] = n_local + s;
    const uint4* src = reinterpret_cast<const uint4*>(x + t * H);
    uint4* dst = reinterpret_cast<uint4*>(rows + r * H);
    for (int64_t c = threadIdx.x; c < oct; c += kEpThreads) dst[c] = src[c];
  }
}

// Shared-expert output of this rank's tokens from the own block's fp32
// partials: out[t] = (0 + p(t, 0)) + p(t, 1) + ... in expert order, rounded
// once: what the layer's combine gives for the shared experts with weight 1.
template <typename T>
__global__ void __launch_bounds__(kEpThreads) ep_shared_sum_kernel(
    const float* __restrict__ partial, const int32_t* __restrict__ pos_of_slot, int64_t base,
    int64_t n_tokens, int n_shared, int64_t H, T* __restrict__ out) {
  for (int64_t t = blockIdx.x; t < n_tokens; t += gridDim.x) {
    for (int64_t h = threadIdx.x; h < H; h += kEpThreads) {
      float acc = 0.f;
      for (int s = 0; s < n_shared; ++s) {
        const int pos = pos_of_slot[base + t * n_shared + s];
        if (pos >= 0) acc = __fadd_rn(acc, __ldg(partial + static_cast<int64_t>(pos) * H + h));
      }
      out[t * H + h] = from_f32<T>(acc);
    }
  }
}

__global__ void ep_fill_kernel(float* p, int64_t n, float v) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    p[i] = v;
}

bool is_act(int d) { return d == EXQ_F16 || d == EXQ_BF16; }

size_t pack_smem(int n_ranks, int64_t n) {
  return sizeof(int) * (static_cast<size_t>(kEpWarps + 1) * n_ranks + 1 + 2 * n);
}

template <bool kPeer>
int launch_pack(const EpPackArgs& a, cudaStream_t s) {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaFuncSetAttribute(ep_pack_kernel<kPeer>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(pack_smem(kEpMaxRanks, kRouteGatherMaxSlots)));
    attr_set[dev] = true;
  }
  int64_t grid = a.n > 0 ? a.n : 1;
  if (grid > 2 * num_sms()) grid = 2 * num_sms();
  ep_pack_kernel<kPeer><<<static_cast<int>(grid), kEpThreads, pack_smem(a.n_ranks, a.n), s>>>(a);
  EXQ_CHECK_LAUNCH("ep_pack_kernel");
  return EXQ_OK;
}

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
  EpPackArgs a{};
  a.ids = topk_ids;
  a.ids_dtype = ids_dtype;
  a.n = static_cast<int>(n);
  a.top_k = top_k;
  a.per_rank = experts_per_rank;
  a.n_ranks = n_ranks;
  a.hidden = static_cast<const uint8_t*>(hidden);
  a.row_bytes = hidden_size * 2;
  a.send_rows = static_cast<uint8_t*>(send_rows);
  a.send_ids = send_ids;
  a.counts = counts;
  a.slot_row = slot_row;
  a.status = st;
  return launch_pack<false>(a, s);
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
        hidden_size, static_cast<const __half*>(base), static_cast<__half*>(out), nullptr, 0,
        nullptr, 0ull);
  else
    ep_combine_kernel<__nv_bfloat16><<<grid, threads, 0, s>>>(
        static_cast<const __nv_bfloat16*>(rows), slot_row, weights, w_dtype, n_tokens, top_k,
        hidden_size, static_cast<const __nv_bfloat16*>(base), static_cast<__nv_bfloat16*>(out),
        nullptr, 0, nullptr, 0ull);
  EXQ_CHECK_LAUNCH("ep_combine_kernel");
  return EXQ_OK;
}

// ------------------------------------------------------------ peer exchange

static bool ep_sizes_ok(int32_t n_ranks, int64_t capacity, int64_t hidden_size) {
  return n_ranks > 0 && n_ranks <= kEpMaxRanks && capacity > 0 && hidden_size > 0 &&
         hidden_size % 8 == 0 && capacity * n_ranks <= (int64_t{1} << 30);
}

extern "C" size_t exq_ep_buffer_bytes(int32_t n_ranks, int64_t capacity, int64_t hidden_size) {
  if (!ep_sizes_ok(n_ranks, capacity, hidden_size)) return 0;
  return static_cast<size_t>(ep_layout(n_ranks, capacity, 2 * hidden_size).bytes);
}

extern "C" int exq_ep_set_wait_timeout(uint64_t ns) {
  g_ep_wait_ns = ns == 0 ? kEpWaitNsDefault : static_cast<unsigned long long>(ns);
  return EXQ_OK;
}

extern "C" int exq_ep_buffer_init(void* buffer, int32_t n_ranks, int64_t capacity,
                                  int64_t hidden_size, void* stream) {
  EXQ_CHECK_ARG(ep_sizes_ok(n_ranks, capacity, hidden_size),
                "ep_buffer_init: bad sizes (ranks %d, capacity %lld, hidden %lld)", n_ranks,
                (long long)capacity, (long long)hidden_size);
  EXQ_CHECK_ARG(buffer, "ep_buffer_init: buffer is null");
  auto s = static_cast<cudaStream_t>(stream);
  const EpLayout l = ep_layout(n_ranks, capacity, 2 * hidden_size);
  const int64_t rows = static_cast<int64_t>(n_ranks + 1) * capacity;  // with the own block
  uint8_t* b = static_cast<uint8_t*>(buffer);
  if (cudaMemsetAsync(b, 0, kEpHeaderBytes, s) != cudaSuccess ||
      cudaMemsetAsync(b + l.ids, 0xFF, 4 * rows, s) != cudaSuccess) {
    set_error("ep_buffer_init: cudaMemsetAsync failed");
    return EXQ_ERR_CUDA;
  }
  ep_fill_kernel<<<static_cast<int>(rows / 256 + 1 < 1024 ? rows / 256 + 1 : 1024), 256, 0, s>>>(
      reinterpret_cast<float*>(b + l.ones), rows, 1.0f);
  EXQ_CHECK_LAUNCH("ep_fill_kernel");
  return EXQ_OK;
}

extern "C" int exq_ep_ipc_alloc(size_t bytes, void** ptr_out, void* handle_out) {
  EXQ_CHECK_ARG(bytes > 0 && ptr_out && handle_out, "ep_ipc_alloc: bad arguments");
  static_assert(sizeof(cudaIpcMemHandle_t) == EXQ_IPC_HANDLE_BYTES, "IPC handle size");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) {
    set_error("ep_ipc_alloc: cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    return EXQ_ERR_CUDA;
  }
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    set_error("ep_ipc_alloc: cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
    return EXQ_ERR_CUDA;
  }
  memcpy(handle_out, &h, sizeof(h));
  *ptr_out = p;
  return EXQ_OK;
}

extern "C" int exq_ep_ipc_free(void* ptr) {
  if (!ptr) return EXQ_OK;
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) {
    set_error("ep_ipc_free: %s", cudaGetErrorString(e));
    return EXQ_ERR_CUDA;
  }
  return EXQ_OK;
}

extern "C" int exq_ep_ipc_open(const void* handle, void** ptr_out) {
  EXQ_CHECK_ARG(handle && ptr_out, "ep_ipc_open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    set_error("ep_ipc_open: %s", cudaGetErrorString(e));
    return EXQ_ERR_CUDA;
  }
  *ptr_out = p;
  return EXQ_OK;
}

extern "C" int exq_ep_ipc_close(void* ptr) {
  if (!ptr) return EXQ_OK;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) {
    set_error("ep_ipc_close: %s", cudaGetErrorString(e));
    return EXQ_ERR_CUDA;
  }
  return EXQ_OK;
}

extern "C" int exq_ep_dispatch(const void* topk_ids, int ids_dtype, int64_t n_tokens,
                               int32_t top_k, int32_t experts_per_rank, int32_t n_ranks,
                               int32_t rank, const void* hidden, int dtype, int64_t hidden_size,
                               int64_t capacity, void* const* peers, int32_t* slot_row,
                               void* stream) {
  EXQ_CHECK_ARG(ids_dtype == EXQ_I32 || ids_dtype == EXQ_I64,
                "ep_dispatch: ids must be int32/int64");
  EXQ_CHECK_ARG(is_act(dtype), "ep_dispatch: hidden must be fp16 or bf16");
  EXQ_CHECK_ARG(ep_sizes_ok(n_ranks, capacity, hidden_size) && 0 <= rank && rank < n_ranks &&
                    top_k > 0 && experts_per_rank > 0 && n_tokens >= 0,
                "ep_dispatch: bad sizes (rank %d of %d, capacity %lld, hidden %lld, top_k %d)",
                rank, n_ranks, (long long)capacity, (long long)hidden_size, top_k);
  const int64_t n = n_tokens * top_k;
  if (n > kRouteGatherMaxSlots) {
    set_error("ep_dispatch: %lld slots exceed %lld per call", (long long)n,
              (long long)kRouteGatherMaxSlots);
    return EXQ_ERR_UNSUPPORTED;
  }
  EXQ_CHECK_ARG(peers && (n == 0 || (topk_ids && hidden && slot_row)),
                "ep_dispatch: null pointer");
  EXQ_CHECK_ARG(reinterpret_cast<uintptr_t>(hidden) % 16 == 0,
                "ep_dispatch: hidden must be 16-byte aligned");
  uint32_t* st = device_status_ptr();
  if (!st) return EXQ_ERR_CUDA;
  EpPackArgs a{};
  a.ids = topk_ids;
  a.ids_dtype = ids_dtype;
  a.n = static_cast<int>(n);
  a.top_k = top_k;
  a.per_rank = experts_per_rank;
  a.n_ranks = n_ranks;
  a.hidden = static_cast<const uint8_t*>(hidden);
  a.row_bytes = hidden_size * 2;
  a.peers = reinterpret_cast<uint8_t* const*>(peers);
  a.rank = rank;
  a.cap = static_cast<int>(capacity);
  a.lay = ep_layout(n_ranks, capacity, 2 * hidden_size);
  a.slot_row = slot_row;
  a.status = st;
  return launch_pack<true>(a, static_cast<cudaStream_t>(stream));
}

extern "C" int exq_ep_expert_forward(const exq_moe_weights* weights, int dtype, int32_t n_ranks,
                                     int32_t rank, int64_t capacity, void* buffer,
                                     void* const* peers, void* workspace, size_t workspace_bytes,
                                     void* stream) {
  EXQ_CHECK_ARG(weights && buffer && peers, "ep_expert_forward: null pointer");
  EXQ_CHECK_ARG(is_act(dtype), "ep_expert_forward: dtype must be fp16 or bf16");
  EXQ_CHECK_ARG(weights->n_shared == 0, "ep_expert_forward: shared experts run outside the exchange");
  const int64_t H = weights->hidden;
  EXQ_CHECK_ARG(ep_sizes_ok(n_ranks, capacity, H) && 0 <= rank && rank < n_ranks,
                "ep_expert_forward: bad sizes (rank %d of %d, capacity %lld)", rank, n_ranks,
                (long long)capacity);
  uint32_t* st = device_status_ptr();
  if (!st) return EXQ_ERR_CUDA;
  auto s = static_cast<cudaStream_t>(stream);
  uint8_t* b = static_cast<uint8_t*>(buffer);
  const EpLayout l = ep_layout(n_ranks, capacity, 2 * H);
  const int64_t rows = static_cast<int64_t>(n_ranks) * capacity;
  ep_wait_arrivals_kernel<<<1, kEpMaxRanks, 0, s>>>(reinterpret_cast<uint32_t*>(b), n_ranks, st,
                                                     g_ep_wait_ns);
  EXQ_CHECK_LAUNCH("ep_wait_arrivals_kernel");
  int r = exq_moe_layer_forward_range(weights, b + l.recv, dtype, rows, b + l.ids, EXQ_I32,
                                      b + l.ones, EXQ_F32, 1, b + l.back, workspace,
                                      workspace_bytes, stream, 0, 4);
  if (r != EXQ_OK) return r;
  const float* partial = nullptr;
  const int32_t* pos = nullptr;
  layer_partials(workspace, rows, rows, weights->n_routed, H, weights->inter, &partial, &pos);
  int grid = static_cast<int>(rows < 2 * num_sms() ? rows : 2 * num_sms());
  if (dtype == EXQ_F16)
    ep_return_kernel<__half><<<grid, kEpThreads, 0, s>>>(
        partial, pos, H, static_cast<int>(rows), static_cast<int>(capacity), n_ranks, rank,
        reinterpret_cast<uint8_t* const*>(peers), l.back);
  else
    ep_return_kernel<__nv_bfloat16><<<grid, kEpThreads, 0, s>>>(
        partial, pos, H, static_cast<int>(rows), static_cast<int>(capacity), n_ranks, rank,
        reinterpret_cast<uint8_t* const*>(peers), l.back);
  EXQ_CHECK_LAUNCH("ep_return_kernel");
  return EXQ_OK;
}

extern "C" int exq_ep_expert_forward_shared(const exq_moe_weights* weights, int dtype,
                                            int32_t n_ranks, int32_t rank, int64_t capacity,
                                            void* buffer, void* const* peers, const void* hidden,
                                            int64_t n_tokens, int32_t n_shared, void* shared_out,
                                            void* workspace, size_t workspace_bytes,
                                            void* stream) {
  EXQ_CHECK_ARG(weights && buffer && peers, "ep_expert_forward_shared: null pointer");
  EXQ_CHECK_ARG(is_act(dtype), "ep_expert_forward_shared: dtype must be fp16 or bf16");
  EXQ_CHECK_ARG(weights->n_shared == 0 && n_shared >= 1 && n_shared < weights->n_routed,
                "ep_expert_forward_shared: the bank holds the local experts, then the %d shared "
                "ones, all as routed experts", n_shared);
  const int64_t H = weights->hidden;
  EXQ_CHECK_ARG(ep_sizes_ok(n_ranks, capacity, H) && 0 <= rank && rank < n_ranks,
                "ep_expert_forward_shared: bad sizes (rank %d of %d, capacity %lld)", rank,
                n_ranks, (long long)capacity);
  EXQ_CHECK_ARG(n_tokens >= 0 && n_tokens * n_shared <= capacity,
                "ep_expert_forward_shared: %lld tokens x %d shared experts exceed the %lld rows "
                "of the own block", (long long)n_tokens, n_shared, (long long)capacity);
  EXQ_CHECK_ARG(n_tokens == 0 || (hidden && shared_out), "ep_expert_forward_shared: null pointer");
  EXQ_CHECK_ARG(reinterpret_cast<uintptr_t>(hidden) % 16 == 0,
                "ep_expert_forward_shared: hidden must be 16-byte aligned");
  uint32_t* st = device_status_ptr();
  if (!st) return EXQ_ERR_CUDA;
  auto s = static_cast<cudaStream_t>(stream);
  uint8_t* b = static_cast<uint8_t*>(buffer);
  const EpLayout l = ep_layout(n_ranks, capacity, 2 * H);
  const int64_t peer_rows = static_cast<int64_t>(n_ranks) * capacity;
  const int64_t rows = peer_rows + capacity;  // the peers' blocks and the own block
  const int n_local = weights->n_routed - n_shared;
  {
    const int grid = static_cast<int>(capacity < 2 * num_sms() ? capacity : 2 * num_sms());
    int32_t* ids = reinterpret_cast<int32_t*>(b + l.ids) + peer_rows;
    if (dtype == EXQ_F16)
      ep_own_block_kernel<__half><<<grid, kEpThreads, 0, s>>>(
          static_cast<const __half*>(hidden), n_tokens, n_shared, n_local, H,
          static_cast<int>(capacity), reinterpret_cast<__half*>(b + l.recv) + peer_rows * H, ids);
    else
      ep_own_block_kernel<__nv_bfloat16><<<grid, kEpThreads, 0, s>>>(
          static_cast<const __nv_bfloat16*>(hidden), n_tokens, n_shared, n_local, H,
          static_cast<int>(capacity), reinterpret_cast<__nv_bfloat16*>(b + l.recv) + peer_rows * H,
          ids);
    EXQ_CHECK_LAUNCH("ep_own_block_kernel");
  }
  ep_wait_arrivals_kernel<<<1, kEpMaxRanks, 0, s>>>(reinterpret_cast<uint32_t*>(b), n_ranks, st,
                                                     g_ep_wait_ns);
  EXQ_CHECK_LAUNCH("ep_wait_arrivals_kernel");
  // one layer call: the received rows for the local experts and this rank's
  // own tokens for the shared experts
  int r = exq_moe_layer_forward_range(weights, b + l.recv, dtype, rows, b + l.ids, EXQ_I32,
                                      b + l.ones, EXQ_F32, 1, b + l.back, workspace,
                                      workspace_bytes, stream, 0, 4);
  if (r != EXQ_OK) return r;
  const float* partial = nullptr;
  const int32_t* pos = nullptr;
  layer_partials(workspace, rows, rows, weights->n_routed, H, weights->inter, &partial, &pos);
  const int grid = static_cast<int>(peer_rows < 2 * num_sms() ? peer_rows : 2 * num_sms());
  const int sgrid = static_cast<int>(n_tokens < 2 * num_sms() ? (n_tokens > 0 ? n_tokens : 1)
                                                                 : 2 * num_sms());
  if (dtype == EXQ_F16) {
    ep_return_kernel<__half><<<grid, kEpThreads, 0, s>>>(
        partial, pos, H, static_cast<int>(peer_rows), static_cast<int>(capacity), n_ranks, rank,
        reinterpret_cast<uint8_t* const*>(peers), l.back);
    ep_shared_sum_kernel<__half><<<sgrid, kEpThreads, 0, s>>>(
        partial, pos, peer_rows, n_tokens, n_shared, H, static_cast<__half*>(shared_out));
  } else {
    ep_return_kernel<__nv_bfloat16><<<grid, kEpThreads, 0, s>>>(
        partial, pos, H, static_cast<int>(peer_rows), static_cast<int>(capacity), n_ranks, rank,
        reinterpret_cast<uint8_t* const*>(peers), l.back);
    ep_shared_sum_kernel<__nv_bfloat16><<<sgrid, kEpThreads, 0, s>>>(
        partial, pos, peer_rows, n_tokens, n_shared, H,
        static_cast<__nv_bfloat16*>(shared_out));
  }
  EXQ_CHECK_LAUNCH("ep_return_kernel / ep_shared_sum_kernel");
  return EXQ_OK;
}

extern "C" int exq_ep_combine_peer(const void* buffer, int32_t n_ranks, int64_t capacity,
                                   int64_t hidden_size, int dtype, const int32_t* slot_row,
                                   const void* weights, int w_dtype, int64_t n_tokens,
                                   int32_t top_k, const void* base, void* out, void* stream) {
  EXQ_CHECK_ARG(is_act(dtype), "ep_combine_peer: dtype must be fp16 or bf16");
  EXQ_CHECK_ARG(w_dtype == EXQ_F32 || is_act(w_dtype), "ep_combine_peer: weights dtype unsupported");
  EXQ_CHECK_ARG(ep_sizes_ok(n_ranks, capacity, hidden_size) && top_k > 0 && n_tokens >= 0,
                "ep_combine_peer: bad sizes");
  EXQ_CHECK_ARG(buffer && (n_tokens == 0 || (slot_row && weights && out)),
                "ep_combine_peer: null pointer");
  uint32_t* st = device_status_ptr();
  if (!st) return EXQ_ERR_CUDA;
  auto s = static_cast<cudaStream_t>(stream);
  const uint8_t* b = static_cast<const uint8_t*>(buffer);
  const EpLayout l = ep_layout(n_ranks, capacity, 2 * hidden_size);
  uint32_t* hdr = reinterpret_cast<uint32_t*>(const_cast<uint8_t*>(b));
  // with no tokens one CTA still waits, so that the step ends with every return
  const int threads = static_cast<int>(hidden_size < 256 ? (hidden_size < kEpMaxRanks ? kEpMaxRanks : hidden_size) : 256);
  const int grid = static_cast<int>(n_tokens == 0 ? 1 : (n_tokens < 65535 ? n_tokens : 65535));
  if (dtype == EXQ_F16)
    ep_combine_kernel<__half><<<grid, threads, 0, s>>>(
        reinterpret_cast<const __half*>(b + l.back), slot_row, weights, w_dtype, n_tokens, top_k,
        hidden_size, static_cast<const __half*>(base), static_cast<__half*>(out), hdr, n_ranks,
        st, g_ep_wait_ns);
  else
    ep_combine_kernel<__nv_bfloat16><<<grid, threads, 0, s>>>(
        reinterpret_cast<const __nv_bfloat16*>(b + l.back), slot_row, weights, w_dtype, n_tokens,
        top_k, hidden_size, static_cast<const __nv_bfloat16*>(base),
        static_cast<__nv_bfloat16*>(out), hdr, n_ranks, st, g_ep_wait_ns);
  EXQ_CHECK_LAUNCH("ep_combine_kernel");
  return EXQ_OK;
}
