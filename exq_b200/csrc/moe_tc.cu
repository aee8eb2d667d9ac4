// Warp-specialised tcgen05 grouped GEMM for the MoE expert layer (sm_100a).
//
// Replaces the reference's two Triton INT4 GEMM launches plus gather,
// silu_and_mul and the down half of the combine
// (exq/kernels/moe_int4_kernel.py:124-240, :374-426;
// exq/runtime/sglang_backend.py:117-156) for experts that mix BF16, INT8 and
// INT4 weight tiers.
//
// One persistent CTA per SM (672 threads, 21 warps):
//   warp 0       weight producer: one TMA per 16 KB slot brings 128 weight rows
//                x 256 k (INT4; INT8 128 k, 16-bit 64 k) into a 6-slot smem
//                ring, plus one TMA for the INT4 group scales of the slot
//   warp 1       activation producer: TMA 2D loads (128B swizzle) of the
//                item's token rows into a 3-slot ring of 32 KB slots; a slot
//                holds 256/N k-stages of N rows (a whole number of weight
//                slots), so small items prefetch deep
//   warp 2       MMA issuer: one thread issues tcgen05.mma with A (weights) in
//                tensor memory and B (tokens) in shared memory, M=128 rows,
//                N=tokens, K=16, into a double-buffered accumulator
//   warps 3-6    epilogue: tcgen05.ld of the accumulator, fused SiLU*mul
//                (gate_up) or fp32 partials, INT8 row scale applied (down);
//                the router weights are applied by the combine
//   warps 7-18   dequantisers, three groups of four warps (one per lane
//                quarter).  Group g takes every third weight slot (weight-ring
//                positions g and g+3, tensor-memory A buffer g), so each ring
//                position and A buffer has one consumer group and the groups
//                run staggered.  A warp turns its 32 rows x the slot's k (INT4
//                256 k, INT8 128 k, 16-bit 64 k) into fp16 (scale applied) in
//                registers, 64 k at a time, and writes them to its lanes of the
//                A buffer with tcgen05.st
//   warps 19-20  combine: stage the slot positions and weights of this CTA's
//                tokens, wait until every CTA's down items are stored, then
//                (with warps 3-18) sum each token's partial rows
// A work item is (expert, 128-row block of the projection, up to MT tokens
// of that expert): every weight byte is dequantised once per item and all the
// expert's tokens ride in the MMA's N dimension.  gate_up items come first,
// then down items; a down item's activation producer waits on its tile's count
// of stored gate_up row blocks (both projections in one launch).
//
// Tensor memory (512 columns), MT = 64: accumulators at [0,64) and [64,128);
// three A buffers of 128 columns (128 rows x 256 fp16) at [128,512); the third
// A buffer lets the dequantisers run one weight slot further ahead of the MMA.
// MT = 128 (calls with many rows per expert): accumulators at [0,128) and
// [128,256), two A buffers at [256,512), two dequant groups (warps 15-18 have
// no slots).
//
// K order.  Inside every 8-element octet the k order is permuted to
// [0,4,1,5,2,6,3,7] identically for weights and activations (a dot product
// does not depend on term order).  With it a packed INT4 word dequantises with
// the 1024.0 magic-number trick straight into K-adjacent fp16 pairs, the INT8
// and 16-bit tiers are stored pre-permuted at pack time, and the activation
// prep kernel permutes rows.
#include <string.h>

#include <type_traits>

#include "tc_common.cuh"

namespace exq {
namespace tc {

constexpr int kWarps = 21;
constexpr int kThreads = kWarps * 32;
constexpr int kWarpW = 0, kWarpB = 1, kWarpMma = 2;
constexpr int kWarpCmb0 = 19, kNumCmb = 2;  // wait for the down items, then join the combine
constexpr int kTailWarp0 = 3, kTailWarps = kWarps - 3;  // epilogue, dequant and combine warps
constexpr int kCmbMaxSpt = 16;  // slots per token the fused combine handles
constexpr int kEpiWarp0 = 3, kNumEpiWarps = 4;
constexpr int kDqWarp0 = 7, kDqGroups = 3, kDqGroupWarps = 4;  // 3 groups x 4 lane quarters
constexpr int kWStages = 6, kABufs = 3, kBStages = 3;  // weight slots, TMEM A buffers, B slots
constexpr int kWSlot = 16384, kSSlot = 512, kBSlot = 32768;
constexpr int kACols = 128;  // tensor-memory columns per A buffer (128 rows x 256 fp16)
// Tokens per item (the MMA's N), a template parameter of the kernel:
//   64: two accumulators of 64 columns + three 128-column A buffers (three
//       dequant groups), the decode build;
//  128: two accumulators of 128 columns + two A buffers (two dequant groups),
//       for calls with many rows per expert: each expert's weights are
//       streamed and converted once per 128 tokens instead of 64.
// Either way the 512 tensor-memory columns are full.
constexpr int kMaxN = 64;
constexpr int kWideN = 128;
constexpr int kBRows = 256;      // activation rows one B slot holds (256 rows x 128 B)
constexpr int kTmemCols = 512;
constexpr int kKS = 64;          // k per pipeline stage

constexpr int kOffB = 0;
constexpr int kOffW = kOffB + kBStages * kBSlot;
constexpr int kOffS = kOffW + kWStages * kWSlot;
constexpr int kOffBar = kOffS + kWStages * kSSlot;
constexpr int kNumBars = 2 * kWStages + 2 * kABufs + 2 * kBStages + 4;
constexpr int kOffMisc = kOffBar + kNumBars * 8;
constexpr int kItemTab = 128;  // work items of this CTA decoded into shared memory up front
constexpr int kOffItems = kOffMisc + 64;
constexpr int kItemBytes = 48;  // sizeof(Item)
constexpr int kHistBuckets = 1024;  // experts the in-kernel tile list handles
constexpr int kOffHist = kOffItems + kItemTab * kItemBytes;  // 3 x (kHistBuckets + 1) ints
// The histogram region is free once the item table is built; the combine at
// the end of the launch then keeps there the slot positions and router
// weights of this CTA's share of the tokens (kCmbEntries ints + floats).
constexpr int kOffCmb = kOffHist;
constexpr int kHistRegion = 3 * (kHistBuckets + 1) * 4;
constexpr int kCmbEntries = kHistRegion / 8;
constexpr int kSmemBytes = kOffHist + kHistRegion + 1024;  // + slack to align the base to 1024 B
static_assert(kSmemBytes <= 232448, "shared memory per CTA");
constexpr int kEpiBar = 1;   // named barrier of the four epilogue warps
constexpr int kTailBar = 2;  // named barrier of the combine at the end (kTailWarps warps)

enum : int { kTierBF16 = EXQ_TIER_BF16, kTierINT8 = EXQ_TIER_INT8, kTierINT4 = EXQ_TIER_INT4 };

// Constants of one projection (gate_up or down).
struct ProjParams {
  CUtensorMap tm_w[3];  // weights per tier storage
  CUtensorMap tm_s;     // INT4 group scales (group-major)
  CUtensorMap tm_b[4];  // activations, stage-major [k/64][n_pos][64] fp16 (octet-permuted);
                        // map b: box of N = 16(b+1) rows x the stages of one B slot
  const __half* s8;     // INT8 per-row scales
  void* out;            // gate_up: mid (fp16, stage-major); down: fp32 partials [n_pos, H]
  int64_t out_stride;
  int gate_up;          // 1: gate_up (rows interleave gate/up), 0: down
  int n_rows;           // rows of the projection (2I or H)
  int k;
  int nblocks;          // row blocks per tile: I/64 gate/up pairs, or H/128
};

// A launch runs the gate_up items (if run_gu) and then the down items (if
// run_dn) of every tile.  Items are numbered tile-major inside each
// projection: gate_up item i is (tile i / nb_gu, row block i % nb_gu).
struct TcParams {
  ProjParams pj[2];  // [0] gate_up, [1] down
  int run_gu, run_dn;
  // link (both projections in one launch): a gate_up item adds 1 to
  // tile_done[tile] once its mid rows are stored; a down item's activation
  // producer waits until all nb_gu row blocks of its tile have done so.
  int link;
  int* tile_done;
  // fuse_combine: every CTA adds 1 to *dn_done (zeroed by the route stage)
  // once its epilogue has stored all its items; when all have, the CTAs sum
  // y[t] = sum_j w[t, j] * partial[pos(t, j)] for their share of the tokens,
  // in slot order with the rounding of combine_partials_kernel.
  int fuse_combine;
  int* dn_done;
  const int32_t* sorted_slot;  // slot at every sorted position
  const int32_t* pos_of_slot;  // sorted position of every slot (-1: dropped)
  const void* topk_w;
  int w_dtype;
  void* y;
  int y_dtype;
  int64_t hidden;
  const int32_t* expert_slot;  // tier << 24 | index inside the tier storage
  const int32_t* tile_info;
  const int32_t* n_tiles_ptr;
  int max_tiles;
  int inter;
  int weights_early;      // 1: the tile list is complete before this kernel starts (see below)
  // tiles_from_ids: build the tile list from the routing ids (below) instead of
  // reading tile_info, so the weight stream need not wait for the predecessor
  int tiles_from_ids;
  const void* ids;        // [T, top_k] expert ids
  int ids_dtype, top_k, spt, n_routed, n_buckets;
  int64_t n_slots;
  int64_t n_pos;          // rows of the activation / mid buffers
  uint32_t* status;
};

// k-stages (64 k each) carried by one 16 KB weight slot: 128 rows x 128 bytes.
__device__ __forceinline__ int stages_per_slot(int tier) {
  return tier == kTierINT4 ? 4 : (tier == kTierINT8 ? 2 : 1);
}

// k-stages of n activation rows one B slot carries.  64-token items: a
// multiple of 4 (the stages of an INT4 weight slot), so a weight slot never
// straddles two B slots; one 3D TMA box (n rows x these stages) fills the
// slot.  128-token items: boxes of 128 rows (rows past the tile are unused),
// 2 stages per slot, an INT4 weight slot spanning two B slots.
__host__ __device__ __forceinline__ int b_stages_per_slot(int n) {
  return (kBRows / n) & ~3;
}
__host__ __device__ __forceinline__ int b_slot_stages(int mt, int n) {
  return mt == kWideN ? kBRows / kWideN : b_stages_per_slot(n);
}

// Everything a warp needs about a work item, computed once per CTA.
struct Item {
  int e, m0, mc, nb;      // expert, first sorted row, rows, row block of the projection
  int tier, idx, n, r0;   // tier, index in the tier storage, MMA N (mc rounded up to 16), first row
  int sps, per_slot, prj, tile;  // k-stages per weight slot, per activation slot; projection, tile
};

static_assert(sizeof(Item) == kItemBytes, "item table entry size");

__device__ __forceinline__ int num_items(const TcParams& p, int n_tiles) {
  return (p.run_gu ? n_tiles * p.pj[0].nblocks : 0) + (p.run_dn ? n_tiles * p.pj[1].nblocks : 0);
}

// Projection, tile and row block of global item `item` (gate_up items first).
__device__ __forceinline__ void item_coords(const TcParams& p, int item, int n_tiles, int& prj,
                                            int& tile, int& nb) {
  const int ngu = p.run_gu ? n_tiles * p.pj[0].nblocks : 0;
  prj = (item < ngu) ? 0 : 1;
  const int j = item - (prj ? ngu : 0);
  const int nbk = p.pj[prj].nblocks;
  tile = j / nbk;
  nb = j - tile * nbk;
}

// The fields that follow from (expert, rows, projection, row block).
template <int MT>
__device__ __forceinline__ void finish_item(const TcParams& p, Item& it) {
  const int code = __ldg(p.expert_slot + it.e);
  it.tier = code >> 24;
  it.idx = code & 0xFFFFFF;
  it.n = max(16, (it.mc + 15) & ~15);
  it.r0 = p.pj[it.prj].gate_up ? it.nb * 64 : it.nb * 128;
  it.sps = stages_per_slot(it.tier);
  it.per_slot = b_slot_stages(MT, it.n);
}

template <int MT>
__device__ __forceinline__ Item make_item(const TcParams& p, int item, int n_tiles) {
  Item it;
  item_coords(p, item, n_tiles, it.prj, it.tile, it.nb);
  it.e = __ldcg(p.tile_info + 3 * it.tile);
  it.m0 = __ldcg(p.tile_info + 3 * it.tile + 1);
  it.mc = __ldcg(p.tile_info + 3 * it.tile + 2);
  finish_item<MT>(p, it);
  return it;
}

// Bounded acquire-spin until *ctr >= target (one thread).  False on timeout
// (about 2 s), after flagging the device status.
__device__ __forceinline__ bool wait_count(const int* ctr, int target, uint32_t* status) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];\n" : "=r"(v) : "l"(ctr) : "memory");
  if (v >= target) return true;
  const long long t0 = clock64();
  for (;;) {
    __nanosleep(128);
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];\n" : "=r"(v) : "l"(ctr) : "memory");
    if (v >= target) return true;
    if (clock64() - t0 > 4000000000LL) {
      atomicOr(status, EXQ_DEV_TIMEOUT);
      return false;
    }
  }
}

// Generic-proxy global writes/reads of this thread ordered against its
// async-proxy (TMA) accesses.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;\n" ::: "memory");
}

// Bounded acquire-spin until *ctr >= target that gives up only after about
// 2 s without progress (the counter grows while other CTAs work).
__device__ __forceinline__ bool wait_progress(const int* ctr, int target, uint32_t* status) {
  int v, last = -1;
  long long t0 = clock64();
  for (;;) {
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];\n" : "=r"(v) : "l"(ctr) : "memory");
    if (v >= target) return true;
    if (v != last) {
      last = v;
      t0 = clock64();
    } else if (clock64() - t0 > 4000000000LL) {
      atomicOr(status, EXQ_DEV_TIMEOUT);
      return false;
    }
    __nanosleep(128);  // one thread of every CTA polls this line
  }
}

// The CTA's li-th work item (global index `item`): from the shared table for
// the first kItemTab, else from global memory.  False for an unknown tier.
template <int MT>
__device__ __forceinline__ bool decode_item(const TcParams& p, const Item* tab, int li, int item,
                                            int n_tiles, Item& it) {
  it = li < kItemTab ? tab[li] : make_item<MT>(p, item, n_tiles);
  return it.tier == kTierINT4 || it.tier == kTierINT8 || it.tier == kTierBF16;
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
__device__ __forceinline__ void dq_int4_word(uint32_t w, __half2 s, uint32_t* o) {
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
  o[0] = *reinterpret_cast<uint32_t*>(&h0);
  o[1] = *reinterpret_cast<uint32_t*>(&h1);
  o[2] = *reinterpret_cast<uint32_t*>(&h2);
  o[3] = *reinterpret_cast<uint32_t*>(&h3);
}

// INT8 (bytes stored in permuted octet order): 4 weights -> 2 fp16 pairs.
__device__ __forceinline__ void dq_int8_word(uint32_t w, uint32_t* o) {
  const uint32_t u = w ^ 0x80808080u;
  uint32_t a = prmt(u, 0x64646464u, 0x4140u);
  uint32_t b = prmt(u, 0x64646464u, 0x4342u);
  const __half2 sub = __float2half2_rn(1152.0f);
  __half2 ha = __hsub2(*reinterpret_cast<__half2*>(&a), sub);
  __half2 hb = __hsub2(*reinterpret_cast<__half2*>(&b), sub);
  o[0] = *reinterpret_cast<uint32_t*>(&ha);
  o[1] = *reinterpret_cast<uint32_t*>(&hb);
}

// One lane of a converged warp (the same lane on every call with a full mask).
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n .reg .b32 r;\n .reg .pred p;\n elect.sync r|p, 0xffffffff;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(pred));
  return pred != 0;
}

__device__ __forceinline__ uint16_t lds16(uint32_t addr) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];\n" : "=h"(v) : "r"(addr));
  return v;
}

// 32 lanes x 32 consecutive 32-bit columns from registers to tensor memory.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
      "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]),
      "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]),
      "r"(v[30]), "r"(v[31]));
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
}
// A from tensor memory, B from shared memory.
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n"
      " setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// Per-item constants of the MMA warp.
struct MmaItem {
  uint32_t d, idesc, stage_desc, bar_bfull, bar_bempty;
  int nk, per_slot;
  uint64_t bdesc0;
  uint32_t* status;
};

// MMAs of one weight slot (SPS k-stages of 64, A in tensor memory at `abuf`).
// B stages are consumed from the activation ring; a ring slot is released
// once its last stage has been issued.  Runs on the whole (converged) warp.
template <int SPS>
__device__ __forceinline__ bool mma_slot(const MmaItem& mi, uint32_t abuf, int kc0, Ring& rb,
                                         int& sidx) {
  if (SPS > 1 && sidx + SPS <= mi.per_slot && kc0 + SPS <= mi.nk) {
    // Fast path (N <= 32 for INT4): all SPS stages lie in the current B slot,
    // so one wait at most and all 4*SPS MMAs from one elected block, with the
    // descriptors computed by the whole warp beforehand.
    if (sidx == 0) {
      if (!__all_sync(0xffffffffu, mbar_wait(mi.bar_bfull + 8u * rb.idx, rb.phase, mi.status)))
        return false;
      tc_fence_after();
    }
    uint64_t bd[SPS];
    bd[0] = mi.bdesc0 + rb.idx * (kBSlot >> 4) + sidx * mi.stage_desc;
#pragma unroll
    for (int sub = 1; sub < SPS; ++sub) bd[sub] = bd[sub - 1] + mi.stage_desc;
    const bool release_b = (sidx + SPS == mi.per_slot) || (kc0 + SPS == mi.nk);
    const uint32_t first = kc0 != 0;
    if (elect_one()) {
#pragma unroll
      for (int sub = 0; sub < SPS; ++sub) {
        const uint32_t a = abuf + 32 * sub;
        tc_mma_f16_ts(mi.d, a, bd[sub], mi.idesc, sub == 0 ? first : 1u);
        tc_mma_f16_ts(mi.d, a + 8, bd[sub] + 2, mi.idesc, 1u);
        tc_mma_f16_ts(mi.d, a + 16, bd[sub] + 4, mi.idesc, 1u);
        tc_mma_f16_ts(mi.d, a + 24, bd[sub] + 6, mi.idesc, 1u);
      }
      if (release_b) tc_commit(mi.bar_bempty + 8u * rb.idx);
    }
    __syncwarp();
    sidx += SPS;
    if (release_b) {
      rb.next(kBStages);
      sidx = 0;
    }
    return true;
  }
#pragma unroll
  for (int sub = 0; sub < SPS; ++sub) {
    const int kc = kc0 + sub;
    if (kc >= mi.nk) break;
    if (sidx == 0) {
      if (!__all_sync(0xffffffffu, mbar_wait(mi.bar_bfull + 8u * rb.idx, rb.phase, mi.status)))
        return false;
      tc_fence_after();
    }
    const uint64_t bd = mi.bdesc0 + rb.idx * (kBSlot >> 4) + sidx * mi.stage_desc;
    const uint32_t a = abuf + 32 * sub;
    const bool release_b = (++sidx == mi.per_slot) || kc == mi.nk - 1;
    if (elect_one()) {
      tc_mma_f16_ts(mi.d, a, bd, mi.idesc, kc != 0);
      tc_mma_f16_ts(mi.d, a + 8, bd + 2, mi.idesc, 1u);
      tc_mma_f16_ts(mi.d, a + 16, bd + 4, mi.idesc, 1u);
      tc_mma_f16_ts(mi.d, a + 24, bd + 6, mi.idesc, 1u);
      if (release_b) tc_commit(mi.bar_bempty + 8u * rb.idx);
    }
    __syncwarp();
    if (release_b) {
      rb.next(kBStages);
      sidx = 0;
    }
  }
  return true;
}

template <int MT>
__global__ void __launch_bounds__(kThreads, 1) moe_tc_kernel(const __grid_constant__ TcParams p) {
  static_assert(MT == kMaxN || MT == kWideN, "tile heights");
  constexpr int NG = MT == kWideN ? 2 : kDqGroups;  // dequant groups = TMEM A buffers
  constexpr int kTmemA = 2 * MT;                     // first tensor-memory column of the A buffers
  static_assert(kTmemA + NG * kACols == kTmemCols, "tensor-memory columns");
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t sB = base + kOffB, sW = base + kOffW, sS = base + kOffS;
  const uint32_t bar0 = base + kOffBar;
  auto W_full = [&](int i) { return bar0 + 8u * i; };
  auto W_empty = [&](int i) { return bar0 + 8u * (kWStages + i); };
  constexpr int kBarA = 2 * kWStages, kBarAe = kBarA + kABufs, kBarB = kBarAe + kABufs;
  constexpr int kBarAcc = kBarB + 2 * kBStages;
  auto A_full = [&](int i) { return bar0 + 8u * (kBarA + i); };
  auto A_empty = [&](int i) { return bar0 + 8u * (kBarAe + i); };
  auto B_full = [&](int i) { return bar0 + 8u * (kBarB + i); };
  auto B_empty = [&](int i) { return bar0 + 8u * (kBarB + kBStages + i); };
  auto Acc_full = [&](int i) { return bar0 + 8u * (kBarAcc + i); };
  auto Acc_empty = [&](int i) { return bar0 + 8u * (kBarAcc + 2 + i); };

  volatile uint32_t* misc = reinterpret_cast<volatile uint32_t*>(gbase + kOffMisc);
  // misc[0] = TMEM base address, misc[1] = abort flag

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kWStages; ++i) {
      mbar_init(W_full(i), 1);
      mbar_init(W_empty(i), kDqGroupWarps);
    }
    for (int i = 0; i < NG; ++i) {
      mbar_init(A_full(i), kDqGroupWarps);
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
  if (threadIdx.x == 32 * kWarpW) {  // tensor-map descriptors into the TMA unit's cache
    for (int j = 0; j < 2; ++j) {
      if (j == 0 ? !p.run_gu : !p.run_dn) continue;
      for (int i = 0; i < 3; ++i) tma_prefetch_desc(&p.pj[j].tm_w[i]);
      tma_prefetch_desc(&p.pj[j].tm_s);
    }
  } else if (threadIdx.x == 32 * kWarpB) {
    for (int j = 0; j < 2; ++j) {
      if (j == 0 ? !p.run_gu : !p.run_dn) continue;
      for (int i = 0; i < (MT == kWideN ? 1 : 4); ++i) tma_prefetch_desc(&p.pj[j].tm_b[i]);
    }
  }
  if (warp == kWarpMma) {
    tmem_alloc(base + kOffMisc, kTmemCols);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[0];
  // everything above overlaps the tail of the previous kernel in the stream.
  // With p.weights_early the tile list was written two launches back, by a
  // routing kernel that had finished before the predecessor let this kernel
  // launch; with p.tiles_from_ids the CTA builds it from the routing ids, which
  // predate the routing kernel.  Either way only the activation producer
  // (which reads the predecessor's output) waits, and the weight producer and
  // the dequantisers start on the first slots at once.
  const bool early = p.weights_early || p.tiles_from_ids;
  if (!early) pdl_wait();
  pdl_trigger();
  Item* items_tab = reinterpret_cast<Item*>(gbase + kOffItems);
  int n_tiles;
  if (p.tiles_from_ids) {
    // The same tile list the routing kernel writes: experts in order, rows in
    // tiles of kMaxN from each expert's first sorted position.  Per-expert
    // counts (an order-independent histogram), then two exclusive scans.
    int* cnt = reinterpret_cast<int*>(gbase + kOffHist);
    int* rbase = cnt + kHistBuckets + 1;
    int* tstart = rbase + kHistBuckets + 1;
    const int nbk = p.n_buckets;
    for (int i = threadIdx.x; i < nbk; i += kThreads) cnt[i] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < p.n_slots; i += kThreads) {
      const int t = i / p.spt, j = i - t * p.spt;
      int e = p.n_routed + (j - p.top_k);  // always-on shared expert
      if (j < p.top_k) {
        const int64_t v = load_index(p.ids, p.ids_dtype, static_cast<int64_t>(t) * p.top_k + j);
        e = (v >= 0 && v < p.n_routed) ? static_cast<int>(v) : -1;  // dropped (flagged by routing)
      }
      if (e >= 0) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    if (warp == 0) {
      const int per = (nbk + 31) / 32;
      const int lo = lane * per, hi = min(nbk, lo + per);
      int rs = 0, ts = 0;
      for (int e = lo; e < hi; ++e) {
        rs += cnt[e];
        ts += (cnt[e] + MT - 1) / MT;
      }
      int rx = rs, tx = ts;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, rx, o);
        const int z = __shfl_up_sync(0xffffffffu, tx, o);
        if (lane >= o) {
          rx += y;
          tx += z;
        }
      }
      if (lane == 31) tstart[nbk] = tx;
      rx -= rs;
      tx -= ts;
      for (int e = lo; e < hi; ++e) {
        rbase[e] = rx;
        tstart[e] = tx;
        rx += cnt[e];
        tx += (cnt[e] + MT - 1) / MT;
      }
    }
    __syncthreads();
    n_tiles = min(tstart[nbk], p.max_tiles);
    const int n_items0 = num_items(p, n_tiles);
    for (int t = threadIdx.x; t < kItemTab; t += kThreads) {
      const int item = static_cast<int>(blockIdx.x) + t * static_cast<int>(gridDim.x);
      if (item >= n_items0) continue;
      Item it;
      item_coords(p, item, n_tiles, it.prj, it.tile, it.nb);
      int lo = 0, hi = nbk - 1;  // last expert whose first tile is <= tile
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (tstart[mid] <= it.tile) lo = mid;
        else hi = mid - 1;
      }
      const int lt = it.tile - tstart[lo];
      it.e = lo;
      it.m0 = rbase[lo] + lt * MT;
      it.mc = min(MT, cnt[lo] - lt * MT);
      finish_item<MT>(p, it);
      items_tab[t] = it;
    }
  } else {
    n_tiles = min(__ldcg(p.n_tiles_ptr), p.max_tiles);
    // decode this CTA's items once, so no role waits on global loads at an item boundary
    const int n_items0 = num_items(p, n_tiles);
    for (int t = threadIdx.x; t < kItemTab; t += kThreads) {
      const int item = static_cast<int>(blockIdx.x) + t * static_cast<int>(gridDim.x);
      if (item < n_items0) items_tab[t] = make_item<MT>(p, item, n_tiles);
    }
  }
  const int n_items = num_items(p, n_tiles);
  __syncthreads();
  auto aborted = [&]() { return misc[1] != 0; };
  auto do_abort = [&]() { misc[1] = 1; };

  if (warp == kWarpW) {
    // ---------------------------------------------------------- weights
    // The whole warp walks the loop (waits are uniform); one elected lane
    // issues, which keeps the issue path on the warp-uniform datapath.
    Ring r;
    int issued = 0;
    for (int item = blockIdx.x, li = 0; item < n_items && !aborted(); item += gridDim.x, ++li) {
      Item it;
      if (!decode_item<MT>(p, items_tab, li, item, n_tiles, it)) {
        if (lane == 0) atomicOr(p.status, EXQ_DEV_BAD_TIER);
        continue;
      }
      const ProjParams& pj = p.pj[it.prj];
      const int G = pj.k >> 7;
      const int nk = pj.k / kKS;
      const int sps = it.sps;
      bool ok = true;
      for (int kc0 = 0; kc0 < nk; kc0 += sps) {
        if (!__all_sync(0xffffffffu, mbar_wait(W_empty(r.idx), r.phase ^ 1, p.status))) {
          ok = false;
          break;
        }
        const uint32_t dst = sW + r.idx * kWSlot, bar = W_full(r.idx);
        const int xb = kc0 * (it.tier == kTierINT4 ? 32 : 64);
        if (elect_one()) {
          if (it.tier == kTierINT4) {
            mbar_arrive_tx(bar, kWSlot + kSSlot);
            if (pj.gate_up) {
              // weights: (byte, row in block, block, gate/up, expert)
              tma_load_5d(dst, &pj.tm_w[kTierINT4], bar, xb, 0, it.nb, 0, it.idx);
              // scales: (element in block, block, gate/up, group, expert); 2 groups
              tma_load_5d(sS + r.idx * kSSlot, &pj.tm_s, bar, 0, it.nb, 0, kc0 >> 1, it.idx);
            } else {
              tma_load_2d(dst, &pj.tm_w[kTierINT4], bar, xb, it.idx * pj.n_rows + it.r0);
              tma_load_2d(sS + r.idx * kSSlot, &pj.tm_s, bar, it.r0, it.idx * G + (kc0 >> 1));
            }
          } else {
            mbar_arrive_tx(bar, kWSlot);
            if (pj.gate_up)
              tma_load_5d(dst, &pj.tm_w[it.tier], bar, xb, 0, it.nb, 0, it.idx);
            else
              tma_load_2d(dst, &pj.tm_w[it.tier], bar, xb, it.idx * pj.n_rows + it.r0);
          }
        }
        __syncwarp();
        r.next(kWStages);
        ++issued;
      }
      if (!ok) {
        do_abort();
        break;
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
  } else if (warp == kWarpB) {
    // ---------------------------------------------------------- activations
    if (early) pdl_wait();
    Ring r;
    int issued = 0;
    for (int item = blockIdx.x, li = 0; item < n_items && !aborted(); item += gridDim.x, ++li) {
      Item it;
      if (!decode_item<MT>(p, items_tab, li, item, n_tiles, it)) continue;
      const ProjParams& pj = p.pj[it.prj];
      const int nk = pj.k / kKS;
      const int per_slot = it.per_slot;
      const int box_rows = MT == kWideN ? kWideN : it.n;
      const uint32_t stage_bytes = static_cast<uint32_t>(box_rows) * 128u;
      if (p.link && it.prj == 1) {
        // the tile's mid rows come from nb_gu gate_up items of this launch
        bool ok = true;
        if (lane == 0) ok = wait_count(p.tile_done + it.tile, p.pj[0].nblocks, p.status);
        if (!__shfl_sync(0xffffffffu, ok, 0)) {
          do_abort();
          break;
        }
        // every lane acquires (the TMA issuer is elected below), then orders
        // its TMA reads of mid after the acquire
        int seen;
        asm volatile("ld.acquire.gpu.global.b32 %0, [%1];\n"
                     : "=r"(seen) : "l"(p.tile_done + it.tile) : "memory");
        (void)seen;
        fence_proxy_async_global();
      }
      bool ok = true;
      for (int kc0 = 0; kc0 < nk; kc0 += per_slot) {
        if (!__all_sync(0xffffffffu, mbar_wait(B_empty(r.idx), r.phase ^ 1, p.status))) {
          ok = false;
          break;
        }
        const uint32_t bar = B_full(r.idx);
        if (elect_one()) {
          // the whole slot in one box: n rows x per_slot stages (stages past k read as zeros)
          mbar_arrive_tx(bar, static_cast<uint32_t>(per_slot) * stage_bytes);
          tma_load_3d(sB + r.idx * kBSlot, &pj.tm_b[MT == kWideN ? 0 : (it.n >> 4) - 1], bar, 0,
                      it.m0, kc0);
        }
        __syncwarp();
        r.next(kBStages);
        ++issued;
      }
      if (!ok) {
        do_abort();
        break;
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
  } else if (warp == kWarpMma) {
    // ---------------------------------------------------------- MMA issue
    // Converged warp; the elected lane issues each group of 4 MMAs (K = 64)
    // and the commits.  The k-stages of one weight slot are unrolled per tier.
    Ring ra, rb;
    int count = 0;
    const uint64_t bdesc0 = smem_desc_sw128(sB);
    for (int item = blockIdx.x, li = 0; item < n_items && !aborted(); item += gridDim.x, ++li) {
      Item it;
      if (!decode_item<MT>(p, items_tab, li, item, n_tiles, it)) continue;
      const int ab = count & 1;
      const uint32_t acc_phase = (count >> 1) & 1;
      ++count;
      if (!__all_sync(0xffffffffu, mbar_wait(Acc_empty(ab), acc_phase ^ 1, p.status))) {
        do_abort();
        break;
      }
      tc_fence_after();
      MmaItem mi;
      mi.d = tmem + ab * MT;
      mi.idesc = idesc_f16_m128(it.n);
      mi.nk = p.pj[it.prj].k / kKS;
      mi.per_slot = it.per_slot;
      // rows of one B stage x 128 B, in 16 B units
      mi.stage_desc = static_cast<uint32_t>(MT == kWideN ? kWideN : it.n) * 8u;
      mi.bdesc0 = bdesc0;
      mi.bar_bfull = B_full(0);
      mi.bar_bempty = B_empty(0);
      mi.status = p.status;
      bool ok = true;
      int sidx = 0;
      const int sps = it.sps;
      for (int kc0 = 0; kc0 < mi.nk; kc0 += sps) {
        if (!__all_sync(0xffffffffu, mbar_wait(A_full(ra.idx), ra.phase, p.status))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t abuf = tmem + kTmemA + ra.idx * kACols;
        if (sps == 4) ok = mma_slot<4>(mi, abuf, kc0, rb, sidx);
        else if (sps == 2) ok = mma_slot<2>(mi, abuf, kc0, rb, sidx);
        else ok = mma_slot<1>(mi, abuf, kc0, rb, sidx);
        if (!ok) break;
        if (elect_one()) tc_commit(A_empty(ra.idx));
        __syncwarp();
        ra.next(NG);
      }
      if (!ok) {
        do_abort();
        break;
      }
      if (elect_one()) tc_commit(Acc_full(ab));
      __syncwarp();
    }
  } else if (warp < kDqWarp0) {
    // ---------------------------------------------------------- epilogue
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
    const int row = 32 * quarter + lane;
    const int et = static_cast<int>(threadIdx.x) - 32 * kEpiWarp0;  // 0..127
    int count = 0;
    // The four warps take every decision together (the named barriers below
    // need all 128 threads): the loop bound and the abort test are agreed at
    // the barrier after each accumulator wait.
    for (int item = blockIdx.x, li = 0; item < n_items; item += gridDim.x, ++li, ++count) {
      Item it;
      if (!decode_item<MT>(p, items_tab, li, item, n_tiles, it)) {
        --count;
        continue;
      }
      const ProjParams& pj = p.pj[it.prj];
      const int ab = count & 1;
      const uint32_t acc_phase = (count >> 1) & 1;
      const bool got = !aborted() && mbar_wait(Acc_full(ab), acc_phase, p.status);
      if (named_barrier_or(kEpiBar, 128, !got)) {
        do_abort();
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem + (static_cast<uint32_t>(32 * quarter) << 16) + ab * MT;
      if (pj.gate_up) {
        // rows in blocks of 8: gate rows have bit 3 clear, the matching up row is row ^ 8
        const int g = it.r0 + ((row >> 4) << 3) + (row & 7);
        const bool is_up = (row & 8) != 0;
        float sg = 1.f, su = 1.f;
        if (it.tier == kTierINT8) {
          const int64_t rb = static_cast<int64_t>(it.idx) * pj.n_rows;
          sg = __half2float(pj.s8[rb + g]);
          su = __half2float(pj.s8[rb + p.inter + g]);
        }
        __half* mid = static_cast<__half*>(pj.out);
        const int col = perm_pos(g);
        // mid is stage-major [I/64][n_pos][64]: column col of row m0 + tok
        __half* mrow = mid + static_cast<int64_t>(col >> 6) * p.n_pos * 64 + (col & 63) +
                       static_cast<int64_t>(it.m0) * 64;
        for (int c = 0; c < it.n; c += 16) {
          uint32_t v[16];
          tmem_ld16(taddr + c, v);
          tmem_wait_ld();
          // gate lanes finish tokens c..c+7, up lanes c+8..c+15: each lane sends
          // its partner (lane ^ 8) the value the partner is missing
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float lo = __uint_as_float(v[i]), hi = __uint_as_float(v[8 + i]);
            const float recv = __shfl_xor_sync(0xffffffffu, is_up ? lo : hi, 8);
            const float gate = (is_up ? recv : lo) * sg;
            const float up = (is_up ? hi : recv) * su;
            const int tok = c + i + (is_up ? 8 : 0);
            if (tok < it.mc)
              mrow[static_cast<int64_t>(tok) * 64] =
                  __float2half_rn(__fdividef(gate, 1.0f + __expf(-gate)) * up);
          }
        }
      } else {
        const int h = it.r0 + row;
        float* prow = static_cast<float*>(pj.out) + static_cast<int64_t>(it.m0) * pj.out_stride + h;
        // the router weights are applied by the combine; INT8 rows carry a scale
        const float s = it.tier == kTierINT8
                            ? __half2float(pj.s8[static_cast<int64_t>(it.idx) * pj.n_rows + h])
                            : 1.f;
        for (int c = 0; c < it.n; c += 16) {
          uint32_t v[16];
          tmem_ld16(taddr + c, v);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int tok = c + i;
            if (tok < it.mc) prow[static_cast<int64_t>(tok) * pj.out_stride] = __uint_as_float(v[i]) * s;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(Acc_empty(ab));
      if (pj.gate_up && p.link) {
        // this row block of the tile's mid rows is stored: count it for the
        // down items of the tile (their TMA loads read mid)
        fence_proxy_async_global();
        named_barrier(kEpiBar, 128);
        if (et == 0) {
          __threadfence();
          atomicAdd(p.tile_done + it.tile, 1);
        }
      }
    }
    if (p.fuse_combine) {
      // every partial row of this CTA's items is stored: count the CTA.  The
      // routing kernel zeroes the count, and a CTA without items gets here
      // without having waited for it (its activation producer waits only per
      // item): an add before that zero would be lost and the combine below
      // would wait for a count that never comes.
      named_barrier(kEpiBar, 128);
      if (et == 0) {
        pdl_wait();
        __threadfence();
        atomicAdd(p.dn_done, 1);
      }
    }
  } else if (warp >= kWarpCmb0 && warp < kWarpCmb0 + kNumCmb) {
    // combine warps: nothing during the items (the combine below)
  } else {
    // ---------------------------------------------------------- dequant
    // Group g = (warp - kDqWarp0) / 4 converts weight slots gs = g, g+NG, ...
    // (gs counts slots over all items): ring position gs % 6 and A buffer
    // gs % NG == g.  The warp's lane quarter is warp % 4 (tensor-memory rule).
    // With two groups (128-token items) warps 15-18 have no slots.
    const int grp = (warp - kDqWarp0) >> 2;
    const int m = 32 * (warp & 3) + lane;
    const uint32_t tlane = static_cast<uint32_t>(32 * (warp & 3)) << 16;
    const uint32_t abuf = tmem + tlane + kTmemA + grp * kACols;
    const uint32_t a_empty = A_empty(grp), a_full = A_full(grp);
    uint32_t gs = 0;  // global slot counter of this CTA
    for (int item = blockIdx.x, li = 0; item < n_items && !aborted(); item += gridDim.x, ++li) {
      Item it;
      if (!decode_item<MT>(p, items_tab, li, item, n_tiles, it)) continue;
      const int nk = p.pj[it.prj].k / kKS;
      const int sps = it.sps;
      // gate_up interleaves gate/up rows in blocks of 8 (the epilogue pairs lanes m, m^8)
      const int lw = p.pj[it.prj].gate_up ? (((m >> 4) << 3) + (m & 7) + ((m & 8) ? 64 : 0)) : m;
      const int swz = lw & 7;
      bool ok = true;
      for (int kc0 = 0; kc0 < nk; kc0 += sps, ++gs) {
        if (static_cast<int>(gs % NG) != grp) continue;
        const int ns = min(sps, nk - kc0);
        const uint32_t wi = gs % kWStages, wph = (gs / kWStages) & 1;
        const uint32_t aph = (gs / NG) & 1;
        bool got = mbar_wait(a_empty, aph ^ 1, p.status);
        if (got) got = mbar_wait(W_full(wi), wph, p.status);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        const uint32_t src = sW + wi * kWSlot + lw * 128;  // 128B-swizzled row
        for (int j = 0; j < ns; ++j) {
          uint32_t v[32];
          if (it.tier == kTierINT4) {
            const uint4 w0 = lds128(src + (((2 * j) ^ swz) << 4));
            const uint4 w1 = lds128(src + (((2 * j + 1) ^ swz) << 4));
            const uint16_t sraw = lds16(sS + wi * kSSlot + (j >> 1) * 256 + lw * 2);
            const __half2 s2 = __halves2half2(__ushort_as_half(sraw), __ushort_as_half(sraw));
            dq_int4_word(w0.x, s2, v + 0);
            dq_int4_word(w0.y, s2, v + 4);
            dq_int4_word(w0.z, s2, v + 8);
            dq_int4_word(w0.w, s2, v + 12);
            dq_int4_word(w1.x, s2, v + 16);
            dq_int4_word(w1.y, s2, v + 20);
            dq_int4_word(w1.z, s2, v + 24);
            dq_int4_word(w1.w, s2, v + 28);
          } else if (it.tier == kTierINT8) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const uint4 wv = lds128(src + (((4 * j + c) ^ swz) << 4));
              dq_int8_word(wv.x, v + 8 * c + 0);
              dq_int8_word(wv.y, v + 8 * c + 2);
              dq_int8_word(wv.z, v + 8 * c + 4);
              dq_int8_word(wv.w, v + 8 * c + 6);
            }
          } else {
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const uint4 wv = lds128(src + ((c ^ swz) << 4));
              v[4 * c + 0] = wv.x;
              v[4 * c + 1] = wv.y;
              v[4 * c + 2] = wv.z;
              v[4 * c + 3] = wv.w;
            }
          }
          tmem_st32(abuf + 32 * j, v);
          tmem_wait_st();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(W_empty(wi));
          mbar_arrive(a_full);
        }
      }
      if (!ok) {
        do_abort();
        break;
      }
    }
  }

  if (p.fuse_combine && warp >= kTailWarp0) {
    // ---------------------------------------------------------- top-k combine
    // Once every CTA has stored its items' partial rows, the epilogue,
    // dequant and combine warps of every CTA sum this CTA's share of the
    // tokens: y[t] = sum_j w[t, j] * partial[pos(t, j)], slot order, product
    // and sum rounded separately (a dropped slot adds 0 * w), exactly as
    // combine_partials_kernel.  The slot positions and weights are staged
    // first; warp kWarpCmb0 waits for the count, the others agree at a barrier.
    const int tt = static_cast<int>(threadIdx.x) - 32 * kTailWarp0;
    const int wk = warp - kTailWarp0;
    pdl_wait();  // pos_of_slot and the count's zero come from the routing kernel
    const int spt = p.spt;
    const int n_tok = static_cast<int>(p.n_slots / spt);
    const int tpc = (n_tok + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x);
    const int t0 = min(n_tok, static_cast<int>(blockIdx.x) * tpc), t1 = min(n_tok, t0 + tpc);
    int* spos = reinterpret_cast<int*>(gbase + kOffCmb);  // [tokens of this CTA][spt]
    float* sw = reinterpret_cast<float*>(spos + kCmbEntries);
    for (int i = tt; i < (t1 - t0) * spt; i += 32 * kTailWarps) {
      const int t = t0 + i / spt, j = i - (i / spt) * spt;
      spos[i] = __ldcg(p.pos_of_slot + static_cast<int64_t>(t) * spt + j);
      sw[i] = j < p.top_k ? load_as_f32(p.topk_w, p.w_dtype, static_cast<int64_t>(t) * p.top_k + j)
                          : 1.0f;
    }
    bool ok = true;
    if (warp == kWarpCmb0) {
      if (lane == 0) ok = wait_progress(p.dn_done, static_cast<int>(gridDim.x), p.status);
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    if (!named_barrier_or(kTailBar, 32 * kTailWarps, !ok || aborted())) {
      int seen;  // the other CTAs' partial rows (their counts were acquired above)
      asm volatile("ld.acquire.gpu.global.b32 %0, [%1];\n" : "=r"(seen) : "l"(p.dn_done) : "memory");
      (void)seen;
      const int nhb = static_cast<int>(p.hidden >> 7);
      const float* part = static_cast<const float*>(p.pj[1].out);
      const int64_t stride = p.pj[1].out_stride;
      for (int q = wk; q < (t1 - t0) * nhb; q += kTailWarps) {
        const int tl = q / nhb, col = (q - tl * nhb) * 128 + 4 * lane;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j0 = 0; j0 < spt; j0 += 8) {
          float4 v[8];
          float wj[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int j = j0 + u;
            const int r = j < spt ? spos[tl * spt + j] : -1;
            wj[u] = j < spt ? sw[tl * spt + j] : 0.f;
            v[u] = r >= 0 ? __ldcg(reinterpret_cast<const float4*>(part + r * stride + col))
                          : make_float4(0.f, 0.f, 0.f, 0.f);
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            acc.x = __fadd_rn(acc.x, __fmul_rn(wj[u], v[u].x));
            acc.y = __fadd_rn(acc.y, __fmul_rn(wj[u], v[u].y));
            acc.z = __fadd_rn(acc.z, __fmul_rn(wj[u], v[u].z));
            acc.w = __fadd_rn(acc.w, __fmul_rn(wj[u], v[u].w));
          }
        }
        const int64_t yo = static_cast<int64_t>(t0 + tl) * p.hidden + col;
        uint2 packed;
        if (p.y_dtype == EXQ_F16) {
          __half2 lo = __floats2half2_rn(acc.x, acc.y), hi = __floats2half2_rn(acc.z, acc.w);
          packed = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
        } else {
          __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y),
                         hi = __floats2bfloat162_rn(acc.z, acc.w);
          packed = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
        }
        *reinterpret_cast<uint2*>(static_cast<__half*>(p.y) + yo) = packed;
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
// k permuted to [0,4,1,5,2,6,3,7].  Positions at or past *routed_total + mt
// are read by no GEMM tile and are left alone (the grid is sized for all
// positions, but only that many rows are live: an expert-parallel receive
// area is mostly padding).  Blocks take kPrepRows rows at a time, threads the
// 16-byte chunks of a row; a thread's loads of the kPrepRows rows are in
// flight together.
constexpr int kPrepRows = 4;
constexpr int kPrepThreads = 256;

template <typename T>
__device__ __forceinline__ uint4 prep_octet(uint4 v) {
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
  return r;
}

template <typename T>
__global__ void __launch_bounds__(kPrepThreads) prep_act_kernel(
    const T* __restrict__ hidden, int64_t hid, int64_t n_tokens, const int32_t* sorted_slot,
    int spt, int64_t n_pos, const int32_t* routed_total, int mt, __half* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int octs = static_cast<int>(hid / 8);
  const int lim = static_cast<int>(min(n_pos, static_cast<int64_t>(*routed_total) + mt));
  uint4* dst = reinterpret_cast<uint4*>(out);
  for (int r0 = blockIdx.x * kPrepRows; r0 < lim; r0 += gridDim.x * kPrepRows) {
    const uint4* src[kPrepRows];
#pragma unroll
    for (int u = 0; u < kPrepRows; ++u) {
      const int pos = r0 + u;
      const int32_t slot = pos < lim ? sorted_slot[pos] : -1;
      const int tok = slot >= 0 ? slot / spt : -1;  // slot < 0: a dropped slot (zero row)
      src[u] = tok >= 0 && tok < n_tokens
                   ? reinterpret_cast<const uint4*>(hidden + static_cast<int64_t>(tok) * hid)
                   : nullptr;
    }
    for (int o = threadIdx.x; o < octs; o += kPrepThreads) {
      uint4 v[kPrepRows];
#pragma unroll
      for (int u = 0; u < kPrepRows; ++u) v[u] = src[u] ? __ldg(src[u] + o) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int u = 0; u < kPrepRows; ++u) {
        const int pos = r0 + u;
        if (pos >= lim) break;
        // stage-major [hid / 64][n_pos][64]
        dst[((static_cast<int64_t>(o) >> 3) * n_pos + pos) * 8 + (o & 7)] =
            src[u] ? prep_octet<T>(v[u]) : make_uint4(0, 0, 0, 0);
      }
    }
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

static bool make_map_nd(CUtensorMap* m, CUtensorMapDataType dt, const void* ptr, int rank,
                        const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                        CUtensorMapSwizzle sw, CUtensorMapL2promotion l2) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is unavailable from the driver");
    return false;
  }
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) st[i] = strides_bytes[i];
  }
  CUresult r = fn(m, dt, rank, const_cast<void*>(ptr), d, st, b, e,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, l2, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) for a rank-%d tensor", (int)r, rank);
    return false;
  }
  return true;
}

// Fill the per-projection maps.  proj 0 = w13 (rows 2I, k = H), 1 = w2 (rows H, k = I).
static int build_maps(const exq_moe_weights* w, int proj, const void* act, int64_t n_pos,
                      int mt, ProjParams& p) {
  const int64_t I = w->inter, H = w->hidden;
  const int64_t rows = proj == 0 ? 2 * I : H;
  const int64_t k = proj == 0 ? H : I;
  const int64_t G = k / 128;
  memset(p.tm_w, 0, sizeof(p.tm_w));
  memset(&p.tm_s, 0, sizeof(p.tm_s));
  const int n4 = w->n_tier[EXQ_TIER_INT4], n8 = w->n_tier[EXQ_TIER_INT8],
            n16 = w->n_tier[EXQ_TIER_BF16];
  const void* const* wt = proj == 0 ? w->w13 : w->w2;
  const void* const* st = proj == 0 ? w->w13_scales : w->w2_scales;
  const auto L2W = CU_TENSOR_MAP_L2_PROMOTION_L2_256B;
  const auto SW = CU_TENSOR_MAP_SWIZZLE_128B;
  // One 16 KB slot = 128 weight rows x 128 bytes (INT4 256 k, INT8 128 k, 16-bit 64 k).
  // gate_up views the [n, 2I, row_bytes] storage as (x, row in 64-row block, block,
  // gate/up, expert) so one box holds 64 gate rows and the matching 64 up rows.
  for (int t = 0; t < 3; ++t) {
    const int n = w->n_tier[t];
    if (n <= 0) continue;
    const CUtensorMapDataType dt =
        t == EXQ_TIER_BF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
    const uint64_t esz = t == EXQ_TIER_BF16 ? 2 : 1;
    const uint64_t xdim = t == EXQ_TIER_INT4 ? k / 2 : k;  // elements per row
    const uint64_t rb = xdim * esz;                          // bytes per row
    const uint32_t box_x = static_cast<uint32_t>(128 / esz);
    bool ok;
    if (proj == 0) {
      const uint64_t d[5] = {xdim, 64, (uint64_t)(I / 64), 2, (uint64_t)n};
      const uint64_t st5[4] = {rb, 64 * rb, (uint64_t)I * rb, 2 * (uint64_t)I * rb};
      const uint32_t b[5] = {box_x, 64, 1, 2, 1};
      ok = make_map_nd(&p.tm_w[t], dt, wt[t], 5, d, st5, b, SW, L2W);
    } else {
      ok = make_map(&p.tm_w[t], dt, wt[t], xdim, (uint64_t)n * rows, rb, box_x, 128, SW, L2W);
    }
    if (!ok) return EXQ_ERR_CUDA;
  }
  if (n4 > 0) {
    bool ok;
    if (proj == 0) {
      // scales [n4, G, 2I] as (element in block, block, gate/up, group, expert); 2 groups
      const uint64_t ds[5] = {64, (uint64_t)(I / 64), 2, (uint64_t)G, (uint64_t)n4};
      const uint64_t ss[4] = {128, (uint64_t)(2 * I), (uint64_t)(4 * I), (uint64_t)(4 * I * G)};
      const uint32_t bs[5] = {64, 1, 2, 2, 1};
      ok = make_map_nd(&p.tm_s, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, st[EXQ_TIER_INT4], 5, ds, ss, bs,
                       CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B);
    } else {
      ok = make_map(&p.tm_s, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, st[EXQ_TIER_INT4], rows,
                    (uint64_t)n4 * G, rows * 2, 128, 2, CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_128B);
    }
    if (!ok) return EXQ_ERR_CUDA;
  }
  (void)n8;
  (void)n16;
  // activations stage-major [k/64][n_pos][64]: (element, row, stage); map b has a
  // box of N = 16(b+1) rows x the stages of one B slot (64-token items), or
  // one map of 128 rows x 2 stages (128-token items)
  for (int b = 0; b < (mt == kWideN ? 1 : 4); ++b) {
    const uint32_t nb = mt == kWideN ? kWideN : 16u * (b + 1);
    const uint64_t d[3] = {64, (uint64_t)n_pos, (uint64_t)(k / 64)};
    const uint64_t s3[2] = {128, (uint64_t)n_pos * 128};
    const uint32_t bx[3] = {64, nb, (uint32_t)b_slot_stages(mt, (int)nb)};
    if (!make_map_nd(&p.tm_b[b], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, act, 3, d, s3, bx,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B))
      return EXQ_ERR_CUDA;
  }
  p.s8 = static_cast<const __half*>(st[EXQ_TIER_INT8]);
  p.n_rows = static_cast<int>(rows);
  p.k = static_cast<int>(k);
  return EXQ_OK;
}

int launch_tc(const TcParams& p, int mt, int max_items, cudaStream_t stream, bool pdl) {
  static int attr_done[2][64] = {{0}};
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  const int wide = mt == kWideN;
  if (!attr_done[wide][dev]) {
    cudaError_t e = cudaFuncSetAttribute(wide ? moe_tc_kernel<kWideN> : moe_tc_kernel<kMaxN>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) {
      set_error("moe_tc_kernel: cannot reserve %d B of shared memory: %s", kSmemBytes,
                cudaGetErrorString(e));
      return EXQ_ERR_CUDA;
    }
    sms[dev] = num_sms();
    attr_done[wide][dev] = 1;
  }
  int grid = sms[dev];
  if (max_items < grid) grid = max_items;
  if (grid < 1) grid = 1;
  const cudaError_t e =
      wide ? launch_pdl(pdl, moe_tc_kernel<kWideN>, dim3(grid), dim3(kThreads), kSmemBytes, stream, p)
           : launch_pdl(pdl, moe_tc_kernel<kMaxN>, dim3(grid), dim3(kThreads), kSmemBytes, stream, p);
  if (e != cudaSuccess) {
    set_error("moe_tc_kernel: %s", cudaGetErrorString(e));
    return EXQ_ERR_CUDA;
  }
  EXQ_CHECK_LAUNCH("moe_tc_kernel");
  return EXQ_OK;
}

int launch_prep(const void* hidden, int act_dtype, int64_t hid, int64_t n_tokens,
                const int32_t* sorted_slot, int spt, int64_t n_pos, const int32_t* routed_total,
                int mt, __half* out, cudaStream_t stream, bool pdl) {
  if (n_pos == 0) return EXQ_OK;
  // row groups, at most eight blocks per SM (grid-stride beyond)
  int64_t grid = (n_pos + kPrepRows - 1) / kPrepRows;
  if (grid > 8 * num_sms()) grid = 8 * num_sms();
  cudaError_t e;
  if (act_dtype == EXQ_F16)
    e = launch_pdl(pdl, prep_act_kernel<__half>, dim3((int)grid), dim3(kPrepThreads), 0, stream,
                   static_cast<const __half*>(hidden), hid, n_tokens, sorted_slot, spt, n_pos,
                   routed_total, mt, out);
  else
    e = launch_pdl(pdl, prep_act_kernel<__nv_bfloat16>, dim3((int)grid), dim3(kPrepThreads), 0,
                   stream,
                   static_cast<const __nv_bfloat16*>(hidden), hid, n_tokens, sorted_slot, spt, n_pos,
                   routed_total, mt, out);
  if (e != cudaSuccess) {
    set_error("prep_act_kernel: %s", cudaGetErrorString(e));
    return EXQ_ERR_CUDA;
  }
  EXQ_CHECK_LAUNCH("prep_act_kernel");
  return EXQ_OK;
}

}  // namespace tc
}  // namespace exq

// ============================================================== C ABI
using namespace exq;

namespace {

// Tokens per GEMM tile (the MMA's N): 128 when the call averages at least 128
// rows per expert bucket (prefill, expert-parallel receive areas, large decode
// batches), which halves how often an expert's weights are streamed and
// converted; else 64, the decode build (at 64 rows per expert the 128-token
// build is slower: Mixtral T=256 359 against 344 us; at 128 it is faster: T=512
// 523 against 557 us).
int layer_mt(int64_t n_slots, int64_t n_buckets) {
  return n_buckets > 0 && n_slots >= 128 * n_buckets ? tc::kWideN : tc::kMaxN;
}

struct TcWs {
  int32_t* sorted_slot;
  int32_t* pos_of_slot;
  float* sorted_w;
  int32_t* ends;
  int32_t* tile_info;
  int32_t* n_tiles;
  int32_t* tile_done;  // [max_tiles] gate_up row blocks stored per tile, then the count of
                       // CTAs whose items are all stored (zeroed by the route stage)
  __half* act;
  __half* mid;
  float* partial;
  int64_t max_tiles;
  int mt;              // tokens per GEMM tile
  int64_t n_counters;  // ints from tile_done on (one contiguous run)
  size_t bytes;
};

TcWs carve_tc(void* base, int64_t n_slots, int64_t n_tokens, int n_buckets, int64_t hidden,
              int64_t inter) {
  TcWs w{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 256);
    return base ? static_cast<char*>(base) + o : nullptr;
  };
  w.mt = layer_mt(n_slots, n_buckets);
  w.max_tiles = n_slots / w.mt + (n_slots < n_buckets ? n_slots : n_buckets) + 1;
  w.sorted_slot = reinterpret_cast<int32_t*>(take(4 * n_slots));
  w.pos_of_slot = reinterpret_cast<int32_t*>(take(4 * n_slots));
  w.sorted_w = reinterpret_cast<float*>(take(4 * n_slots));
  w.ends = reinterpret_cast<int32_t*>(take(4 * (n_buckets + 1)));
  w.tile_info = reinterpret_cast<int32_t*>(take(12 * w.max_tiles));
  w.n_tiles = reinterpret_cast<int32_t*>(take(16));
  (void)n_tokens;
  w.n_counters = w.max_tiles + 1;
  w.tile_done = reinterpret_cast<int32_t*>(take(4 * w.n_counters));
  w.act = reinterpret_cast<__half*>(take(2 * n_slots * hidden));
  w.mid = reinterpret_cast<__half*>(take(2 * n_slots * inter));
  w.partial = reinterpret_cast<float*>(take(4 * n_slots * hidden));
  w.bytes = off;
  return w;
}

bool is_act(int d) { return d == EXQ_F16 || d == EXQ_BF16; }

}  // namespace

void exq::layer_partials(void* workspace, int64_t n_slots, int64_t n_tokens, int n_buckets,
                         int64_t hidden, int64_t inter, const float** partial,
                         const int32_t** pos_of_slot) {
  const TcWs ws = carve_tc(workspace, n_slots, n_tokens, n_buckets, hidden, inter);
  *partial = ws.partial;
  *pos_of_slot = ws.pos_of_slot;
}

extern "C" size_t exq_moe_layer_workspace_bytes(int64_t n_tokens, int32_t top_k, int32_t n_shared,
                                                int32_t n_experts_total, int64_t hidden,
                                                int64_t inter) {
  if (n_tokens < 0 || top_k <= 0 || n_shared < 0 || n_experts_total <= 0) return 0;
  return carve_tc(nullptr, n_tokens * (top_k + n_shared), n_tokens, n_experts_total, hidden, inter)
      .bytes;
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

// The layer's stages [first_stage, end_stage).  chained_start: the call's
// first launch may be programmatic, because the kernel before it on the
// stream is this library's router (which lets it launch early and completes
// before the routing kernel reads the ids).
static int layer_forward(const exq_moe_weights* w, const void* hidden_states, int act_dtype,
                         int64_t n_tokens, const void* topk_ids, int ids_dtype,
                         const void* topk_weights, int w_dtype, int32_t top_k, void* out,
                         void* workspace, size_t workspace_bytes, void* stream,
                         int32_t first_stage, int32_t end_stage, bool chained_start) {
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
  TcWs ws = carve_tc(workspace, n_slots, n_tokens, n_total, H, I);
  uint32_t* status = device_status_ptr();
  if (!status) return EXQ_ERR_CUDA;
  int st = EXQ_OK;
  // Launch programmatically (overlapping the previous kernel's tail) only after
  // a kernel of this call or the router: the first launch may otherwise follow
  // a copy or an event wait.
  bool chained = chained_start;

  // gate_up and down run as one launch when both are asked for; with the
  // combine too, the down items sum each token's slots (no separate combine)
  const bool do_gu = first_stage <= 2 && end_stage > 2;
  const bool do_dn = first_stage <= 3 && end_stage > 3;
  // decode-sized calls route and gather in one kernel (stage 0; stage 1 is empty)
  const bool fused = n_total <= kRouteGatherMaxBuckets &&
                     (n_slots <= kRouteGatherMaxSlots ||
                      (n_slots <= kRouteGatherFusedMaxSlots &&
                       n_slots <= kRouteGatherFusedMaxRowsPerBucket * n_total));
  // decode-sized calls: the GEMM launch also does the combine (its CTAs split
  // the tokens once every item is stored); larger ones launch it apart
  const bool fuse_combine = do_dn && first_stage <= 4 && end_stage > 4 && fused &&
                            spt <= tc::kCmbMaxSpt &&
                            ((n_tokens + num_sms() - 1) / num_sms() + 1) * spt <= tc::kCmbEntries;
  if (fused && first_stage <= 0 && end_stage > 0) {
    RouteGatherParams rg{};
    rg.ids = topk_ids;
    rg.ids_dtype = ids_dtype;
    rg.topk_w = topk_weights;
    rg.w_dtype = w_dtype;
    rg.hidden = hidden_states;
    rg.act_dtype = act_dtype;
    rg.hidden_size = H;
    rg.top_k = top_k;
    rg.spt = spt;
    rg.n_routed = w->n_routed;
    rg.n_buckets = n_total;
    rg.mt = ws.mt;
    rg.n = n_slots;
    rg.act = ws.act;
    rg.pos_of_slot = ws.pos_of_slot;
    rg.sorted_w = ws.sorted_w;
    rg.ends = ws.ends;
    rg.tile_info = ws.tile_info;
    rg.n_tiles = ws.n_tiles;
    rg.max_tiles = ws.max_tiles;
    rg.sorted_slot = ws.sorted_slot;
    rg.counters = ws.tile_done;
    rg.n_counters = ws.n_counters;
    st = launch_route_gather(rg, s, chained);
    if (st != EXQ_OK) return st;
    chained = true;
  }
  if (!fused && first_stage <= 0 && end_stage > 0) {
    RouteParams rp{};
    rp.ids = topk_ids;
    rp.ids_dtype = ids_dtype;
    rp.n = n_slots;
    rp.n_buckets = n_total;
    rp.n_routed = w->n_routed;
    rp.top_k = top_k;
    rp.slots_per_token = spt;
    rp.mt = ws.mt;
    rp.sorted_i32 = ws.sorted_slot;
    rp.pos_of_slot = ws.pos_of_slot;
    rp.sorted_w = ws.sorted_w;
    rp.topk_w = topk_weights;
    rp.w_dtype = w_dtype;
    rp.ends = ws.ends;
    rp.tile_info = ws.tile_info;
    rp.n_tiles = ws.n_tiles;
    rp.max_tiles = ws.max_tiles;
    rp.counters = ws.tile_done;
    rp.n_counters = ws.n_counters;
    st = launch_route(rp, kRouteLayer, s, chained);
    if (st != EXQ_OK) return st;
    chained = true;
  }
  if (!fused && first_stage <= 1 && end_stage > 1) {
    st = tc::launch_prep(hidden_states, act_dtype, H, n_tokens, ws.sorted_slot, spt, n_slots,
                         ws.ends + n_total, ws.mt, ws.act, s, chained);
    if (st != EXQ_OK) return st;
    chained = true;
  }
  if (do_gu || do_dn) {
    tc::TcParams p;
    memset(&p, 0, sizeof(p));
    for (int proj = 0; proj < 2; ++proj) {
      if (!(proj == 0 ? do_gu : do_dn)) continue;
      tc::ProjParams& pj = p.pj[proj];
      st = tc::build_maps(w, proj, proj == 0 ? ws.act : ws.mid, n_slots, ws.mt, pj);
      if (st != EXQ_OK) return st;
      pj.gate_up = proj == 0;
      pj.nblocks = static_cast<int>(proj == 0 ? I / 64 : H / 128);
      pj.out = proj == 0 ? static_cast<void*>(ws.mid) : static_cast<void*>(ws.partial);
      pj.out_stride = proj == 0 ? I : H;
    }
    p.run_gu = do_gu;
    p.run_dn = do_dn;
    p.link = do_gu && do_dn;
    p.tile_done = ws.tile_done;
    p.fuse_combine = fuse_combine;
    p.dn_done = ws.tile_done + ws.max_tiles;
    p.sorted_slot = ws.sorted_slot;
    p.pos_of_slot = ws.pos_of_slot;
    p.topk_w = topk_weights;
    p.w_dtype = w_dtype;
    p.y = out;
    p.y_dtype = act_dtype;
    p.hidden = H;
    p.expert_slot = w->expert_slot;
    p.tile_info = ws.tile_info;
    p.n_tiles_ptr = ws.n_tiles;
    p.max_tiles = static_cast<int>(ws.max_tiles);
    p.inter = static_cast<int>(I);
    p.n_pos = n_slots;
    p.status = status;
    const int64_t per_tile = (do_gu ? I / 64 : 0) + (do_dn ? H / 128 : 0);
    const int64_t max_items = ws.max_tiles * per_tile;
    const int64_t grid = max_items < num_sms() ? max_items : num_sms();
    // a CTA can build its items from the ids: the experts fit the histogram and
    // every CTA's items fit its shared table
    const bool ids_ok = n_total <= tc::kHistBuckets &&
                        max_items <= static_cast<int64_t>(tc::kItemTab) * (grid > 0 ? grid : 1);
    if (fused && first_stage == 0) {
      // right after the fused routing of this call: build the tiles from the
      // ids (complete before routing started) and stream weights at once;
      // otherwise wait for the routing kernel before reading its tile list
      p.tiles_from_ids = ids_ok;
    } else {
      // the tile list was complete before this launch could start: written by
      // the route kernel two launches back (route -> prep -> here) or by an
      // earlier call
      p.weights_early = 1;
    }
    p.ids = topk_ids;
    p.ids_dtype = ids_dtype;
    p.top_k = top_k;
    p.spt = spt;
    p.n_routed = w->n_routed;
    p.n_buckets = n_total;
    p.n_slots = n_slots;
    st = tc::launch_tc(p, ws.mt, static_cast<int>(max_items < INT32_MAX ? max_items : INT32_MAX), s,
                       chained);
    if (st != EXQ_OK) return st;
    chained = true;
  }
  if (first_stage <= 4 && end_stage > 4 && !fuse_combine)
    return launch_combine_partials(ws.partial, H, ws.pos_of_slot, topk_weights, w_dtype, top_k,
                                   n_tokens, spt, out, act_dtype, s, chained);
  return EXQ_OK;
}

extern "C" int exq_moe_layer_forward_range(const exq_moe_weights* w, const void* hidden_states,
                                           int act_dtype, int64_t n_tokens, const void* topk_ids,
                                           int ids_dtype, const void* topk_weights, int w_dtype,
                                           int32_t top_k, void* out, void* workspace,
                                           size_t workspace_bytes, void* stream,
                                           int32_t first_stage, int32_t end_stage) {
  return layer_forward(w, hidden_states, act_dtype, n_tokens, topk_ids, ids_dtype, topk_weights,
                       w_dtype, top_k, out, workspace, workspace_bytes, stream, first_stage,
                       end_stage, false);
}

extern "C" size_t exq_moe_layer_from_logits_workspace_bytes(int64_t n_tokens, int32_t top_k,
                                                            int32_t n_shared,
                                                            int32_t n_experts_total,
                                                            int64_t hidden, int64_t inter) {
  const size_t layer = exq_moe_layer_workspace_bytes(n_tokens, top_k, n_shared, n_experts_total,
                                                     hidden, inter);
  if (layer == 0 && n_tokens > 0) return 0;
  return align_up(layer, 256) + 2 * align_up(static_cast<size_t>(n_tokens) * top_k * 4, 256);
}

extern "C" int exq_moe_layer_forward_from_logits(const exq_moe_weights* w,
                                                 const void* hidden_states, int act_dtype,
                                                 int64_t n_tokens, const void* router_logits,
                                                 int logits_dtype, int32_t top_k,
                                                 int32_t renormalize, void* out, void* workspace,
                                                 size_t workspace_bytes, void* stream) {
  EXQ_CHECK_ARG(w, "moe_layer: weights is null");
  const int st = check_router_args(logits_dtype, n_tokens, w->n_routed, top_k);
  if (st != EXQ_OK) return st;
  const size_t need = exq_moe_layer_from_logits_workspace_bytes(
      n_tokens, top_k, w->n_shared, w->n_routed + w->n_shared, w->hidden, w->inter);
  if (!workspace || workspace_bytes < need) {
    set_error("moe_layer_from_logits: workspace of %zu bytes needed", need);
    return EXQ_ERR_WORKSPACE;
  }
  if (n_tokens == 0) return EXQ_OK;
  EXQ_CHECK_ARG(router_logits, "moe_layer_from_logits: router_logits is null");
  // the router's ids and weights after the layer's own workspace
  const size_t layer = align_up(exq_moe_layer_workspace_bytes(n_tokens, top_k, w->n_shared,
                                                               w->n_routed + w->n_shared,
                                                               w->hidden, w->inter), 256);
  char* base = static_cast<char*>(workspace);
  int32_t* ids = reinterpret_cast<int32_t*>(base + layer);
  float* wts = reinterpret_cast<float*>(base + layer +
                                        align_up(static_cast<size_t>(n_tokens) * top_k * 4, 256));
  const cudaError_t e = launch_router_topk(router_logits, logits_dtype, n_tokens, w->n_routed,
                                           top_k, renormalize, ids, wts,
                                           static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    set_error("router_topk_kernel: %s", cudaGetErrorString(e));
    return EXQ_ERR_CUDA;
  }
  return layer_forward(w, hidden_states, act_dtype, n_tokens, ids, EXQ_I32, wts, EXQ_F32, top_k,
                       out, workspace, layer, stream, 0, EXQ_LAYER_STAGES, true);
}
