// C ABI glue: error reporting, the device status word, and the two
// multi-kernel entry points (one projection, whole layer).
#include <string.h>

#include "internal.cuh"

namespace exq {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

// Device status word that kernels OR EXQ_DEV_* bits into.
__device__ uint32_t g_device_status;

uint32_t* device_status_ptr() {
  static uint32_t* ptrs[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    set_error("cudaGetDevice failed");
    return nullptr;
  }
  if (!ptrs[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_device_status);
    if (e != cudaSuccess) {
      set_error("cudaGetSymbolAddress(status): %s", cudaGetErrorString(e));
      return nullptr;
    }
    ptrs[dev] = static_cast<uint32_t*>(p);
  }
  return ptrs[dev];
}

}  // namespace exq

using namespace exq;

extern "C" int exq_abi_version(void) { return EXQ_ABI_VERSION; }

extern "C" const char* exq_last_error(void) { return g_err; }

extern "C" const char* exq_status_string(int status) {
  switch (status) {
    case EXQ_OK: return "ok";
    case EXQ_ERR_INVALID: return "invalid argument";
    case EXQ_ERR_UNSUPPORTED: return "unsupported";
    case EXQ_ERR_CUDA: return "CUDA error";
    case EXQ_ERR_WORKSPACE: return "workspace missing or too small";
    default: return "unknown status";
  }
}

extern "C" int exq_read_device_status(uint32_t* status_out, int clear, void* stream) {
  EXQ_CHECK_ARG(status_out, "status_out is null");
  uint32_t* d = device_status_ptr();
  if (!d) return EXQ_ERR_CUDA;
  auto s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(status_out, d, sizeof(uint32_t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess && clear) e = cudaMemsetAsync(d, 0, sizeof(uint32_t), s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    set_error("read_device_status: %s", cudaGetErrorString(e));
    return EXQ_ERR_CUDA;
  }
  return EXQ_OK;
}

namespace {

// Workspace carving shared by the projection and the layer entry points.
struct LayerWs {
  int32_t* sorted_slot;
  int32_t* pos_of_slot;
  int32_t* ends;
  int32_t* tile_info;
  int32_t* n_tiles;
  void* mid;
  float* partial;
  size_t bytes;
};

int64_t max_tiles_for(int64_t n_slots, int n_buckets) {
  return n_slots / kGmMTHost + (n_slots < n_buckets ? n_slots : n_buckets) + 1;
}

LayerWs carve(void* base, int64_t n_slots, int n_buckets, int64_t inter, int64_t hidden,
              bool with_layer_buffers) {
  LayerWs w{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 256);
    return base ? static_cast<char*>(base) + o : nullptr;
  };
  w.sorted_slot = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * n_slots));
  w.pos_of_slot = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * n_slots));
  w.ends = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * (n_buckets + 1)));
  w.tile_info = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * 3 * max_tiles_for(n_slots, n_buckets)));
  w.n_tiles = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * 4));
  if (with_layer_buffers) {
    w.mid = take(2 * static_cast<size_t>(n_slots) * inter);
    w.partial = reinterpret_cast<float*>(take(sizeof(float) * static_cast<size_t>(n_slots) * hidden));
  }
  w.bytes = off;
  return w;
}

bool is_act(int d) { return d == EXQ_F16 || d == EXQ_BF16; }

}  // namespace

extern "C" size_t exq_moe_gemm_workspace_bytes(int64_t n_tokens, int32_t top_k,
                                               int32_t n_experts) {
  if (n_tokens < 0 || top_k <= 0 || n_experts <= 0) return 0;
  return carve(nullptr, n_tokens * top_k, n_experts, 0, 0, false).bytes;
}

extern "C" int exq_moe_gemm(const exq_expert_desc* experts, int32_t n_experts, int64_t n_rows,
                            int64_t k, const void* hidden, int act_dtype, int64_t n_tokens,
                            const void* topk_ids, int ids_dtype, int32_t top_k, void* out,
                            int out_dtype, int64_t* sort_order_out, int32_t* expert_ends_out,
                            void* workspace, size_t workspace_bytes, void* stream) {
  EXQ_CHECK_ARG(is_act(act_dtype), "moe_gemm: activations must be fp16 or bf16");
  EXQ_CHECK_ARG(is_act(out_dtype), "moe_gemm: output must be fp16 or bf16");
  EXQ_CHECK_ARG(ids_dtype == EXQ_I32 || ids_dtype == EXQ_I64, "moe_gemm: ids must be int32/int64");
  EXQ_CHECK_ARG(n_experts > 0 && top_k > 0 && n_tokens >= 0, "moe_gemm: bad sizes");
  EXQ_CHECK_ARG(n_rows > 0 && n_rows % 16 == 0, "moe_gemm: N=%lld must be a positive multiple of 16",
                (long long)n_rows);
  if (k <= 0 || k % 128 != 0) {
    set_error("moe_gemm: K=%lld must be a positive multiple of 128 (group size 128)", (long long)k);
    return EXQ_ERR_UNSUPPORTED;
  }
  EXQ_CHECK_ARG(experts, "moe_gemm: experts is null");
  const int64_t n_slots = n_tokens * top_k;
  const size_t need = exq_moe_gemm_workspace_bytes(n_tokens, top_k, n_experts);
  if (!workspace || workspace_bytes < need) {
    set_error("moe_gemm: workspace of %zu bytes needed", need);
    return EXQ_ERR_WORKSPACE;
  }
  auto s = static_cast<cudaStream_t>(stream);
  LayerWs w = carve(workspace, n_slots, n_experts, 0, 0, false);
  RouteParams rp{};
  rp.ids = topk_ids;
  rp.ids_dtype = ids_dtype;
  rp.n = n_slots;
  rp.n_buckets = n_experts;
  rp.n_routed = n_experts;
  rp.top_k = top_k;
  rp.slots_per_token = top_k;
  rp.mt = kGmMTHost;
  rp.sorted_i32 = w.sorted_slot;
  rp.pos_of_slot = w.pos_of_slot;
  rp.ends = expert_ends_out ? expert_ends_out : w.ends;
  rp.order_i64 = sort_order_out;
  rp.tile_info = w.tile_info;
  rp.n_tiles = w.n_tiles;
  rp.max_tiles = max_tiles_for(n_slots, n_experts);
  int st = launch_route(rp, kRouteLayer, s);
  if (st != EXQ_OK) return st;
  if (n_slots == 0) return EXQ_OK;
  EXQ_CHECK_ARG(hidden && out && topk_ids, "moe_gemm: null pointer");
  GemmParams gp{};
  gp.experts = experts;
  gp.proj = 0;
  gp.mode = kGemmModePlain;
  gp.n_rows = static_cast<int>(n_rows);
  gp.k = static_cast<int>(k);
  gp.nblocks = static_cast<int>((n_rows + kGmRBHost - 1) / kGmRBHost);
  gp.act = hidden;
  gp.act_stride = k;
  gp.gather = 1;
  gp.spt = top_k;
  gp.top_k = top_k;
  gp.sorted_slot = w.sorted_slot;
  gp.tile_info = w.tile_info;
  gp.n_tiles_ptr = w.n_tiles;
  gp.max_tiles = static_cast<int>(rp.max_tiles);
  gp.out = out;
  gp.out_dtype = out_dtype;
  gp.out_stride = n_rows;
  gp.status = device_status_ptr();
  const int64_t max_items = rp.max_tiles * gp.nblocks;
  return launch_gemm(gp, act_dtype, static_cast<int>(max_items < INT32_MAX ? max_items : INT32_MAX), s);
}

