// The C ABI of include/wmoe.h: argument checks, scratch planning and the order of launches. Kernels live in
// dequant.cu, route.cu, dispatch.cu, gemv.cu, decode.cu and store.cu.
#include <dlfcn.h>

#include <atomic>
#include <chrono>
#include <cstdlib>
#include <memory>
#include <cstring>
#include <thread>
#include <nccl.h>

#include <algorithm>
#include <string>
#include <vector>

#include "../../include/wmoe.h"
#include "common.cuh"
#include "kernels.cuh"
#include "store.h"

#include <cstddef>

// wmoe_decode_stack hands the caller's wmoe_layer_weights array to the kernels as DecodeLayer: same layout
static_assert(sizeof(wmoe_layer_weights) == sizeof(wmoe::DecodeLayer), "layer weight layouts differ");
static_assert(offsetof(wmoe_layer_weights, router_packed) == offsetof(wmoe::DecodeLayer, router_packed) &&
                  offsetof(wmoe_layer_weights, router_split) == offsetof(wmoe::DecodeLayer, router_split),
              "layer weight layouts differ");

using namespace wmoe;

int ctx_fail(wmoe_ctx* ctx, int code, const std::string& msg) {
  if (ctx) ctx->error = msg;
  return code;
}

void ctx_count_launch(wmoe_ctx* ctx, int n) {
  if (ctx) ctx->launches += uint64_t(n);
}

static int cuda_fail(wmoe_ctx* ctx, cudaError_t e, const char* where) {
  return ctx_fail(ctx, WMOE_ERR_CUDA, std::string(where) + ": " + cudaGetErrorString(e));
}

#define WMOE_CHECK_CUDA(ctx, expr, where)              \
  do {                                                 \
    const cudaError_t e_ = (expr);                     \
    if (e_ != cudaSuccess) return cuda_fail(ctx, e_, where); \
  } while (0)

// Bump allocator over the context's scratch buffer (256-byte aligned pieces).
struct Plan {
  size_t bytes = 0;
  template <typename T>
  size_t take(size_t count) {
    const size_t off = bytes;
    bytes += (count * sizeof(T) + 255) / 256 * 256;
    return off;
  }
};

static int ensure_scratch(wmoe_ctx* ctx, size_t bytes) {
  if (bytes <= ctx->scratch_bytes) return WMOE_OK;
  if (ctx->scratch) {
    WMOE_CHECK_CUDA(ctx, cudaDeviceSynchronize(), "scratch resize");
    cudaFree(ctx->scratch);
    ctx->scratch = nullptr;
    ctx->scratch_bytes = 0;
  }
  const size_t grown = std::max(bytes, size_t(1) << 20);
  WMOE_CHECK_CUDA(ctx, cudaMalloc(&ctx->scratch, grown), "scratch allocation");
  ctx->scratch_bytes = grown;
  return WMOE_OK;
}

template <typename T>
static T* at(wmoe_ctx* ctx, size_t off) {
  return reinterpret_cast<T*>(static_cast<char*>(ctx->scratch) + off);
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

extern "C" {

int wmoe_init(int device, wmoe_ctx** out) {
  if (!out) return WMOE_ERR_INVALID;
  *out = nullptr;
  auto* ctx = new wmoe_ctx();
  ctx->device = device;
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&ctx->sm_count, cudaDevAttrMultiProcessorCount, device);
  if (e == cudaSuccess) e = cudaMalloc(&ctx->d_status, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(ctx->d_status, 0, sizeof(int));
  if (e != cudaSuccess) {
    delete ctx;
    return WMOE_ERR_CUDA;
  }
  ctx->decode_ctas = decode_num_ctas(device);
  *out = ctx;
  return WMOE_OK;
}

static void free_profiling(wmoe_ctx* ctx);
static void ep_release(wmoe_ctx* ctx);

void wmoe_destroy(wmoe_ctx* ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->device);
  cudaDeviceSynchronize();
  free_profiling(ctx);
  ep_release(ctx);
  cudaFree(ctx->scratch);
  cudaFree(ctx->stack_xn);
  cudaFree(ctx->stage_dev);
  cudaFreeHost(ctx->stage_host);
  for (cudaEvent_t ev : ctx->stage_ev)
    if (ev) cudaEventDestroy(ev);
  cudaFree(ctx->d_status);
  delete ctx;
}

const char* wmoe_last_error(const wmoe_ctx* ctx) { return ctx ? ctx->error.c_str() : "null context"; }

uint64_t wmoe_launch_count(const wmoe_ctx* ctx) { return ctx ? ctx->launches : 0; }

int wmoe_set_trace(wmoe_ctx* ctx, uint64_t* trace, size_t entries) {
  if (!ctx) return WMOE_ERR_INVALID;
  ctx->trace = entries ? trace : nullptr;
  ctx->trace_entries = trace ? entries : 0;
  return WMOE_OK;
}

int wmoe_decode_ctas(const wmoe_ctx* ctx) { return ctx ? ctx->decode_ctas : 0; }

static void free_profiling(wmoe_ctx* ctx) {
  for (cudaEvent_t e : ctx->prof_events) cudaEventDestroy(e);
  ctx->prof_events.clear();
  ctx->profile_calls = 0;
  ctx->profile_seq = 0;
}

int wmoe_set_profiling(wmoe_ctx* ctx, int calls) {
  if (!ctx) return WMOE_ERR_INVALID;
  if (calls < 0 || calls > 100000) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_set_profiling: bad call count");
  cudaSetDevice(ctx->device);
  free_profiling(ctx);
  if (calls == 0) return WMOE_OK;
  ctx->prof_events.resize(size_t(calls) * wmoe_ctx::kProfMarks, nullptr);
  for (cudaEvent_t& e : ctx->prof_events) {
    const cudaError_t err = cudaEventCreate(&e);
    if (err != cudaSuccess) {
      e = nullptr;
      free_profiling(ctx);
      return cuda_fail(ctx, err, "wmoe_set_profiling");
    }
  }
  ctx->profile_calls = calls;
  return WMOE_OK;
}

int wmoe_phase_ms(wmoe_ctx* ctx, int ago, int phase, float* ms) {
  if (!ctx) return WMOE_ERR_INVALID;
  if (!ms || phase < 0 || phase >= WMOE_PHASES || ctx->profile_calls == 0 || ago < 0 ||
      uint64_t(ago) >= ctx->profile_seq || ago >= ctx->profile_calls)
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_phase_ms: no such recorded call or phase");
  const size_t slot = size_t((ctx->profile_seq - 1 - uint64_t(ago)) % uint64_t(ctx->profile_calls));
  cudaEvent_t* ev = &ctx->prof_events[slot * wmoe_ctx::kProfMarks];
  cudaError_t e = cudaEventSynchronize(ev[phase + 1]);
  if (e == cudaSuccess) e = cudaEventElapsedTime(ms, ev[phase], ev[phase + 1]);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "wmoe_phase_ms");
  return WMOE_OK;
}

int wmoe_set_prefill_threshold(wmoe_ctx* ctx, int tokens) {
  if (!ctx || tokens < 1) return WMOE_ERR_INVALID;
  const int prev = ctx->prefill_threshold;
  ctx->prefill_threshold = tokens;
  return prev;
}

int wmoe_set_min_expert_weight(wmoe_ctx* ctx, float weight) {
  if (!ctx) return WMOE_ERR_INVALID;
  if (!(weight >= 0.f && weight < 1.f))
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_set_min_expert_weight: the weight must lie in [0, 1)");
  ctx->min_expert_weight = weight;
  return WMOE_OK;
}

int wmoe_set_decode_kernel(wmoe_ctx* ctx, int enable) {
  if (!ctx) return WMOE_ERR_INVALID;
  const int prev = ctx->use_decode_kernel ? 1 : 0;
  ctx->use_decode_kernel = enable != 0;
  return prev;
}

int wmoe_device_status(wmoe_ctx* ctx, int* status, void* stream) {
  if (!ctx || !status) return WMOE_ERR_INVALID;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  int v = 0;
  WMOE_CHECK_CUDA(ctx, cudaMemcpyAsync(&v, ctx->d_status, sizeof(int), cudaMemcpyDeviceToHost, st), "status read");
  WMOE_CHECK_CUDA(ctx, cudaStreamSynchronize(st), "status read");
  WMOE_CHECK_CUDA(ctx, cudaMemsetAsync(ctx->d_status, 0, sizeof(int), st), "status clear");
  *status = v;
  return WMOE_OK;
}

int wmoe_dequant(wmoe_ctx* ctx, int ggml_type, const uint8_t* blocks, size_t nblocks, void* out, int out_dtype,
                 void* stream) {
  if (!ctx) return WMOE_ERR_INVALID;
  if (ggml_row_bytes(ggml_type, 256) == 0)
    return ctx_fail(ctx, WMOE_ERR_UNSUPPORTED, "wmoe_dequant: type " + std::to_string(ggml_type) +
                                                   " is not one of the WMOE_GGML_* types");
  if (out_dtype != WMOE_F32 && out_dtype != WMOE_BF16 && out_dtype != WMOE_F16)
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_dequant: bad output dtype");
  if (nblocks && (!blocks || !out)) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_dequant: null pointer");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (ggml_type == WMOE_GGML_Q4_K || ggml_type == WMOE_GGML_Q6_K)
    WMOE_CHECK_CUDA(ctx, dequant(ggml_type, blocks, nblocks, out, out_dtype, st), "wmoe_dequant");
  else
    WMOE_CHECK_CUDA(ctx, ggml_dequant(ggml_type, blocks, nblocks, out, out_dtype, st), "wmoe_dequant");
  ctx->launches += nblocks ? 1 : 0;
  return WMOE_OK;
}

// Router + top-k + shared gate of T tokens into caller buffers: for bf16 tokens with the split router, logits on the
// tensor cores (partial sums of a K split); otherwise float32 on the CUDA cores, through the sliced router above 8
// tokens (the same bits per token whatever the call's size). logits: router_logit_floats() floats of scratch.
static bool use_router_tc(const void* router_split, int x_dtype, int T, int H, int E) {
  return router_split && x_dtype == WMOE_BF16 && T >= 16 && router_tc_supported(T, H, E);
}
static size_t router_logit_floats(bool tc, int T, int E, int H) {
  if (tc) return size_t(kRouterKSplit) * T * E;
  if (T > 8) return size_t(router_slice_outputs(T, H)) * T * E;
  return size_t(T) * (E + 1);
}
static cudaError_t route_topk(bool tc, const void* x, int x_dtype, int T, int H, int E, int k, const float* router_w,
                              const float* router_bias, const float* shared_gate, const void* router_split,
                              float* logits, float* topk_w, int32_t* topk_idx, float* shared_s, int* status,
                              cudaStream_t st, int* n, float* logits_out) {
  cudaError_t e;
  if (tc) {
    if ((e = router_logits_tc(x, T, H, E, router_split, logits, status, st, n)) != cudaSuccess) return e;
    return router_topk_split(logits, kRouterKSplit, T, E, k, router_bias, topk_w, topk_idx, shared_s, logits_out, x,
                             x_dtype, shared_gate, H, st, n);
  }
  if (T > 8) {
    if ((e = router_logits_sliced(x, x_dtype, T, H, E, router_w, logits, st, n)) != cudaSuccess) return e;
    return router_topk_split(logits, router_slice_outputs(T, H), T, E, k, router_bias, topk_w, topk_idx, shared_s,
                             logits_out, x, x_dtype, shared_gate, H, st, n);
  }
  if ((e = router_logits(x, x_dtype, T, H, E, router_w, shared_gate, logits, st, n)) != cudaSuccess) return e;
  return router_topk(logits, T, E, k, router_bias, topk_w, topk_idx, shared_s, logits_out, st, n);
}
// The routing of every multi-token path: route_topk, then willow's skip_small_experts when min_w > 0 (the dropped
// picks keep their ids internally, with weight 0).
static cudaError_t route_tokens(bool tc, const void* x, int x_dtype, int T, int H, int E, int k, const float* router_w,
                                const float* router_bias, const float* shared_gate, const void* router_split,
                                float* logits, float* topk_w, int32_t* topk_idx, float* shared_s, int* status,
                                cudaStream_t st, int* n, float min_w, float* logits_out = nullptr) {
  const cudaError_t e = route_topk(tc, x, x_dtype, T, H, E, k, router_w, router_bias, shared_gate, router_split, logits,
                                   topk_w, topk_idx, shared_s, status, st, n, logits_out);
  if (e != cudaSuccess) return e;
  return skip_small_experts(topk_w, T, k, min_w, st, n);
}

// A caller's copy of the picks: -1 where skip_small_experts dropped one (as willow marks them), else the ids.
static cudaError_t copy_picks(const int32_t* topk_idx, const float* topk_w, int32_t* out, int n, float min_w,
                              cudaStream_t st, int* launches) {
  if (min_w > 0.f) return mark_dropped(topk_idx, topk_w, out, n, st, launches);
  return cudaMemcpyAsync(out, topk_idx, size_t(n) * sizeof(int32_t), cudaMemcpyDeviceToDevice, st);
}

int wmoe_route(wmoe_ctx* ctx, const void* x, int x_dtype, int T, int hidden, int experts, int top_k,
               const float* router_w, const float* router_bias, const float* shared_gate, float* topk_w,
               int32_t* topk_idx, float* shared_s, float* logits, void* stream) {
  if (!ctx) return WMOE_ERR_INVALID;
  if (T < 0 || hidden <= 0 || hidden % 128 || experts <= 0 || experts > 512 || top_k <= 0 || top_k > 32 ||
      top_k > experts)
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_route: bad shape");
  if (x_dtype != WMOE_F32 && x_dtype != WMOE_BF16) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_route: bad dtype");
  if (T == 0) return WMOE_OK;
  if (!x || !router_w || !topk_w || !topk_idx || (shared_s && !shared_gate))
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_route: null pointer");
  Plan plan;
  const size_t o_logits = plan.take<float>(router_logit_floats(false, T, experts, hidden));
  if (int rc = ensure_scratch(ctx, plan.bytes)) return rc;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  int n = 0;
  WMOE_CHECK_CUDA(ctx,
                  route_tokens(false, x, x_dtype, T, hidden, experts, top_k, router_w, router_bias, shared_gate,
                               nullptr, at<float>(ctx, o_logits), topk_w, topk_idx, shared_s, ctx->d_status, st, &n,
                               ctx->min_expert_weight, logits),
                  "router");
  ctx->launches += uint64_t(n);
  return WMOE_OK;
}

int wmoe_pack_router(wmoe_ctx* ctx, const float* router_w, const float* shared_gate, int experts, int hidden,
                     float* out, void* stream) {
  if (!ctx) return WMOE_ERR_INVALID;
  if (experts <= 0 || experts >= WMOE_ROUTER_STRIDE || hidden <= 0)
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_pack_router: bad shape");
  if (!router_w || !shared_gate || !out) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_pack_router: null pointer");
  WMOE_CHECK_CUDA(ctx, pack_router(router_w, shared_gate, experts, hidden, out, static_cast<cudaStream_t>(stream)),
                  "wmoe_pack_router");
  ctx->launches += 1;
  return WMOE_OK;
}

int wmoe_split_router(wmoe_ctx* ctx, const float* router_w, int experts, int hidden, uint16_t* out, void* stream) {
  if (!ctx) return WMOE_ERR_INVALID;
  if (experts <= 0 || hidden <= 0) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_split_router: bad shape");
  if (!router_w || !out) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_split_router: null pointer");
  WMOE_CHECK_CUDA(ctx, router_split(router_w, experts, hidden, out, static_cast<cudaStream_t>(stream)),
                  "wmoe_split_router");
  ctx->launches += 1;
  return WMOE_OK;
}

int wmoe_dispatch(wmoe_ctx* ctx, const int32_t* topk_idx, int T, int top_k, int experts, int32_t* counts,
                  int32_t* offsets, int32_t* perm, int64_t* usage, void* stream) {
  if (!ctx) return WMOE_ERR_INVALID;
  if (T < 0 || top_k <= 0 || experts <= 0 || experts > 992) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_dispatch: bad shape");
  if (!counts || !offsets || (T > 0 && (!topk_idx || !perm)))
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_dispatch: null pointer");
  Plan plan;
  const size_t o_disp = plan.bytes;
  plan.bytes += (dispatch_scratch_bytes(T, experts) + 255) / 256 * 256;
  const size_t o_pos = plan.take<int32_t>(size_t(T) * top_k + 1);
  const size_t o_used = plan.take<int32_t>(size_t(experts) + 1);
  const size_t o_seg = plan.take<int32_t>(size_t(experts) + 2);
  const size_t o_nused = plan.take<int32_t>(1);
  if (int rc = ensure_scratch(ctx, plan.bytes)) return rc;
  int n = 0;
  WMOE_CHECK_CUDA(ctx,
                  dispatch(topk_idx, T, top_k, experts, at<void>(ctx, o_disp), counts, offsets, perm,
                           at<int32_t>(ctx, o_pos), at<int32_t>(ctx, o_used), at<int32_t>(ctx, o_seg),
                           at<int32_t>(ctx, o_nused), usage, ctx->d_status, static_cast<cudaStream_t>(stream), &n),
                  "wmoe_dispatch");
  ctx->launches += uint64_t(n);
  return WMOE_OK;
}

int wmoe_store_create(wmoe_ctx* ctx, int layers, int experts, int hidden, int ffn, size_t cap_bytes,
                      wmoe_store** out) {
  return wmoe_store_create_range(ctx, layers, experts, 0, experts, hidden, ffn, cap_bytes, out);
}

int wmoe_store_create_range(wmoe_ctx* ctx, int layers, int experts, int expert_begin, int expert_end, int hidden,
                            int ffn, size_t cap_bytes, wmoe_store** out) {
  if (!ctx) return WMOE_ERR_INVALID;
  if (!out || layers <= 0 || experts <= 0 || hidden <= 0 || ffn <= 0 || hidden % 256 || ffn % 256 ||
      expert_begin < 0 || expert_end > experts || expert_begin >= expert_end)
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_store_create: bad arguments");
  *out = nullptr;
  return store_create(ctx, layers, experts, expert_begin, expert_end, hidden, ffn, cap_bytes, out);
}

void wmoe_store_destroy(wmoe_store* store) { store_destroy(store); }

int wmoe_store_upload(wmoe_store* store, int layer, int expert, const void* host_src, void* stream) {
  if (!store) return WMOE_ERR_INVALID;
  return store_upload(store, layer, expert, host_src, static_cast<cudaStream_t>(stream));
}

int wmoe_store_fill_synthetic(wmoe_store* store, uint64_t seed, int layer_begin, int layer_end, void* stream) {
  if (!store) return WMOE_ERR_INVALID;
  return store_fill_synthetic(store, seed, layer_begin, layer_end, static_cast<cudaStream_t>(stream));
}

size_t wmoe_store_blob_bytes(const wmoe_store* store) { return store ? store->blob_bytes : 0; }

int wmoe_store_set_down_type(wmoe_store* store, int layer, int ggml_type) {
  if (!store) return WMOE_ERR_INVALID;
  return store_set_down_type(store, layer, ggml_type);
}

size_t wmoe_store_layer_blob_bytes(const wmoe_store* store, int layer) {
  if (!store || layer < 0 || layer >= store->layers) return 0;
  return store->layer_blob_bytes(layer);
}

int wmoe_store_prepare(wmoe_store* store, int layer, const int32_t* experts, int n, void* stream) {
  if (!store || (n > 0 && !experts)) return WMOE_ERR_INVALID;
  return store_prepare(store, layer, experts, n, static_cast<cudaStream_t>(stream));
}

int wmoe_store_download(wmoe_store* store, int layer, int expert, void* host_dst, void* stream) {
  if (!store) return WMOE_ERR_INVALID;
  wmoe_ctx* ctx = store->ctx;
  if (layer < 0 || layer >= store->layers || expert < 0 || expert >= store->experts || !host_dst)
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_store_download: bad arguments");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t key = size_t(layer) * store->experts + expert;
  const int slot = store->slot_of[key];
  if (!store->owns(expert)) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_store_download: expert outside the store's range");
  if (slot >= 0) {
    WMOE_CHECK_CUDA(ctx, cudaMemcpyAsync(host_dst, store->d_slab + size_t(slot) * store->slot_stride,
                                         store->layer_blob_bytes(layer), cudaMemcpyDeviceToHost, st),
                    "wmoe_store_download");
    WMOE_CHECK_CUDA(ctx, cudaStreamSynchronize(st), "wmoe_store_download");
  } else if (store->h_master) {
    WMOE_CHECK_CUDA(ctx, cudaStreamSynchronize(st), "wmoe_store_download");
    memcpy(host_dst, store->h_master + store->blob_index(layer, expert) * store->blob_bytes,
           store->layer_blob_bytes(layer));
  } else {
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_store_download: blob not present");
  }
  return WMOE_OK;
}

const uint8_t* wmoe_store_blob(const wmoe_store* store, int layer, int expert) {
  if (!store || layer < 0 || layer >= store->layers || expert < 0 || expert >= store->experts) return nullptr;
  const int slot = store->slot_of[size_t(layer) * store->experts + expert];
  return slot < 0 ? nullptr : store->d_slab + size_t(slot) * store->slot_stride;
}

int wmoe_store_prefetch(wmoe_store* store, int layer, const int32_t* experts, int n, void* stream) {
  if (!store) return WMOE_ERR_INVALID;
  if (n < 0 || (n > 0 && !experts))
    return ctx_fail(store->ctx, WMOE_ERR_INVALID, "wmoe_store_prefetch: bad expert list");
  std::vector<int32_t> all;
  if (!experts) {
    // the guess: the experts this layer has been routed to before (the usage table), most used first; with no
    // history, every expert of the layer the store holds (a prefill batch reads most of them)
    const size_t base = size_t(layer >= 0 && layer < store->layers ? layer : 0) * size_t(store->experts);
    for (int e = store->expert_begin; e < store->expert_end; ++e)
      if (store->usage[base + size_t(e)] > 0) all.push_back(e);
    std::stable_sort(all.begin(), all.end(),
                     [&](int32_t a, int32_t b) { return store->usage[base + size_t(a)] > store->usage[base + size_t(b)]; });
    if (all.empty())
      for (int e = store->expert_begin; e < store->expert_end; ++e) all.push_back(e);
    experts = all.data();
    n = int(all.size());
  }
  return store_prefetch(store, layer, experts, n, static_cast<cudaStream_t>(stream));
}

int wmoe_store_choose_hot(wmoe_store* store, double share) {
  if (!store) return WMOE_ERR_INVALID;
  return store_choose_hot(store, share);
}

int wmoe_store_prefetch_stats(const wmoe_store* store, uint64_t* prefetched, uint64_t* prefetch_used) {
  if (!store) return WMOE_ERR_INVALID;
  if (prefetched) *prefetched = store->prefetched;
  if (prefetch_used) *prefetch_used = store->prefetch_used;
  return WMOE_OK;
}

int wmoe_add_rmsnorm(wmoe_ctx* ctx, const float* x, const void* y, int y_dtype, int T, int hidden, float eps,
                     float* x_out, void* xn_out, int xn_dtype, void* stream) {
  if (!ctx) return WMOE_ERR_INVALID;
  if (T < 0 || hidden <= 0 || hidden % 4 || !(eps >= 0.f))
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_add_rmsnorm: bad shape or eps");
  if ((y && y_dtype != WMOE_F32 && y_dtype != WMOE_BF16) || (xn_dtype != WMOE_F32 && xn_dtype != WMOE_BF16))
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_add_rmsnorm: bad dtype");
  if (T == 0) return WMOE_OK;
  if (!x || !x_out || !xn_out) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_add_rmsnorm: null pointer");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(x_out) |
       reinterpret_cast<uintptr_t>(xn_out)) % 16)
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_add_rmsnorm: buffers must be 16-byte aligned");
  int n = 0;
  WMOE_CHECK_CUDA(ctx,
                  add_rmsnorm(x, y, y_dtype, T, hidden, eps, x_out, xn_out, xn_dtype,
                              static_cast<cudaStream_t>(stream), &n),
                  "wmoe_add_rmsnorm");
  ctx->launches += uint64_t(n);
  return WMOE_OK;
}

int wmoe_store_stats(const wmoe_store* store, uint64_t* hits, uint64_t* misses, uint64_t* bytes_in,
                     uint64_t* evictions) {
  if (!store) return WMOE_ERR_INVALID;
  if (hits) *hits = store->hits;
  if (misses) *misses = store->misses;
  if (bytes_in) *bytes_in = store->bytes_in;
  if (evictions) *evictions = store->evictions;
  return WMOE_OK;
}

static int moe_forward_impl(wmoe_ctx* ctx, wmoe_store* store, int layer, const void* x, int x_dtype, int T,
                            int top_k, const float* router_w, const float* router_bias, const float* shared_gate,
                            const uint8_t* shared_gate_up, const uint8_t* shared_down, const float* router_packed,
                            const void* router_split, void* out, int out_dtype, int32_t* topk_idx_out,
                            float* topk_w_out, void* stream, const AddNorm* an = nullptr) {
  if (!ctx) return WMOE_ERR_INVALID;
  if (!store) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_moe_forward: null store");
  if (store->ctx != ctx) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_moe_forward: store belongs to another context");
  const int H = store->hidden, F = store->ffn, E = store->experts;
  if (layer < 0 || layer >= store->layers || T < 0 || top_k <= 0 || top_k > E)
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_moe_forward: bad layer, token count or top_k");
  if ((x_dtype != WMOE_F32 && x_dtype != WMOE_BF16) || (out_dtype != WMOE_F32 && out_dtype != WMOE_BF16))
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_moe_forward: activations must be F32 or BF16");
  if (H != 2048 || F != 512 || top_k != 8 || E > 512)
    return ctx_fail(ctx, WMOE_ERR_UNSUPPORTED, "wmoe_moe_forward: this build runs hidden 2048, ffn 512, top-8");
  if (T == 0) return WMOE_OK;
  if (!x || !router_w || !shared_gate || !shared_gate_up || !shared_down || (!out && !an))
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_moe_forward: null pointer");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const AddNorm epi = an ? *an : AddNorm{};
  if (T == 1 && !an && !store->capped && ctx->use_decode_kernel && ctx->decode_ctas > 0 && E == 256 &&
      aligned16(router_packed) && aligned16(x)) {
    // one token, every expert resident: the persistent decode kernel (one launch, no host synchronisation)
    if (int rc = ensure_scratch(ctx, decode_scratch_bytes(H, F, E, ctx->decode_ctas))) return rc;
    DecodeLayer dl{router_w, router_bias, shared_gate, shared_gate_up, shared_down, router_packed, router_split};
    int n = 0;
    const int down_type = store->down_type[size_t(layer)];
    const cudaError_t e = decode_persistent(store_source(store, layer, shared_gate_up, shared_down), &down_type,
                                            layer, 1, &dl, H, F, E, top_k, 0.f, false, x, x_dtype, out, out_dtype,
                                            topk_idx_out, topk_w_out, ctx->scratch, ctx->decode_ctas,
                                            ctx->d_status, ctx->trace, ctx->trace_entries, st, &n,
                                            ctx->min_expert_weight);
    ctx->launches += uint64_t(n);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "decode kernel");
    return WMOE_OK;
  }
  const int k = top_k, P = T * (k + 1);
  Plan plan;
  // router logits on the tensor cores for bf16 tokens when the split router is given (partial sums of a K split),
  // else float32 on the CUDA cores ([T][E + 1] with the shared gate as column E)
  const bool router_tc = use_router_tc(router_split, x_dtype, T, H, E);
  const size_t o_logits = plan.take<float>(router_logit_floats(router_tc, T, E, H));
  const size_t o_w = plan.take<float>(size_t(T) * k);
  const size_t o_idx = plan.take<int32_t>(size_t(T) * k);
  const size_t o_s = plan.take<float>(size_t(T));
  const size_t o_counts = plan.take<int32_t>(size_t(E));
  const size_t o_offsets = plan.take<int32_t>(size_t(E) + 1);
  const size_t o_perm = plan.take<int32_t>(size_t(T) * k);
  const size_t o_pos = plan.take<int32_t>(size_t(T) * k);
  const size_t o_used = plan.take<int32_t>(size_t(E) + 1);
  const size_t o_seg = plan.take<int32_t>(size_t(E) + 2);
  const size_t o_nused = plan.take<int32_t>(1);
  const size_t o_disp = plan.bytes;
  plan.bytes += (dispatch_scratch_bytes(T, E) + 255) / 256 * 256;
  // many tokens per expert: tcgen05 grouped GEMMs; few: the dequant-GEMV kernels (their buffers share the region)
  const bool gemm_path = T >= ctx->prefill_threshold;
  const size_t o_region = plan.bytes;
  const size_t o_xq = plan.take<int16_t>(size_t(T) * H);
  const size_t o_xs = plan.take<float>(size_t(T) * H / 32);
  const size_t o_xsum = plan.take<int32_t>(size_t(T) * H / 16);
  const size_t o_h = plan.take<float>(size_t(P) * F);
  const size_t o_hq = plan.take<int16_t>(size_t(P) * F);
  const size_t o_hs = plan.take<float>(size_t(P) * F / 32);
  const size_t o_hsum = plan.take<int32_t>(size_t(P) * F / 16);
  const size_t o_y = plan.take<float>(size_t(P) * H);
  if (gemm_path) plan.bytes = o_region + (prefill_scratch_bytes(T, k, E, H, F) + 255) / 256 * 256;
  if (int rc = ensure_scratch(ctx, plan.bytes)) return rc;

  int n = 0;
  // opt-in phase marks (wmoe_set_profiling): 0 start, 1 routed, 2 dispatched, 3-6 inside the expert products
  cudaEvent_t* marks = ctx->profile_calls > 0
                           ? &ctx->prof_events[size_t(ctx->profile_seq % uint64_t(ctx->profile_calls)) *
                                               wmoe_ctx::kProfMarks]
                           : nullptr;
  auto mark = [&](int i) {
    if (marks) cudaEventRecord(marks[i], st);
  };
  mark(0);
  float* topk_w = at<float>(ctx, o_w);
  int32_t* topk_idx = at<int32_t>(ctx, o_idx);
  float* shared_s = at<float>(ctx, o_s);
  WMOE_CHECK_CUDA(ctx,
                  route_tokens(router_tc, x, x_dtype, T, H, E, k, router_w, router_bias, shared_gate, router_split,
                               at<float>(ctx, o_logits), topk_w, topk_idx, shared_s, ctx->d_status, st, &n,
                               ctx->min_expert_weight),
                  "router");
  mark(1);
  std::vector<int32_t> experts_used;
  if (store->capped) {
    // the store must copy this call's experts in first: one wait for the routing (engines/base.py:456-460 does
    // the same with selected.cpu())
    std::vector<int32_t> sel(size_t(T) * k);
    WMOE_CHECK_CUDA(ctx, cudaMemcpyAsync(sel.data(), topk_idx, sel.size() * sizeof(int32_t), cudaMemcpyDeviceToHost, st),
                    "routing read-back");
    WMOE_CHECK_CUDA(ctx, cudaStreamSynchronize(st), "routing read-back");
    store_record_usage(store, layer, sel.data(), sel.size());
    experts_used = sel;
    std::sort(experts_used.begin(), experts_used.end());
    experts_used.erase(std::unique(experts_used.begin(), experts_used.end()), experts_used.end());
    if (int rc = store_prepare(store, layer, experts_used.data(), int(experts_used.size()), st)) return rc;
  }
  PairMap pm;
  pm.T = T;
  pm.k = k;
  pm.E = E;
  pm.perm = at<int32_t>(ctx, o_perm);
  pm.pos = at<int32_t>(ctx, o_pos);
  pm.used = at<int32_t>(ctx, o_used);
  pm.seg = at<int32_t>(ctx, o_seg);
  pm.n_used = at<int32_t>(ctx, o_nused);
  WMOE_CHECK_CUDA(ctx,
                  dispatch(topk_idx, T, k, E, at<void>(ctx, o_disp), at<int32_t>(ctx, o_counts),
                           at<int32_t>(ctx, o_offsets), at<int32_t>(ctx, o_perm), at<int32_t>(ctx, o_pos),
                           at<int32_t>(ctx, o_used), at<int32_t>(ctx, o_seg), at<int32_t>(ctx, o_nused), nullptr,
                           ctx->d_status, st, &n),
                  "dispatch");
  mark(2);
  const ExpertSource src = store_source(store, layer, shared_gate_up, shared_down);
  if (gemm_path) {
    WMOE_CHECK_CUDA(ctx,
                    prefill_experts(src, layer, pm, topk_idx, H, F, x, x_dtype, topk_w, shared_s, out, out_dtype,
                                    epi, at<void>(ctx, o_region), ctx->sm_count, ctx->d_status, marks ? marks + 3 : nullptr,
                                    st, &n),
                    "grouped GEMM");
  } else {
    int16_t* xq = at<int16_t>(ctx, o_xq);
    float* xs = at<float>(ctx, o_xs);
    int32_t* xsum = at<int32_t>(ctx, o_xsum);
    WMOE_CHECK_CUDA(ctx, quant_rows(x, x_dtype, T, H, xq, xs, xsum, st, &n), "activation quantisation");
    mark(3);
    float* h = at<float>(ctx, o_h);
    WMOE_CHECK_CUDA(ctx, gate_up_gemv(src, layer, pm, H, F, xq, xs, xsum, h, ctx->d_status, st, &n), "gate_up");
    int16_t* hq = at<int16_t>(ctx, o_hq);
    float* hs = at<float>(ctx, o_hs);
    int32_t* hsum = at<int32_t>(ctx, o_hsum);
    WMOE_CHECK_CUDA(ctx, quant_rows(h, WMOE_F32, P, F, hq, hs, hsum, st, &n), "hidden quantisation");
    mark(4);
    float* y = at<float>(ctx, o_y);
    WMOE_CHECK_CUDA(ctx, down_gemv(src, layer, pm, H, F, hq, hs, hsum, y, ctx->d_status, st, &n), "down");
    mark(5);
    WMOE_CHECK_CUDA(ctx, combine(pm, H, topk_w, shared_s, y, out, out_dtype, epi, st, &n), "combine");
    mark(6);
  }
  if (marks) ++ctx->profile_seq;
  if (topk_idx_out)
    WMOE_CHECK_CUDA(ctx, copy_picks(topk_idx, topk_w, topk_idx_out, T * k, ctx->min_expert_weight, st, &n),
                    "routing copy");
  if (topk_w_out)
    WMOE_CHECK_CUDA(ctx, cudaMemcpyAsync(topk_w_out, topk_w, size_t(T) * k * sizeof(float), cudaMemcpyDeviceToDevice, st),
                    "routing copy");
  ctx->launches += uint64_t(n);
  if (store->capped)
    if (int rc = store_mark_used(store, layer, experts_used.data(), int(experts_used.size()), st)) return rc;
  return WMOE_OK;
}

int wmoe_moe_forward(wmoe_ctx* ctx, wmoe_store* store, int layer, const void* x, int x_dtype, int T, int top_k,
                     const float* router_w, const float* router_bias, const float* shared_gate,
                     const uint8_t* shared_gate_up, const uint8_t* shared_down, void* out, int out_dtype,
                     int32_t* topk_idx_out, float* topk_w_out, void* stream) {
  return moe_forward_impl(ctx, store, layer, x, x_dtype, T, top_k, router_w, router_bias, shared_gate, shared_gate_up,
                          shared_down, nullptr, nullptr, out, out_dtype, topk_idx_out, topk_w_out, stream);
}

int wmoe_moe_forward_layer(wmoe_ctx* ctx, wmoe_store* store, int layer, const void* x, int x_dtype, int T, int top_k,
                           const wmoe_layer_weights* w, void* out, int out_dtype, int32_t* topk_idx_out,
                           float* topk_w_out, void* stream) {
  if (!ctx) return WMOE_ERR_INVALID;
  if (!w) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_moe_forward_layer: null weights");
  return moe_forward_impl(ctx, store, layer, x, x_dtype, T, top_k, w->router_w, w->router_bias, w->shared_gate,
                          w->shared_gate_up, w->shared_down, w->router_packed, w->router_split, out, out_dtype,
                          topk_idx_out, topk_w_out, stream);
}

static int check_layer(wmoe_ctx* ctx, const wmoe_layer_weights* w, const char* fn) {
  if (!w || !w->router_w || !w->shared_gate || !w->shared_gate_up || !w->shared_down)
    return ctx_fail(ctx, WMOE_ERR_INVALID, std::string(fn) + ": null weight pointer");
  return WMOE_OK;
}

int wmoe_ep_route_plan(wmoe_ctx* ctx, int world, const void* x, int x_dtype, int T, int top_k, int experts,
                       int hidden, const wmoe_layer_weights* w, float* topk_w, int32_t* topk_idx, float* shared_s,
                       int32_t* send_rows, int32_t* send_pairs, int32_t* send_tok, int32_t* pair_list,
                       int32_t* ret_index, uint16_t* send_buf, void* stream) {
  if (!ctx) return WMOE_ERR_INVALID;
  if (world < 1 || world > kMaxRanks || experts <= 0 || experts % world || T < 0 || top_k != 8 || hidden != 2048 ||
      (x_dtype != WMOE_F32 && x_dtype != WMOE_BF16))
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_ep_route_plan: bad world, shape or dtype");
  if (int rc = check_layer(ctx, w, "wmoe_ep_route_plan")) return rc;
  if (!send_rows || !send_pairs || (T > 0 && (!x || !topk_w || !topk_idx || !shared_s || !send_tok || !pair_list ||
                                              !ret_index || !send_buf)))
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_ep_route_plan: null pointer");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (T == 0) {
    WMOE_CHECK_CUDA(ctx, cudaMemsetAsync(send_rows, 0, world * sizeof(int32_t), st), "wmoe_ep_route_plan");
    WMOE_CHECK_CUDA(ctx, cudaMemsetAsync(send_pairs, 0, world * sizeof(int32_t), st), "wmoe_ep_route_plan");
    return WMOE_OK;
  }
  const bool tc = use_router_tc(w->router_split, x_dtype, T, hidden, experts);
  Plan plan;
  const size_t o_logits = plan.take<float>(router_logit_floats(tc, T, experts, hidden));
  const size_t o_plan = plan.take<char>(ep_plan_scratch_bytes(T, world));
  if (int rc = ensure_scratch(ctx, plan.bytes)) return rc;
  int n = 0;
  WMOE_CHECK_CUDA(ctx,
                  route_tokens(tc, x, x_dtype, T, hidden, experts, top_k, w->router_w, w->router_bias, w->shared_gate,
                               w->router_split, at<float>(ctx, o_logits), topk_w, topk_idx, shared_s, ctx->d_status,
                               st, &n, ctx->min_expert_weight),
                  "router");
  WMOE_CHECK_CUDA(ctx,
                  ep_plan(topk_idx, T, top_k, experts, world, send_rows, send_pairs, 1, send_tok, pair_list,
                          ret_index, at<void>(ctx, o_plan), ctx->d_status, st, &n),
                  "wmoe_ep_route_plan: plan");
  WMOE_CHECK_CUDA(ctx,
                  ep_pack(x, x_dtype, hidden, send_tok, send_rows, 1, world, T * std::min(top_k, world), send_buf, st,
                          &n),
                  "wmoe_ep_route_plan: rows");
  ctx->launches += uint64_t(n);
  return WMOE_OK;
}

// Scratch of the expert stage of an expert-parallel layer: P_r received pairs, T own tokens.
static size_t ep_experts_scratch_bytes(int P_r, int T, int E, int H, int F) {
  Plan plan;
  const size_t P = size_t(P_r) + size_t(T);
  plan.take<int32_t>(size_t(P_r));                   // pair_row
  plan.take<int32_t>(size_t(P_r));                   // pair_exp
  plan.take<int32_t>(size_t(E));                     // counts
  plan.take<int32_t>(size_t(E) + 1);                 // offsets
  plan.take<int32_t>(size_t(P_r));                   // perm
  plan.take<int32_t>(size_t(P_r));                   // pos
  plan.take<int32_t>(size_t(E) + 1);                 // used
  plan.take<int32_t>(size_t(E) + 2);                 // seg
  plan.take<int32_t>(1);                             // n_used
  plan.take<char>(dispatch_scratch_bytes(P_r, E));   // dispatch
  plan.take<uint16_t>(P * H);                        // xg
  plan.take<char>(prefill_gemm_scratch_bytes(P, E, H, F));
  return plan.bytes;
}

static int ep_experts_impl(wmoe_ctx* ctx, wmoe_store* store, int layer, int world, const int32_t* recv_rows,
                           const int32_t* recv_pairs, const uint16_t* recv_buf, const int32_t* recv_pair_list,
                           const void* x, int x_dtype, int T, const wmoe_layer_weights* w, uint16_t* y,
                           char* scratch, cudaStream_t st, int gemm_ctas) {
  const int H = store->hidden, F = store->ffn, E = store->experts;
  int P_r = 0;
  for (int s = 0; s < world; ++s) P_r += recv_pairs[s];
  const size_t P = size_t(P_r) + size_t(T);
  if (P == 0) return WMOE_OK;
  Plan plan;
  const size_t o_row = plan.take<int32_t>(size_t(P_r));
  const size_t o_exp = plan.take<int32_t>(size_t(P_r));
  const size_t o_counts = plan.take<int32_t>(size_t(E));
  const size_t o_offsets = plan.take<int32_t>(size_t(E) + 1);
  const size_t o_perm = plan.take<int32_t>(size_t(P_r));
  const size_t o_pos = plan.take<int32_t>(size_t(P_r));
  const size_t o_used = plan.take<int32_t>(size_t(E) + 1);
  const size_t o_seg = plan.take<int32_t>(size_t(E) + 2);
  const size_t o_nused = plan.take<int32_t>(1);
  const size_t o_disp = plan.take<char>(dispatch_scratch_bytes(P_r, E));
  const size_t o_xg = plan.take<uint16_t>(P * H);
  const size_t o_gemm = plan.take<char>(prefill_gemm_scratch_bytes(P, E, H, F));
  auto sp = [&](size_t off) { return static_cast<void*>(scratch + off); };
  int n = 0;
  int32_t* pair_row = static_cast<int32_t*>(sp(o_row));
  int32_t* pair_exp = static_cast<int32_t*>(sp(o_exp));
  WMOE_CHECK_CUDA(ctx, ep_fixup(recv_pair_list, P_r, world, recv_rows, recv_pairs, pair_row, pair_exp, st, &n),
                  "expert stage: pair lists");
  std::vector<int32_t> experts_used;
  if (store->capped && P_r > 0) {
    // the store must copy the received pairs' experts in first: one wait for the pair list
    std::vector<int32_t> ex(static_cast<size_t>(P_r));
    WMOE_CHECK_CUDA(ctx, cudaMemcpyAsync(ex.data(), pair_exp, ex.size() * sizeof(int32_t), cudaMemcpyDeviceToHost, st),
                    "pair read-back");
    WMOE_CHECK_CUDA(ctx, cudaStreamSynchronize(st), "pair read-back");
    store_record_usage(store, layer, ex.data(), ex.size());
    std::sort(ex.begin(), ex.end());
    ex.erase(std::unique(ex.begin(), ex.end()), ex.end());
    experts_used = ex;
    if (int rc = store_prepare(store, layer, experts_used.data(), int(experts_used.size()), st)) return rc;
  }
  PairMap pm;
  pm.T = P_r;
  pm.k = 1;
  pm.E = E;
  pm.perm = static_cast<int32_t*>(sp(o_perm));
  pm.pos = static_cast<int32_t*>(sp(o_pos));
  pm.used = static_cast<int32_t*>(sp(o_used));
  pm.seg = static_cast<int32_t*>(sp(o_seg));
  pm.n_used = static_cast<int32_t*>(sp(o_nused));
  WMOE_CHECK_CUDA(ctx,
                  dispatch_rows(pair_exp, P_r, 1, E, T, sp(o_disp), static_cast<int32_t*>(sp(o_counts)),
                                static_cast<int32_t*>(sp(o_offsets)), const_cast<int32_t*>(pm.perm),
                                const_cast<int32_t*>(pm.pos), const_cast<int32_t*>(pm.used),
                                const_cast<int32_t*>(pm.seg), const_cast<int32_t*>(pm.n_used), nullptr, ctx->d_status,
                                st, &n),
                  "expert stage: dispatch");
  __half* xg = static_cast<__half*>(sp(o_xg));
  WMOE_CHECK_CUDA(ctx, ep_gather(pm.perm, pair_row, P_r, recv_buf, x, x_dtype, T, H, xg, st, &n),
                  "expert stage: gather");
  const ExpertSource src = store_source(store, layer, w->shared_gate_up, w->shared_down);
  WMOE_CHECK_CUDA(ctx,
                  prefill_gemms(src, layer, pm, P, H, F, xg, reinterpret_cast<__half*>(y), pm.perm, P_r, sp(o_gemm),
                                gemm_ctas, ctx->d_status, nullptr, st, &n),
                  "expert stage: grouped GEMM");
  ctx->launches += uint64_t(n);
  if (store->capped && !experts_used.empty())
    if (int rc = store_mark_used(store, layer, experts_used.data(), int(experts_used.size()), st)) return rc;
  return WMOE_OK;
}

static int check_ep_counts(wmoe_ctx* ctx, int world, const int32_t* recv_rows, const int32_t* recv_pairs, int T,
                           const char* fn) {
  long long R = 0, Pr = 0;
  for (int s = 0; s < world; ++s) {
    if (recv_rows[s] < 0 || recv_pairs[s] < 0) return ctx_fail(ctx, WMOE_ERR_INVALID, std::string(fn) + ": bad counts");
    R += recv_rows[s];
    Pr += recv_pairs[s];
  }
  if (Pr + T > (1ll << 30) || Pr > R * 8) return ctx_fail(ctx, WMOE_ERR_INVALID, std::string(fn) + ": bad counts");
  return WMOE_OK;
}

int wmoe_ep_experts(wmoe_ctx* ctx, wmoe_store* store, int layer, int world, const int32_t* recv_rows,
                    const int32_t* recv_pairs, const uint16_t* recv_buf, const int32_t* recv_pair_list,
                    const void* x, int x_dtype, int T, const wmoe_layer_weights* w, uint16_t* y, void* stream) {
  if (!ctx) return WMOE_ERR_INVALID;
  if (!store || store->ctx != ctx) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_ep_experts: bad store");
  if (world < 1 || world > kMaxRanks || !recv_rows || !recv_pairs || layer < 0 || layer >= store->layers || T < 0 ||
      (x_dtype != WMOE_F32 && x_dtype != WMOE_BF16))
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_ep_experts: bad arguments");
  if (int rc = check_layer(ctx, w, "wmoe_ep_experts")) return rc;
  if (store->hidden != 2048 || store->ffn != 512)
    return ctx_fail(ctx, WMOE_ERR_UNSUPPORTED, "wmoe_ep_experts: this build runs hidden 2048, ffn 512");
  if (int rc = check_ep_counts(ctx, world, recv_rows, recv_pairs, T, "wmoe_ep_experts")) return rc;
  int P_r = 0, R = 0;
  for (int s = 0; s < world; ++s) P_r += recv_pairs[s], R += recv_rows[s];
  if (P_r + T == 0) return WMOE_OK;
  if (!y || (T > 0 && !x) || (P_r > 0 && (!recv_buf || !recv_pair_list)))
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_ep_experts: null pointer");
  if (int rc = ensure_scratch(ctx, ep_experts_scratch_bytes(P_r, T, store->experts, store->hidden, store->ffn)))
    return rc;
  return ep_experts_impl(ctx, store, layer, world, recv_rows, recv_pairs, recv_buf, recv_pair_list, x, x_dtype, T, w, y,
                         static_cast<char*>(ctx->scratch), static_cast<cudaStream_t>(stream), ctx->sm_count);
}

int wmoe_ep_combine(wmoe_ctx* ctx, int T, int top_k, int hidden, const int32_t* topk_idx, const float* topk_w,
                    const int32_t* ret_index, const float* shared_s, const uint16_t* y_returned,
                    const uint16_t* y_shared, void* out, int out_dtype, void* stream) {
  if (!ctx) return WMOE_ERR_INVALID;
  if (T < 0 || top_k != 8 || hidden <= 0 || hidden % 8 || (out_dtype != WMOE_F32 && out_dtype != WMOE_BF16))
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_ep_combine: bad arguments");
  if (T == 0) return WMOE_OK;
  if (!topk_idx || !topk_w || !ret_index || !shared_s || !y_returned || !y_shared || !out)
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_ep_combine: null pointer");
  int n = 0;
  WMOE_CHECK_CUDA(ctx,
                  combine_rows(T, top_k, hidden, topk_idx, topk_w, ret_index, shared_s,
                               reinterpret_cast<const __half*>(y_returned), reinterpret_cast<const __half*>(y_shared),
                               out, out_dtype, AddNorm{}, static_cast<cudaStream_t>(stream), &n),
                  "wmoe_ep_combine");
  ctx->launches += uint64_t(n);
  return WMOE_OK;
}

// ---- expert parallelism over the library's own NCCL communicator ----------------------------------------------
// NCCL is resolved at run time (dlopen of libnccl.so.2, reusing the copy already loaded in the process, e.g. by
// torch), so the library loads without it and only wmoe_ep_init needs it.
struct NcclApi {
  bool ok = false;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

static NcclApi& nccl() {
  static NcclApi api;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h) {
      auto get = [&](const char* name) { return dlsym(h, name); };
      api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(get("ncclGetUniqueId"));
      api.CommInitRankConfig = reinterpret_cast<decltype(api.CommInitRankConfig)>(get("ncclCommInitRankConfig"));
      api.CommGetAsyncError = reinterpret_cast<decltype(api.CommGetAsyncError)>(get("ncclCommGetAsyncError"));
      api.CommAbort = reinterpret_cast<decltype(api.CommAbort)>(get("ncclCommAbort"));
      api.CommFinalize = reinterpret_cast<decltype(api.CommFinalize)>(get("ncclCommFinalize"));
      api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(get("ncclCommDestroy"));
      api.GroupStart = reinterpret_cast<decltype(api.GroupStart)>(get("ncclGroupStart"));
      api.GroupEnd = reinterpret_cast<decltype(api.GroupEnd)>(get("ncclGroupEnd"));
      api.Send = reinterpret_cast<decltype(api.Send)>(get("ncclSend"));
      api.Recv = reinterpret_cast<decltype(api.Recv)>(get("ncclRecv"));
      api.AllGather = reinterpret_cast<decltype(api.AllGather)>(get("ncclAllGather"));
      api.AllReduce = reinterpret_cast<decltype(api.AllReduce)>(get("ncclAllReduce"));
      api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(get("ncclGetErrorString"));
      api.ok = api.GetUniqueId && api.CommInitRankConfig && api.CommGetAsyncError && api.CommAbort &&
               api.CommFinalize && api.CommDestroy && api.GroupStart && api.GroupEnd && api.Send && api.Recv && api.AllGather &&
               api.AllReduce && api.GetErrorString;
    }
  }
  return api;
}

static void ep_release(wmoe_ctx* ctx);

static long long now_ms() {
  return std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

// One step of a host poll: spins (yielding the core) for the first 5 ms of a wait, then sleeps 50 us at a time. A
// sleep from the start would cost every settled call and every count read-back the timer slack (~50 us or more).
static void poll_pause(long long t0) {
  if (now_ms() - t0 < 5)
    std::this_thread::yield();
  else
    std::this_thread::sleep_for(std::chrono::microseconds(50));
}

// ncclCommAbort on a helper thread, waited for at most timeout_ms: the abort makes the communicator's kernels
// return and frees its resources; should it itself not return, the host is not held (the thread is left to it).
// Returns whether it finished.
static bool abort_comm(ncclComm_t comm, int timeout_ms) {
  auto done = std::make_shared<std::atomic<bool>>(false);
  std::thread([comm, done] {
    nccl().CommAbort(comm);
    done->store(true);
  }).detach();
  const long long t0 = now_ms();
  while (!done->load() && now_ms() - t0 <= timeout_ms) poll_pause(t0);
  return done->load();
}

// A failure of the communicator: the context aborts it (its kernels in flight return) and keeps no exchange state;
// every later EP call fails until wmoe_ep_finalize and a new wmoe_ep_init.
static int nccl_fail(wmoe_ctx* ctx, ncclResult_t r, const char* where) {
  std::string msg = std::string(where) + ": " + nccl().GetErrorString(r);
  if (ctx->nccl_comm) {
    const bool aborted = abort_comm(static_cast<ncclComm_t>(ctx->nccl_comm), ctx->ep_timeout_ms);
    ctx->nccl_comm = nullptr;
    ctx->ep_dead = true;
    msg += aborted ? " (communicator aborted)" : " (communicator abort did not finish in time)";
  }
  return ctx_fail(ctx, WMOE_ERR_NCCL, msg);
}

// The communicator is non-blocking: a call may return ncclInProgress and finish in the background. Waits, for at
// most the context's timeout, until its state is settled; an error or the timeout aborts it.
static int nccl_settle(wmoe_ctx* ctx, ncclResult_t r, const char* where) {
  if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(ctx, r, where);
  ncclComm_t comm = static_cast<ncclComm_t>(ctx->nccl_comm);
  const long long t0 = now_ms();
  for (;;) {
    ncclResult_t state = ncclSuccess;
    const ncclResult_t q = nccl().CommGetAsyncError(comm, &state);
    if (q != ncclSuccess) return nccl_fail(ctx, q, where);
    if (state == ncclSuccess) return WMOE_OK;
    if (state != ncclInProgress) return nccl_fail(ctx, state, where);
    if (now_ms() - t0 > ctx->ep_timeout_ms)
      return nccl_fail(ctx, ncclRemoteError, (std::string(where) + ": timed out").c_str());
    poll_pause(t0);
  }
}

#define WMOE_CHECK_NCCL(ctx, call, where)                              \
  do {                                                               \
    if (int rc_ = nccl_settle(ctx, (call), where)) return rc_;       \
  } while (0)

// A host wait for work on a stream that includes communicator kernels: bounded by the context's timeout, and
// watching the communicator for an asynchronous error (a peer that left). Either aborts the communicator.
static int ep_wait(wmoe_ctx* ctx, cudaStream_t st, const char* where) {
  const long long t0 = now_ms();
  for (;;) {
    const cudaError_t e = cudaStreamQuery(st);
    if (e == cudaSuccess) return WMOE_OK;
    if (e != cudaErrorNotReady) return cuda_fail(ctx, e, where);
    ncclResult_t state = ncclSuccess;
    nccl().CommGetAsyncError(static_cast<ncclComm_t>(ctx->nccl_comm), &state);
    if (state != ncclSuccess && state != ncclInProgress) return nccl_fail(ctx, state, where);
    if (now_ms() - t0 > ctx->ep_timeout_ms)
      return nccl_fail(ctx, ncclRemoteError, (std::string(where) + ": timed out waiting for the other ranks").c_str());
    poll_pause(t0);
  }
}

int wmoe_ep_unique_id(void* out) {
  if (!out) return WMOE_ERR_INVALID;
  if (!nccl().ok) return WMOE_ERR_UNSUPPORTED;
  ncclUniqueId id;
  if (nccl().GetUniqueId(&id) != ncclSuccess) return WMOE_ERR_NCCL;
  memcpy(out, &id, sizeof(id));
  return WMOE_OK;
}

int wmoe_ep_set_timeout(wmoe_ctx* ctx, int ms) {
  if (!ctx || ms < 1) return WMOE_ERR_INVALID;
  const int prev = ctx->ep_timeout_ms;
  ctx->ep_timeout_ms = ms;
  return prev;
}

static int ep_setup_windows(wmoe_ctx* ctx);

int wmoe_ep_init(wmoe_ctx* ctx, const void* unique_id, int rank, int world) {
  if (!ctx) return WMOE_ERR_INVALID;
  if (!unique_id || world < 1 || world > WMOE_MAX_RANKS || rank < 0 || rank >= world)
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_ep_init: bad rank / world");
  if (!nccl().ok) return ctx_fail(ctx, WMOE_ERR_UNSUPPORTED, "wmoe_ep_init: libnccl.so.2 not available");
  if (ctx->nccl_comm || ctx->ep_dead)
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_ep_init: already initialised (wmoe_ep_finalize first)");
  WMOE_CHECK_CUDA(ctx, cudaSetDevice(ctx->device), "wmoe_ep_init");
  ncclUniqueId id;
  memcpy(&id, unique_id, sizeof(id));
  ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
  config.blocking = 0;
  ncclComm_t comm = nullptr;
  const ncclResult_t r = nccl().CommInitRankConfig(&comm, world, id, rank, &config);
  ctx->nccl_comm = comm;
  if (int rc = nccl_settle(ctx, r, "wmoe_ep_init")) return rc;
  ctx->ep_rank = rank;
  ctx->ep_world = world;
  // measured at 4096 tokens per rank: one chunk is fastest on two ranks, two on eight (one and four slower: the
  // exchanges' fixed costs against the expert stage's overlap)
  ctx->ep_chunks = world >= 4 ? 2 : 1;
  WMOE_CHECK_CUDA(ctx, cudaStreamCreateWithFlags(&ctx->ep_stream, cudaStreamNonBlocking), "wmoe_ep_init");
  ctx->ep_events.assign(1 + 3 * kMaxEpChunks, nullptr);
  for (cudaEvent_t& e : ctx->ep_events)
    WMOE_CHECK_CUDA(ctx, cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "wmoe_ep_init");
  return ep_setup_windows(ctx);
}

static void ep_close_windows(wmoe_ctx* ctx) {
  for (int d = 0; d < int(ctx->ep_peer_win.size()); ++d)
    if (d != ctx->ep_rank && ctx->ep_peer_win[size_t(d)]) cudaIpcCloseMemHandle(ctx->ep_peer_win[size_t(d)]);
  ctx->ep_peer_win.clear();
  cudaFree(ctx->ep_win);
  ctx->ep_win = nullptr;
  ctx->ep_win_bytes = 0;
}

// Ends the communicator: ncclCommFinalize is collective (it waits for the other ranks' finalize), so its completion
// is polled for at most the context's timeout, and a communicator whose finalize does not complete (a rank left) is
// aborted instead of waited on.
static void ep_end_comm(wmoe_ctx* ctx) {
  if (!ctx->nccl_comm) return;
  ncclComm_t comm = static_cast<ncclComm_t>(ctx->nccl_comm);
  ctx->nccl_comm = nullptr;
  const ncclResult_t r = nccl().CommFinalize(comm);
  bool done = r == ncclSuccess;
  if (r == ncclInProgress) {
    const long long t0 = now_ms();
    for (;;) {
      ncclResult_t state = ncclSuccess;
      if (nccl().CommGetAsyncError(comm, &state) != ncclSuccess) break;
      if (state == ncclSuccess) {
        done = true;
        break;
      }
      if (state != ncclInProgress || now_ms() - t0 > ctx->ep_timeout_ms) break;
      poll_pause(t0);
    }
  }
  if (done)
    nccl().CommDestroy(comm);
  else
    abort_comm(comm, ctx->ep_timeout_ms);
}

static void ep_release(wmoe_ctx* ctx) {
  ep_end_comm(ctx);
  ctx->ep_dead = false;
  ep_close_windows(ctx);
  for (cudaStream_t s : ctx->ep_peer_streams)
    if (s) cudaStreamDestroy(s);
  ctx->ep_peer_streams.clear();
  for (cudaEvent_t e : ctx->ep_peer_events)
    if (e) cudaEventDestroy(e);
  ctx->ep_peer_events.clear();
  cudaFree(ctx->ep_flag);
  ctx->ep_flag = nullptr;
  cudaFree(ctx->ep_handles);
  ctx->ep_handles = nullptr;
  cudaFreeHost(ctx->ep_host_counts);
  ctx->ep_host_counts = nullptr;
  cudaFreeHost(ctx->ep_host_handles);
  ctx->ep_host_handles = nullptr;
  ctx->ep_ipc = false;
  for (cudaEvent_t e : ctx->ep_events)
    if (e) cudaEventDestroy(e);
  ctx->ep_events.clear();
  if (ctx->ep_stream) cudaStreamDestroy(ctx->ep_stream);
  ctx->ep_stream = nullptr;
  ctx->ep_world = 0;
  cudaFree(ctx->ep_buf);
  ctx->ep_buf = nullptr;
  ctx->ep_buf_bytes = 0;
}

int wmoe_ep_finalize(wmoe_ctx* ctx) {
  if (!ctx) return WMOE_ERR_INVALID;
  cudaSetDevice(ctx->device);
  if (!ctx->ep_dead) {
    const cudaError_t e = cudaDeviceSynchronize();
    ep_release(ctx);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "wmoe_ep_finalize");
    return WMOE_OK;
  }
  // after an abort: the aborted kernels return, so the EP streams drain; wait for that for at most the timeout
  // (cudaFree and cudaDeviceSynchronize would block for good behind a stream that did not)
  std::vector<cudaStream_t> streams(ctx->ep_peer_streams);
  streams.push_back(ctx->ep_stream);
  const long long t0 = now_ms();
  bool drained = false;
  while (!drained && now_ms() - t0 <= ctx->ep_timeout_ms) {
    drained = true;
    for (cudaStream_t s : streams)
      if (s && cudaStreamQuery(s) == cudaErrorNotReady) drained = false;
    if (!drained) poll_pause(t0);
  }
  if (!drained)
    return ctx_fail(ctx, WMOE_ERR_NCCL, "wmoe_ep_finalize: the exchange streams did not drain after the abort; "
                                        "their buffers are left allocated");
  ep_release(ctx);
  return WMOE_OK;
}

// The exchange machinery beside the communicator: a stream and an event per destination rank, the barrier word and
// the staging of the IPC handle all-gather. Windows themselves are made by ep_grow_windows when a call first
// needs them. Without peer access between every pair of devices the rows go through NCCL send/recv instead.
static int ep_setup_windows(wmoe_ctx* ctx) {
  const int world = ctx->ep_world;
  ctx->ep_peer_streams.assign(size_t(world), nullptr);
  ctx->ep_peer_events.assign(size_t(world), nullptr);
  for (int d = 0; d < world; ++d) {
    WMOE_CHECK_CUDA(ctx, cudaStreamCreateWithFlags(&ctx->ep_peer_streams[size_t(d)], cudaStreamNonBlocking),
                    "wmoe_ep_init");
    WMOE_CHECK_CUDA(ctx, cudaEventCreateWithFlags(&ctx->ep_peer_events[size_t(d)], cudaEventDisableTiming),
                    "wmoe_ep_init");
  }
  WMOE_CHECK_CUDA(ctx, cudaMalloc(&ctx->ep_flag, 256), "wmoe_ep_init");
  WMOE_CHECK_CUDA(ctx, cudaMemset(ctx->ep_flag, 0, 256), "wmoe_ep_init");
  WMOE_CHECK_CUDA(ctx, cudaMalloc(&ctx->ep_handles, size_t(world) * sizeof(cudaIpcMemHandle_t)), "wmoe_ep_init");
  WMOE_CHECK_CUDA(ctx, cudaMallocHost(&ctx->ep_host_counts, size_t(kMaxRanks) * kMaxRanks * kCountWords * 4),
                  "wmoe_ep_init");
  WMOE_CHECK_CUDA(ctx, cudaMallocHost(&ctx->ep_host_handles, size_t(kMaxRanks) * sizeof(cudaIpcMemHandle_t)),
                  "wmoe_ep_init");
  // the rows' exchange: copy engines into the peers' windows, or NCCL send/recv (WMOE_EP_NCCL_ROWS); the environment
  // decides, read here once
  ctx->ep_ipc = std::getenv("WMOE_EP_NCCL_ROWS") == nullptr;
  return WMOE_OK;
}

int wmoe_ep_uses_copy_engines(const wmoe_ctx* ctx) {
  if (!ctx || !ctx->nccl_comm) return -1;
  return ctx->ep_ipc ? 1 : 0;
}

// The exchanges' barrier: a one-int all-reduce on stream st. Every rank issues it after its copies into the peers'
// windows (ordered on st), so when it completes on a rank, every copy into that rank's window has landed.
static int ep_barrier(wmoe_ctx* ctx, cudaStream_t st, const char* where) {
  WMOE_CHECK_NCCL(ctx, nccl().AllReduce(ctx->ep_flag, ctx->ep_flag, 1, ncclInt32, ncclSum,
                                        static_cast<ncclComm_t>(ctx->nccl_comm), st),
                  where);
  return WMOE_OK;
}

// Windows of at least `need` bytes on every rank. Every rank calls this with the same `need` (it is computed from the
// all-gathered counts), so all of them grow together: close the peers' old windows, free this one, allocate and
// export the new one, all-gather the handles, open the peers'. Nothing writes into the old windows any more: a call's
// copies into a rank's window end before that call's last barrier, and the growth comes after the next call's count
// exchange.
static int ep_grow_windows(wmoe_ctx* ctx, size_t need, cudaStream_t st) {
  if (need <= ctx->ep_win_bytes) return WMOE_OK;
  const int world = ctx->ep_world, rank = ctx->ep_rank;
  WMOE_CHECK_CUDA(ctx, cudaStreamSynchronize(st), "EP windows");
  for (int d = 0; d < int(ctx->ep_peer_win.size()); ++d)
    if (d != rank && ctx->ep_peer_win[size_t(d)]) cudaIpcCloseMemHandle(ctx->ep_peer_win[size_t(d)]);
  ctx->ep_peer_win.clear();
  // every rank has closed its mappings of the old windows before any frees one
  if (int rc = ep_barrier(ctx, st, "EP windows")) return rc;
  if (int rc = ep_wait(ctx, st, "EP windows")) return rc;
  cudaFree(ctx->ep_win);
  ctx->ep_win = nullptr;
  const size_t bytes = std::max(need + need / 4, size_t(64) << 20);
  WMOE_CHECK_CUDA(ctx, cudaMalloc(&ctx->ep_win, bytes), "EP window allocation");
  ctx->ep_win_bytes = bytes;
  cudaIpcMemHandle_t mine;
  WMOE_CHECK_CUDA(ctx, cudaIpcGetMemHandle(&mine, ctx->ep_win), "EP window export");
  char* staged = static_cast<char*>(ctx->ep_handles);
  WMOE_CHECK_CUDA(ctx, cudaMemcpyAsync(staged + size_t(rank) * sizeof(mine), &mine, sizeof(mine),
                                       cudaMemcpyHostToDevice, st),
                  "EP windows");
  WMOE_CHECK_NCCL(ctx, nccl().AllGather(staged + size_t(rank) * sizeof(mine), staged, sizeof(mine), ncclUint8,
                                        static_cast<ncclComm_t>(ctx->nccl_comm), st),
                  "EP windows");
  cudaIpcMemHandle_t* all = static_cast<cudaIpcMemHandle_t*>(ctx->ep_host_handles);  // pinned: the copy is async
  WMOE_CHECK_CUDA(ctx, cudaMemcpyAsync(all, staged, size_t(world) * sizeof(mine), cudaMemcpyDeviceToHost, st),
                  "EP windows");
  if (int rc = ep_wait(ctx, st, "EP windows")) return rc;
  ctx->ep_peer_win.assign(size_t(world), nullptr);
  for (int d = 0; d < world; ++d) {
    if (d == rank) {
      ctx->ep_peer_win[size_t(d)] = ctx->ep_win;
      continue;
    }
    WMOE_CHECK_CUDA(ctx, cudaIpcOpenMemHandle(&ctx->ep_peer_win[size_t(d)], all[d],
                                              cudaIpcMemLazyEnablePeerAccess),
                    "EP window import");
  }
  return WMOE_OK;
}

static int ensure_ep_buf(wmoe_ctx* ctx, size_t bytes) {
  if (bytes <= ctx->ep_buf_bytes) return WMOE_OK;
  if (ctx->ep_buf) {
    WMOE_CHECK_CUDA(ctx, cudaDeviceSynchronize(), "EP buffer resize");
    cudaFree(ctx->ep_buf);
    ctx->ep_buf = nullptr;
    ctx->ep_buf_bytes = 0;
  }
  const size_t grown = std::max(bytes + bytes / 4, size_t(1) << 24);
  WMOE_CHECK_CUDA(ctx, cudaMalloc(&ctx->ep_buf, grown), "EP buffer allocation");
  ctx->ep_buf_bytes = grown;
  return WMOE_OK;
}

// One all-to-all-v round on the communicator: block d of `send` (send_n[d] elements) goes to rank d, block s of `recv`
// (recv_n[s] elements) comes from rank s; blocks in rank order, counts in elements of `type`.
static int ep_alltoallv(wmoe_ctx* ctx, const void* send, const int64_t* send_n, void* recv, const int64_t* recv_n,
                        ncclDataType_t type, size_t elem, cudaStream_t st, const char* where) {
  // the rank's own block goes through NCCL too: inside one group its copy runs alongside the peer transfers
  // (a separate cudaMemcpyAsync after the group measured slower)
  const NcclApi& api = nccl();
  ncclComm_t comm = static_cast<ncclComm_t>(ctx->nccl_comm);
  size_t so = 0, ro = 0;
  // calls inside the group only queue; the group's end settles them
  auto queued = [](ncclResult_t r) { return r == ncclSuccess || r == ncclInProgress; };
  ncclResult_t r = api.GroupStart();
  for (int d = 0; d < ctx->ep_world && queued(r); ++d) {
    if (send_n[d] > 0)
      r = api.Send(static_cast<const char*>(send) + so * elem, size_t(send_n[d]), type, d, comm, st);
    if (recv_n[d] > 0 && queued(r))
      r = api.Recv(static_cast<char*>(recv) + ro * elem, size_t(recv_n[d]), type, d, comm, st);
    so += size_t(send_n[d]);
    ro += size_t(recv_n[d]);
  }
  const ncclResult_t end = api.GroupEnd();
  if (!queued(r)) return nccl_fail(ctx, r, where);
  WMOE_CHECK_NCCL(ctx, end, where);
  return WMOE_OK;
}

int wmoe_ep_set_chunks(wmoe_ctx* ctx, int chunks) {
  if (!ctx || chunks < 1 || chunks > kMaxEpChunks) return WMOE_ERR_INVALID;
  const int prev = ctx->ep_chunks;
  ctx->ep_chunks = chunks;
  return prev;
}

// The layer in C chunks of the rank's tokens so that the exchanges of some chunks overlap the expert stage of
// others: the exchanges run on the context's communication stream, the rest on the caller's stream, ordered by
// events. Chunks are planned first and their counts exchanged together (one host read of the transfer sizes).
static int moe_forward_ep_impl(wmoe_ctx* ctx, wmoe_store* store, int layer, const void* x, int x_dtype, int T,
                               int top_k, const wmoe_layer_weights* w, void* out, int out_dtype,
                               int32_t* topk_idx_out, float* topk_w_out, void* stream, const AddNorm* an) {
  if (!ctx) return WMOE_ERR_INVALID;
  if (ctx->ep_dead)
    return ctx_fail(ctx, WMOE_ERR_NCCL, "wmoe_moe_forward_ep: the communicator was aborted after a failure; "
                                        "wmoe_ep_finalize, then wmoe_ep_init again");
  if (!ctx->nccl_comm) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_moe_forward_ep: call wmoe_ep_init first");
  if (!store || store->ctx != ctx) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_moe_forward_ep: bad store");
  const int world = ctx->ep_world, rank = ctx->ep_rank, E = store->experts, H = store->hidden, F = store->ffn;
  if (E % world || store->expert_begin != rank * (E / world) || store->expert_end != (rank + 1) * (E / world))
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_moe_forward_ep: the store must hold this rank's block of experts");
  if (layer < 0 || layer >= store->layers || T < 0 || top_k != 8 || H != 2048 || F != 512 ||
      (x_dtype != WMOE_F32 && x_dtype != WMOE_BF16) || (out_dtype != WMOE_F32 && out_dtype != WMOE_BF16))
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_moe_forward_ep: bad layer, shape or dtype");
  if (int rc = check_layer(ctx, w, "wmoe_moe_forward_ep")) return rc;
  if (T > 0 && (!x || (!out && !an))) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_moe_forward_ep: null pointer");
  const cudaStream_t st = static_cast<cudaStream_t>(stream), cs = ctx->ep_stream;
  const int k = top_k, kw = std::min(k, world);
  // the chunk count is the context's setting only (never derived from local data): every rank must run the same
  // exchanges; the count exchange below checks it
  const int C = ctx->ep_chunks;
  auto chunk_begin = [&](int c) { return int(int64_t(T) * c / C); };
  const size_t xsz = x_dtype == WMOE_F32 ? 4 : 2, osz = out_dtype == WMOE_F32 ? 4 : 2;
  // stage A (sized by T) in the context scratch
  const bool tc = use_router_tc(w->router_split, x_dtype, T, H, E);
  const int max_chunk = (T + C - 1) / C + 1;
  Plan pa;
  const size_t o_logits = pa.take<float>(std::max<size_t>(router_logit_floats(tc, T, E, H), 1));
  const size_t o_w = pa.take<float>(size_t(T) * k + 1);
  const size_t o_idx = pa.take<int32_t>(size_t(T) * k + 1);
  const size_t o_s = pa.take<float>(size_t(T) + 1);
  // send [world][kCountWords] (per destination the chunk count, then (rows, pairs) of each chunk), then every rank's
  // send table all-gathered [world][world][kCountWords]
  const size_t o_cnt = pa.take<int32_t>(size_t(world + world * world) * kCountWords);
  const size_t o_tok = pa.take<int32_t>(size_t(T) * kw + 1);
  const size_t o_pl = pa.take<int32_t>(size_t(T) * k * 2 + 2);
  const size_t o_ret = pa.take<int32_t>(size_t(T) * k + 1);
  const size_t o_send = pa.take<uint16_t>(size_t(T) * kw * H + 8);
  const size_t o_plan = pa.take<char>(ep_plan_scratch_bytes(max_chunk, world));
  if (int rc = ensure_scratch(ctx, pa.bytes)) return rc;
  int n = 0;
  cudaEvent_t* marks = ctx->profile_calls > 0
                           ? &ctx->prof_events[size_t(ctx->profile_seq % uint64_t(ctx->profile_calls)) *
                                               wmoe_ctx::kProfMarks]
                           : nullptr;
  auto mark = [&](int i) {
    if (marks) cudaEventRecord(marks[i], st);
  };
  mark(0);
  float* topk_w = at<float>(ctx, o_w);
  int32_t* topk_idx = at<int32_t>(ctx, o_idx);
  float* shared_s = at<float>(ctx, o_s);
  int32_t* cnt_send = at<int32_t>(ctx, o_cnt);                    // [world][kCountWords]
  int32_t* cnt_all = cnt_send + size_t(world) * kCountWords;       // [source][destination][kCountWords]
  int32_t* send_tok = at<int32_t>(ctx, o_tok);
  int32_t* pair_list = at<int32_t>(ctx, o_pl);
  int32_t* ret_index = at<int32_t>(ctx, o_ret);
  uint16_t* send_buf = at<uint16_t>(ctx, o_send);
  WMOE_CHECK_CUDA(ctx, ep_count_header(cnt_send, world, kCountWords, C, st, &n), "EP plan");
  if (T > 0)
    WMOE_CHECK_CUDA(ctx,
                    route_tokens(tc, x, x_dtype, T, H, E, k, w->router_w, w->router_bias, w->shared_gate,
                                 w->router_split, at<float>(ctx, o_logits), topk_w, topk_idx, shared_s, ctx->d_status,
                                 st, &n, ctx->min_expert_weight),
                    "router");
  for (int c = 0; c < C; ++c) {
    const int t0 = chunk_begin(c), tn = chunk_begin(c + 1) - t0;
    if (tn == 0) continue;
    WMOE_CHECK_CUDA(ctx,
                    ep_plan(topk_idx + size_t(t0) * k, tn, k, E, world, cnt_send + 1 + 2 * c, cnt_send + 2 + 2 * c,
                            kCountWords,
                            send_tok + size_t(t0) * kw, pair_list + size_t(t0) * k * 2, ret_index + size_t(t0) * k,
                            at<void>(ctx, o_plan), ctx->d_status, st, &n),
                    "EP plan");
    WMOE_CHECK_CUDA(ctx,
                    ep_pack(static_cast<const char*>(x) + size_t(t0) * H * xsz, x_dtype, H, send_tok + size_t(t0) * kw,
                            cnt_send + 1 + 2 * c, kCountWords, world, tn * kw, send_buf + size_t(t0) * kw * H, st, &n),
                    "EP rows");
  }
  mark(1);
  // every rank's send table to every rank in one fixed-size all-gather, then one bounded read of all of it: each
  // rank then knows every transfer, so every rank computes the same window layouts
  ncclComm_t comm = static_cast<ncclComm_t>(ctx->nccl_comm);
  WMOE_CHECK_NCCL(ctx, nccl().AllGather(cnt_send, cnt_all, size_t(world) * kCountWords, ncclInt32, comm, st),
                  "EP counts");
  const size_t n_cnt = size_t(world) * world * kCountWords;
  // into pinned memory, so that the copy is asynchronous and the host's wait for it is ep_wait's bounded poll
  WMOE_CHECK_CUDA(ctx, cudaMemcpyAsync(ctx->ep_host_counts, cnt_all, n_cnt * sizeof(int32_t), cudaMemcpyDeviceToHost,
                                       st),
                  "EP counts read-back");
  if (int rc = ep_wait(ctx, st, "EP counts read-back")) return rc;
  const std::vector<int32_t> cnt(ctx->ep_host_counts, ctx->ep_host_counts + n_cnt);
  mark(2);
  auto A = [&](int s_, int d_, int i) { return cnt[(size_t(s_) * world + d_) * kCountWords + i]; };
  for (int s_ = 0; s_ < world; ++s_)
    for (int d_ = 0; d_ < world; ++d_)
      if (A(s_, d_, 0) != C)
        return ctx_fail(ctx, WMOE_ERR_INVALID,
                        "wmoe_moe_forward_ep: ranks use different chunk counts (wmoe_ep_set_chunks)");
  auto sr = [&](int d, int c) { return A(rank, d, 1 + 2 * c); };  // rows of chunk c to d
  auto sp = [&](int d, int c) { return A(rank, d, 2 + 2 * c); };  // pairs of chunk c to d
  auto rr = [&](int s_, int c) { return A(s_, rank, 1 + 2 * c); };  // rows from s
  auto rp = [&](int s_, int c) { return A(s_, rank, 2 + 2 * c); };  // pairs from s
  auto a256 = [](size_t b) { return (b + 255) / 256 * 256; };
  // rank q's window: per chunk the rows it receives, their pair lists, and the result rows that come back to it
  struct Layout {
    std::vector<size_t> rows, pairs, ret;
    size_t total = 0;
  };
  auto layout = [&](int q) {
    Layout L;
    for (int c = 0; c < C; ++c) {
      size_t R = 0, P = 0, S = 0;
      for (int o = 0; o < world; ++o) R += size_t(A(o, q, 1 + 2 * c)), P += size_t(A(o, q, 2 + 2 * c)),
                                      S += size_t(A(q, o, 2 + 2 * c));
      L.rows.push_back(L.total);
      L.total += a256(R * H * 2);
      L.pairs.push_back(L.total);
      L.total += a256(P * 8);
      L.ret.push_back(L.total);
      L.total += a256(S * H * 2);
    }
    return L;
  };
  std::vector<Layout> lay;
  size_t need = 0;
  for (int q = 0; q < world; ++q) {
    lay.push_back(layout(q));
    need = std::max(need, lay.back().total);
  }
  const bool ipc = ctx->ep_ipc;
  if (ipc)
    if (int rc = ep_grow_windows(ctx, need, st)) return rc;
  // stage B in the EP buffer: per chunk the expert results (and, on the NCCL path, the received and returned rows),
  // and one expert-stage scratch
  std::vector<size_t> o_y(C), o_recv(C), o_rpl(C), o_yret(C);
  std::vector<int> Pc(C), Tc(C), T0(C);
  Plan pb;
  size_t es = 0;
  for (int c = 0; c < C; ++c) {
    T0[c] = chunk_begin(c);
    Tc[c] = chunk_begin(c + 1) - T0[c];
    long long R = 0, P = 0, S = 0;
    std::vector<int32_t> rrow(static_cast<size_t>(world)), rpair(static_cast<size_t>(world));
    for (int d = 0; d < world; ++d) {
      R += rr(d, c), P += rp(d, c), S += sp(d, c);
      rrow[d] = rr(d, c), rpair[d] = rp(d, c);
    }
    if (int rc = check_ep_counts(ctx, world, rrow.data(), rpair.data(), Tc[c], "wmoe_moe_forward_ep")) return rc;
    Pc[c] = int(P);
    o_y[c] = pb.take<uint16_t>((size_t(P) + Tc[c]) * H + 8);
    if (!ipc) {
      o_recv[c] = pb.take<uint16_t>(size_t(R) * H + 8);
      o_rpl[c] = pb.take<int32_t>(size_t(P) * 2 + 2);
      o_yret[c] = pb.take<uint16_t>(size_t(S) * H + 8);
    }
    es = std::max(es, ep_experts_scratch_bytes(Pc[c], Tc[c], E, H, F));
  }
  const size_t o_es = pb.take<char>(es);
  if (int rc = ensure_ep_buf(ctx, pb.bytes)) return rc;
  char* eb = static_cast<char*>(ctx->ep_buf);
  char* win = static_cast<char*>(ctx->ep_win);
  auto recv_rows = [&](int c) { return ipc ? win + lay[rank].rows[c] : eb + o_recv[c]; };
  auto recv_pairs = [&](int c) { return ipc ? win + lay[rank].pairs[c] : eb + o_rpl[c]; };
  auto returned = [&](int c) { return ipc ? win + lay[rank].ret[c] : eb + o_yret[c]; };
  cudaEvent_t* ev = ctx->ep_events.data();  // [0] planned, then per chunk: rows arrived, results made, results back
  WMOE_CHECK_CUDA(ctx, cudaEventRecord(ev[0], st), "EP ordering");
  WMOE_CHECK_CUDA(ctx, cudaStreamWaitEvent(cs, ev[0], 0), "EP ordering");
  // copies of one exchange into the peers' windows, one stream per destination (the copy engines run them
  // together and take no SM), joined on the communication stream, then the barrier
  struct Copy {
    const char* src;
    char* dst;
    size_t bytes;
  };
  auto copy_out = [&](const std::vector<std::vector<Copy>>& per_dest, cudaEvent_t after, const char* where) -> int {
    for (int d = 0; d < world; ++d) {
      size_t total = 0;
      for (const Copy& cp : per_dest[size_t(d)]) total += cp.bytes;
      if (!total) continue;
      cudaStream_t ps = ctx->ep_peer_streams[size_t(d)];
      WMOE_CHECK_CUDA(ctx, cudaStreamWaitEvent(ps, after, 0), where);
      for (const Copy& cp : per_dest[size_t(d)])
        if (cp.bytes) WMOE_CHECK_CUDA(ctx, cudaMemcpyAsync(cp.dst, cp.src, cp.bytes, cudaMemcpyDeviceToDevice, ps), where);
      WMOE_CHECK_CUDA(ctx, cudaEventRecord(ctx->ep_peer_events[size_t(d)], ps), where);
      WMOE_CHECK_CUDA(ctx, cudaStreamWaitEvent(cs, ctx->ep_peer_events[size_t(d)], 0), where);
    }
    return ep_barrier(ctx, cs, where);
  };
  std::vector<int64_t> sn(static_cast<size_t>(world)), rn(static_cast<size_t>(world));
  // dispatch exchanges of every chunk, in order
  for (int c = 0; c < C; ++c) {
    const size_t t0 = size_t(T0[c]);
    if (ipc) {
      // rows and pair lists of every destination in one exchange: this rank's blocks sit after those of lower ranks
      std::vector<std::vector<Copy>> per_dest(static_cast<size_t>(world));
      size_t so_rows = 0, so_pairs = 0;
      for (int d = 0; d < world; ++d) {
        size_t rows_before = 0, pairs_before = 0;
        for (int o = 0; o < rank; ++o)
          rows_before += size_t(A(o, d, 1 + 2 * c)), pairs_before += size_t(A(o, d, 2 + 2 * c));
        char* w = static_cast<char*>(ctx->ep_peer_win[size_t(d)]);
        per_dest[size_t(d)].push_back({reinterpret_cast<const char*>(send_buf + (t0 * kw + so_rows) * H),
                                       w + lay[d].rows[c] + rows_before * H * 2, size_t(sr(d, c)) * H * 2});
        per_dest[size_t(d)].push_back({reinterpret_cast<const char*>(pair_list + (t0 * k + so_pairs) * 2),
                                       w + lay[d].pairs[c] + pairs_before * 8, size_t(sp(d, c)) * 8});
        so_rows += size_t(sr(d, c));
        so_pairs += size_t(sp(d, c));
      }
      if (int rc = copy_out(per_dest, ev[0], "EP dispatch")) return rc;
    } else {
      for (int d = 0; d < world; ++d) sn[d] = int64_t(sr(d, c)) * H, rn[d] = int64_t(rr(d, c)) * H;
      if (int rc = ep_alltoallv(ctx, send_buf + t0 * kw * H, sn.data(), recv_rows(c), rn.data(), ncclHalf, 2, cs,
                                "EP dispatch rows"))
        return rc;
      for (int d = 0; d < world; ++d) sn[d] = int64_t(sp(d, c)) * 2, rn[d] = int64_t(rp(d, c)) * 2;
      if (int rc = ep_alltoallv(ctx, pair_list + t0 * k * 2, sn.data(), recv_pairs(c), rn.data(), ncclInt32, 4, cs,
                                "EP dispatch pairs"))
        return rc;
    }
    WMOE_CHECK_CUDA(ctx, cudaEventRecord(ev[1 + 3 * c], cs), "EP ordering");
  }
  ctx->launches += uint64_t(n);
  n = 0;
  // SMs the persistent GEMMs leave free while exchanges overlap them: NCCL's send/recv kernels need many; on the
  // copy-engine path only the barriers' one-CTA all-reduces need room
  const int gemm_sms = world > 1 && C > 1 ? std::max(1, ctx->sm_count - (ipc ? kEpBarrierSms : kEpCommSms))
                                          : ctx->sm_count;
  // expert stage of each chunk once its rows are in; its results go back while the next chunk computes
  for (int c = 0; c < C; ++c) {
    WMOE_CHECK_CUDA(ctx, cudaStreamWaitEvent(st, ev[1 + 3 * c], 0), "EP ordering");
    if (c == 0) mark(3);
    std::vector<int32_t> rrow(static_cast<size_t>(world)), rpair(static_cast<size_t>(world));
    for (int d = 0; d < world; ++d) rrow[d] = rr(d, c), rpair[d] = rp(d, c);
    uint16_t* y = reinterpret_cast<uint16_t*>(eb + o_y[c]);
    if (int rc = ep_experts_impl(ctx, store, layer, world, rrow.data(), rpair.data(),
                                 reinterpret_cast<const uint16_t*>(recv_rows(c)),
                                 reinterpret_cast<const int32_t*>(recv_pairs(c)),
                                 static_cast<const char*>(x) + size_t(T0[c]) * H * xsz, x_dtype, Tc[c], w, y, eb + o_es,
                                 st, gemm_sms))
      return rc;
    WMOE_CHECK_CUDA(ctx, cudaEventRecord(ev[2 + 3 * c], st), "EP ordering");
    WMOE_CHECK_CUDA(ctx, cudaStreamWaitEvent(cs, ev[2 + 3 * c], 0), "EP ordering");
    if (ipc) {
      std::vector<std::vector<Copy>> per_dest(static_cast<size_t>(world));
      size_t yo = 0;
      for (int s_ = 0; s_ < world; ++s_) {  // results for source s into its return block, after lower ranks' blocks
        size_t before = 0;
        for (int o = 0; o < rank; ++o) before += size_t(A(s_, o, 2 + 2 * c));
        per_dest[size_t(s_)].push_back({reinterpret_cast<const char*>(y + yo * H),
                                        static_cast<char*>(ctx->ep_peer_win[size_t(s_)]) + lay[s_].ret[c] +
                                            before * H * 2,
                                        size_t(rp(s_, c)) * H * 2});
        yo += size_t(rp(s_, c));
      }
      if (int rc = copy_out(per_dest, ev[2 + 3 * c], "EP combine rows")) return rc;
    } else {
      for (int d = 0; d < world; ++d) sn[d] = int64_t(rp(d, c)) * H, rn[d] = int64_t(sp(d, c)) * H;
      if (int rc = ep_alltoallv(ctx, y, sn.data(), returned(c), rn.data(), ncclHalf, 2, cs, "EP combine rows"))
        return rc;
    }
    WMOE_CHECK_CUDA(ctx, cudaEventRecord(ev[3 + 3 * c], cs), "EP ordering");
  }
  mark(4);
  for (int c = 0; c < C; ++c) {
    WMOE_CHECK_CUDA(ctx, cudaStreamWaitEvent(st, ev[3 + 3 * c], 0), "EP ordering");
    if (c == C - 1) mark(5);
    if (Tc[c] == 0) continue;
    const size_t t0 = size_t(T0[c]);
    const uint16_t* y = reinterpret_cast<const uint16_t*>(eb + o_y[c]);
    AddNorm epi;  // the chunk's rows of the residual epilogue
    if (an) {
      epi = *an;
      epi.h += t0 * H;
      if (epi.xn) epi.xn = static_cast<char*>(epi.xn) + t0 * H * (epi.xn_dtype == WMOE_F32 ? 4 : 2);
    }
    WMOE_CHECK_CUDA(ctx,
                    combine_rows(Tc[c], k, H, topk_idx + t0 * k, topk_w + t0 * k, ret_index + t0 * k, shared_s + t0,
                                 reinterpret_cast<const __half*>(returned(c)),
                                 reinterpret_cast<const __half*>(y) + size_t(Pc[c]) * H,
                                 an ? nullptr : static_cast<char*>(out) + t0 * H * osz, out_dtype, epi, st, &n),
                    "EP combine");
  }
  if (T > 0) {
    if (topk_idx_out)
      WMOE_CHECK_CUDA(ctx, copy_picks(topk_idx, topk_w, topk_idx_out, T * k, ctx->min_expert_weight, st, &n),
                      "routing copy");
    if (topk_w_out)
      WMOE_CHECK_CUDA(ctx, cudaMemcpyAsync(topk_w_out, topk_w, size_t(T) * k * sizeof(float), cudaMemcpyDeviceToDevice,
                                           st),
                      "routing copy");
  }
  mark(6);
  if (marks) ++ctx->profile_seq;
  ctx->launches += uint64_t(n);
  return WMOE_OK;
}

int wmoe_moe_forward_ep(wmoe_ctx* ctx, wmoe_store* store, int layer, const void* x, int x_dtype, int T, int top_k,
                        const wmoe_layer_weights* w, void* out, int out_dtype, int32_t* topk_idx_out,
                        float* topk_w_out, void* stream) {
  return moe_forward_ep_impl(ctx, store, layer, x, x_dtype, T, top_k, w, out, out_dtype, topk_idx_out, topk_w_out,
                             stream, nullptr);
}

int wmoe_decode_stack(wmoe_ctx* ctx, wmoe_store* store, int layer_begin, int n_layers,
                      const wmoe_layer_weights* layers, float eps, const float* h_in, float* h_out,
                      int32_t* topk_idx_out, void* stream) {
  if (!ctx) return WMOE_ERR_INVALID;
  if (!store || store->ctx != ctx) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_decode_stack: bad store");
  if (store->capped) return ctx_fail(ctx, WMOE_ERR_UNSUPPORTED, "wmoe_decode_stack: needs every expert resident");
  if (layer_begin < 0 || n_layers <= 0 || layer_begin + n_layers > store->layers || !layers || !h_in || !h_out)
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_decode_stack: bad arguments");
  if (store->hidden != 2048 || store->ffn != 512 || store->experts != 256)
    return ctx_fail(ctx, WMOE_ERR_UNSUPPORTED, "wmoe_decode_stack: this build runs hidden 2048, ffn 512, 256 experts");
  if (ctx->decode_ctas <= 0)
    return ctx_fail(ctx, WMOE_ERR_UNSUPPORTED, "wmoe_decode_stack: the persistent kernel cannot be co-resident here");
  for (int i = 0; i < n_layers; ++i)
    if (!layers[i].router_w || !layers[i].shared_gate || !layers[i].shared_gate_up || !layers[i].shared_down)
      return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_decode_stack: null weight pointer in layers[]");
  for (int i = 0; i < n_layers; ++i)
    if (!aligned16(layers[i].router_packed))
      return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_decode_stack: a packed router must be 16-byte aligned");
  if (!aligned16(h_in)) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_decode_stack: h_in must be 16-byte aligned");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int rc = ensure_scratch(ctx, decode_scratch_bytes(store->hidden, store->ffn, store->experts, ctx->decode_ctas)))
    return rc;
  int n = 0;
  const ExpertSource src = store_source(store, layer_begin, nullptr, nullptr);
  const cudaError_t e = decode_persistent(src, store->down_type.data() + layer_begin, layer_begin, n_layers,
                                          reinterpret_cast<const DecodeLayer*>(layers), store->hidden, store->ffn,
                                          store->experts, 8, eps, true, h_in, WMOE_F32, h_out, WMOE_F32, topk_idx_out,
                                          nullptr, ctx->scratch, ctx->decode_ctas, ctx->d_status, ctx->trace,
                                          ctx->trace_entries, st, &n, ctx->min_expert_weight);
  ctx->launches += uint64_t(n);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "wmoe_decode_stack");
  return WMOE_OK;
}

int wmoe_decode_stack_noalloc(wmoe_ctx* ctx, wmoe_store* store, int layer_begin, int n_layers,
                              const wmoe_layer_weights* layers, float eps, const float* h_in, float* h_out,
                              int32_t* topk_idx_out, void* stream) {
  // Same work as wmoe_decode_stack; the scratch is the file-scope device array of decode.cu instead of the
  // context's cudaMalloc'd buffer, so nothing here allocates.
  if (!ctx) return WMOE_ERR_INVALID;
  if (!store || store->ctx != ctx) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_decode_stack_noalloc: bad store");
  if (store->capped)
    return ctx_fail(ctx, WMOE_ERR_UNSUPPORTED, "wmoe_decode_stack_noalloc: needs every expert resident");
  if (layer_begin < 0 || n_layers <= 0 || layer_begin + n_layers > store->layers || !layers || !h_in || !h_out)
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_decode_stack_noalloc: bad arguments");
  if (store->hidden != 2048 || store->ffn != 512 || store->experts != 256)
    return ctx_fail(ctx, WMOE_ERR_UNSUPPORTED,
                    "wmoe_decode_stack_noalloc: this build runs hidden 2048, ffn 512, 256 experts");
  if (ctx->decode_ctas <= 0)
    return ctx_fail(ctx, WMOE_ERR_UNSUPPORTED,
                    "wmoe_decode_stack_noalloc: the persistent kernel cannot be co-resident here");
  for (int i = 0; i < n_layers; ++i)
    if (!layers[i].router_w || !layers[i].shared_gate || !layers[i].shared_gate_up || !layers[i].shared_down)
      return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_decode_stack_noalloc: null weight pointer in layers[]");
  for (int i = 0; i < n_layers; ++i)
    if (!aligned16(layers[i].router_packed))
      return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_decode_stack_noalloc: a packed router must be 16-byte aligned");
  if (!aligned16(h_in))
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_decode_stack_noalloc: h_in must be 16-byte aligned");
  const size_t need = decode_scratch_bytes(store->hidden, store->ffn, store->experts, ctx->decode_ctas);
  if (need > static_scratch_bytes())
    return ctx_fail(ctx, WMOE_ERR_CAPACITY,
                    "wmoe_decode_stack_noalloc: needs " + std::to_string(need) + " bytes of scratch, more than the " +
                        std::to_string(static_scratch_bytes()) + "-byte static array");
  int current = -1;
  WMOE_CHECK_CUDA(ctx, cudaGetDevice(&current), "wmoe_decode_stack_noalloc");
  if (current != ctx->device)
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_decode_stack_noalloc: make the context's device current first");
  void* scratch = nullptr;
  WMOE_CHECK_CUDA(ctx, static_scratch(ctx->device, &scratch), "wmoe_decode_stack_noalloc: static scratch address");
  int n = 0;
  const ExpertSource src = store_source(store, layer_begin, nullptr, nullptr);
  const cudaError_t e = decode_persistent(src, store->down_type.data() + layer_begin, layer_begin, n_layers,
                                          reinterpret_cast<const DecodeLayer*>(layers), store->hidden, store->ffn,
                                          store->experts, 8, eps, true, h_in, WMOE_F32, h_out, WMOE_F32, topk_idx_out,
                                          nullptr, scratch, ctx->decode_ctas, ctx->d_status, nullptr, 0,
                                          static_cast<cudaStream_t>(stream), &n, ctx->min_expert_weight);
  ctx->launches += uint64_t(n);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "wmoe_decode_stack_noalloc");
  return WMOE_OK;
}

// The multi-token counterpart of wmoe_decode_stack. One residual + RMSNorm launch before the first layer; after
// that each layer's combine kernel adds its output to h and writes the next layer's input (the residual epilogue),
// so a layer is the router, dispatch and the expert kernels only.
int wmoe_prefill_stack(wmoe_ctx* ctx, wmoe_store* store, int layer_begin, int n_layers,
                       const wmoe_layer_weights* layers, float eps, const float* h_in, int T, int x_dtype,
                       float* h_out, void* stream) {
  if (!ctx) return WMOE_ERR_INVALID;
  if (!store || store->ctx != ctx) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_prefill_stack: bad store");
  if (layer_begin < 0 || n_layers <= 0 || layer_begin + n_layers > store->layers || !layers || T < 0 ||
      !(eps >= 0.f) || (x_dtype != WMOE_F32 && x_dtype != WMOE_BF16))
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_prefill_stack: bad arguments");
  for (int i = 0; i < n_layers; ++i)
    if (int rc = check_layer(ctx, &layers[i], "wmoe_prefill_stack")) return rc;
  // after wmoe_ep_init every layer runs over the context's expert-parallel communicator
  const bool ep = ctx->nccl_comm != nullptr;
  if (T == 0) {
    if (!ep) return WMOE_OK;
    // a rank without tokens still takes part in every layer's exchanges
    for (int i = 0; i < n_layers; ++i)
      if (int rc = moe_forward_ep_impl(ctx, store, layer_begin + i, nullptr, x_dtype, 0, 8, &layers[i], nullptr,
                                       x_dtype, nullptr, nullptr, stream, nullptr))
        return rc;
    return WMOE_OK;
  }
  if (!h_in || !h_out) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_prefill_stack: null pointer");
  if (!aligned16(h_in) || !aligned16(h_out))
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_prefill_stack: h_in and h_out must be 16-byte aligned");
  if (!ep && T == 1 && x_dtype == WMOE_F32 && !store->capped && ctx->use_decode_kernel &&
      ctx->decode_ctas > 0 && store->experts == 256) {
    bool packed = true;
    for (int i = 0; i < n_layers; ++i) packed = packed && aligned16(layers[i].router_packed);
    if (packed) return wmoe_decode_stack(ctx, store, layer_begin, n_layers, layers, eps, h_in, h_out, nullptr, stream);
  }
  const int H = store->hidden;
  const size_t need = size_t(T) * H * (x_dtype == WMOE_F32 ? 4 : 2);
  if (need > ctx->stack_xn_bytes) {
    if (ctx->stack_xn) {
      WMOE_CHECK_CUDA(ctx, cudaDeviceSynchronize(), "wmoe_prefill_stack: buffer resize");
      cudaFree(ctx->stack_xn);
      ctx->stack_xn = nullptr;
      ctx->stack_xn_bytes = 0;
    }
    WMOE_CHECK_CUDA(ctx, cudaMalloc(&ctx->stack_xn, need), "wmoe_prefill_stack: buffer allocation");
    ctx->stack_xn_bytes = need;
  }
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  void* xn = ctx->stack_xn;
  int n = 0;
  WMOE_CHECK_CUDA(ctx, add_rmsnorm(h_in, nullptr, WMOE_F32, T, H, eps, h_out, xn, x_dtype, st, &n),
                  "wmoe_prefill_stack: first norm");
  ctx->launches += uint64_t(n);
  for (int i = 0; i < n_layers; ++i) {
    const int l = layer_begin + i;
    const wmoe_layer_weights& w = layers[i];
    AddNorm an;
    an.h = h_out;
    an.xn = i + 1 < n_layers ? xn : nullptr;
    an.xn_dtype = x_dtype;
    an.eps = eps;
    const int rc = ep ? moe_forward_ep_impl(ctx, store, l, xn, x_dtype, T, 8, &w, nullptr, x_dtype, nullptr, nullptr,
                                            stream, &an)
                      : moe_forward_impl(ctx, store, l, xn, x_dtype, T, 8, w.router_w, w.router_bias, w.shared_gate,
                                         w.shared_gate_up, w.shared_down, w.router_packed, w.router_split, nullptr,
                                         x_dtype, nullptr, nullptr, stream, &an);
    if (rc) return rc;
    // a capped store copies the next layer's experts while this one computes (gguf/store.py:204-219)
    if (store->capped)
      if (int rc2 = wmoe_store_prefetch(store, i + 1 < n_layers ? l + 1 : layer_begin, nullptr, 0, stream)) return rc2;
  }
  return WMOE_OK;
}

size_t wmoe_ggml_row_bytes(int ggml_type, int k) { return ggml_row_bytes(ggml_type, k); }

// the checks every typed-kernel call shares; 0 when the call may go on
static int typed_args(wmoe_ctx* ctx, const char* fn, int type, int rows, int k) {
  if (ggml_row_bytes(type, k) == 0 || k % 32)
    return ctx_fail(ctx, ggml_row_bytes(type, 32 * 256) ? WMOE_ERR_INVALID : WMOE_ERR_UNSUPPORTED,
                    std::string(fn) + ": type " + std::to_string(type) + " with k = " + std::to_string(k) +
                        " is not a whole number of its blocks (or not a type of these kernels)");
  if (rows < 0) return ctx_fail(ctx, WMOE_ERR_INVALID, std::string(fn) + ": rows < 0");
  return 0;
}


int wmoe_gemv(wmoe_ctx* ctx, int ggml_type, const uint8_t* w, int rows, int k, const void* x, int x_dtype,
              int tokens, void* y, int y_dtype, void* stream) {
  if (!ctx) return WMOE_ERR_INVALID;
  if (int rc = typed_args(ctx, "wmoe_gemv", ggml_type, rows, k)) return rc;
  if (tokens < 1 || tokens > 8) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_gemv: tokens must be 1..8");
  if ((x_dtype != WMOE_F32 && x_dtype != WMOE_BF16) || (y_dtype != WMOE_F32 && y_dtype != WMOE_BF16))
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_gemv: x and y are f32 or bf16");
  if (rows == 0) return WMOE_OK;
  if (!w || !x || !y) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_gemv: null pointer");
  if ((reinterpret_cast<uintptr_t>(w) & 1) || !aligned16(x))
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_gemv: w must be 2-byte and x 16-byte aligned");
  const cudaError_t e = ggml_gemv(ggml_type, nullptr, w, nullptr, 1, 1, rows, k, x, x_dtype, tokens, y, y_dtype,
                                  ctx->d_status, static_cast<cudaStream_t>(stream));
  if (e == cudaErrorNotSupported)  // ggml_gemv / ggml_combine: the shared-memory budget, nothing else
    return ctx_fail(ctx, WMOE_ERR_UNSUPPORTED, "wmoe_gemv: the activations and a row tile of this k do not fit shared "
                                               "memory");
  if (e != cudaSuccess) return cuda_fail(ctx, e, "wmoe_gemv");
  ctx->launches += 1;
  return WMOE_OK;
}

int wmoe_gemv_batch(wmoe_ctx* ctx, int ggml_type, const uint8_t* const* weights, const int64_t* positions, int n,
                    int n_out, int rows, int k, const void* x, int x_dtype, void* y, int y_dtype, void* stream) {
  if (!ctx) return WMOE_ERR_INVALID;
  if (int rc = typed_args(ctx, "wmoe_gemv_batch", ggml_type, rows, k)) return rc;
  if (n < 0 || (!positions && n_out < n))
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_gemv_batch: n < 0, or n_out < n without positions");
  if ((x_dtype != WMOE_F32 && x_dtype != WMOE_BF16) || (y_dtype != WMOE_F32 && y_dtype != WMOE_BF16))
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_gemv_batch: x and y are f32 or bf16");
  if (n == 0 || rows == 0) return WMOE_OK;
  if (!weights || !x || !y) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_gemv_batch: null pointer");
  if (!aligned16(x)) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_gemv_batch: x must be 16-byte aligned");
  const cudaError_t e = ggml_gemv(ggml_type, weights, nullptr, positions, n, positions ? n_out : n, rows, k, x,
                                  x_dtype, 1, y, y_dtype, ctx->d_status, static_cast<cudaStream_t>(stream));
  if (e == cudaErrorNotSupported)  // ggml_gemv / ggml_combine: the shared-memory budget, nothing else
    return ctx_fail(ctx, WMOE_ERR_UNSUPPORTED, "wmoe_gemv_batch: the activations and a row tile of this k do not "
                                               "fit shared memory");
  if (e != cudaSuccess) return cuda_fail(ctx, e, "wmoe_gemv_batch");
  ctx->launches += 1;
  return WMOE_OK;
}

int wmoe_gemv_combine(wmoe_ctx* ctx, int ggml_type, const uint8_t* const* weights, const int64_t* perm, int n,
                      int n_route, int rows, int k, const void* x, const void* route_w, int dtype, void* y,
                      void* stream) {
  if (!ctx) return WMOE_ERR_INVALID;
  if (int rc = typed_args(ctx, "wmoe_gemv_combine", ggml_type, rows, k)) return rc;
  if (n < 1 || n_route < 1) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_gemv_combine: n and n_route must be >= 1");
  if (dtype != WMOE_F32 && dtype != WMOE_BF16)
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_gemv_combine: dtype is f32 or bf16");
  if (rows == 0) return WMOE_OK;
  if (!weights || !perm || !x || !route_w || !y)
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_gemv_combine: null pointer");
  if (!aligned16(x)) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_gemv_combine: x must be 16-byte aligned");
  const cudaError_t e = ggml_combine(ggml_type, weights, perm, n, n_route, rows, k, x, route_w, dtype, y,
                                     ctx->d_status, static_cast<cudaStream_t>(stream));
  if (e == cudaErrorNotSupported)  // ggml_gemv / ggml_combine: the shared-memory budget, nothing else
    return ctx_fail(ctx, WMOE_ERR_UNSUPPORTED, "wmoe_gemv_combine: a row tile of this k does not fit shared memory");
  if (e != cudaSuccess) return cuda_fail(ctx, e, "wmoe_gemv_combine");
  ctx->launches += 1;
  return WMOE_OK;
}

int wmoe_expert_gate(wmoe_ctx* ctx, const void* gate_up, int n, int ffn, void* out, void* stream) {
  if (!ctx) return WMOE_ERR_INVALID;
  if (n < 0 || ffn < 1) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_expert_gate: n < 0 or ffn < 1");
  if (n == 0) return WMOE_OK;
  if (!gate_up || !out) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_expert_gate: null pointer");
  WMOE_CHECK_CUDA(ctx, swiglu_bf16(gate_up, n, ffn, out, static_cast<cudaStream_t>(stream)), "wmoe_expert_gate");
  ctx->launches += 1;
  return WMOE_OK;
}

int wmoe_batched_decode_experts(wmoe_ctx* ctx, int gate_up_type, int down_type, int hidden, int ffn,
                                const uint64_t* gate_up_ptrs, const uint64_t* down_ptrs, const int64_t* perm, int n,
                                int n_route, const void* x, const void* route_w, void* y, void* stream) {
  if (!ctx) return WMOE_ERR_INVALID;
  if (int rc = typed_args(ctx, "wmoe_batched_decode_experts", gate_up_type, 2 * ffn, hidden)) return rc;
  if (int rc = typed_args(ctx, "wmoe_batched_decode_experts", down_type, hidden, ffn)) return rc;
  if (n < 1 || n > 256 || n_route < 1 || hidden < 1 || ffn < 1)
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_batched_decode_experts: n must be 1..256, n_route >= 1");
  if (!gate_up_ptrs || !down_ptrs || !perm || !x || !route_w || !y)
    return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_batched_decode_experts: null pointer");
  for (int i = 0; i < n; ++i)
    if (!gate_up_ptrs[i] || !down_ptrs[i] || perm[i] < 0 || perm[i] >= n_route)
      return ctx_fail(ctx, WMOE_ERR_INVALID,
                      "wmoe_batched_decode_experts: null matrix pointer or perm entry outside the routing weights");
  if (!aligned16(x)) return ctx_fail(ctx, WMOE_ERR_INVALID, "wmoe_batched_decode_experts: x must be 16-byte aligned");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  constexpr int kSlots = wmoe_ctx::kStageSlots, kWords = wmoe_ctx::kStageWords;
  if (!ctx->stage_host) {
    WMOE_CHECK_CUDA(ctx, cudaHostAlloc(&ctx->stage_host, sizeof(int64_t) * kSlots * kWords, cudaHostAllocDefault),
                    "wmoe_batched_decode_experts: staging");
    WMOE_CHECK_CUDA(ctx, cudaMalloc(&ctx->stage_dev, sizeof(int64_t) * kSlots * kWords),
                    "wmoe_batched_decode_experts: staging");
    for (cudaEvent_t& ev : ctx->stage_ev)
      WMOE_CHECK_CUDA(ctx, cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "wmoe_batched_decode_experts");
  }
  Plan plan;
  const size_t o_gu = plan.take<uint16_t>(size_t(n) * 2 * ffn);
  if (int rc = ensure_scratch(ctx, plan.bytes)) return rc;
  const int slot = ctx->stage_next;
  ctx->stage_next = (slot + 1) % kSlots;
  if (ctx->stage_used[slot])
    WMOE_CHECK_CUDA(ctx, cudaEventSynchronize(ctx->stage_ev[slot]), "wmoe_batched_decode_experts: staging");
  int64_t* host = ctx->stage_host + size_t(slot) * kWords;
  int64_t* dev = ctx->stage_dev + size_t(slot) * kWords;
  for (int i = 0; i < n; ++i) {
    host[i] = int64_t(gate_up_ptrs[i]);
    host[n + i] = int64_t(down_ptrs[i]);
    host[2 * n + i] = perm[i];
  }
  WMOE_CHECK_CUDA(ctx, cudaMemcpyAsync(dev, host, sizeof(int64_t) * 3 * size_t(n), cudaMemcpyHostToDevice, st),
                  "wmoe_batched_decode_experts: staging");
  void* gu = at<void>(ctx, o_gu);
  // gate_up, then the combine, which applies expert_gate as it loads the gate_up rows
  cudaError_t e = ggml_gemv(gate_up_type, reinterpret_cast<const uint8_t* const*>(dev), nullptr, nullptr, n, n,
                            2 * ffn, hidden, x, WMOE_BF16, 1, gu, WMOE_BF16, ctx->d_status, st);
  if (e == cudaSuccess)
    e = ggml_combine(down_type, reinterpret_cast<const uint8_t* const*>(dev + n), dev + 2 * n, n, n_route, hidden,
                     ffn, gu, route_w, WMOE_BF16, y, ctx->d_status, st, true);
  // the slot is released behind whatever was enqueued, also when a launch was refused
  cudaEventRecord(ctx->stage_ev[slot], st);
  ctx->stage_used[slot] = true;
  if (e == cudaErrorNotSupported)
    return ctx_fail(ctx, WMOE_ERR_UNSUPPORTED,
                    "wmoe_batched_decode_experts: a row tile of this k does not fit shared memory");
  if (e != cudaSuccess) return cuda_fail(ctx, e, "wmoe_batched_decode_experts");
  ctx->launches += 2;
  return WMOE_OK;
}

}  // extern "C"
