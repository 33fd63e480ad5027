// Internal launch interface between the C ABI (capi.cu) and the kernel files.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

namespace wmoe {

// Runs set() (kernel attribute calls) once per device of this process: function attributes belong to a device's
// context, so a process that drives several GPUs sets them on each. `done` holds one bit per device (0-63); a
// concurrent first call on one device sets the attributes twice, which is harmless. Only cudaGetDevice runs on
// later calls, so launches inside CUDA-graph capture make no attribute call.
template <typename F>
inline cudaError_t once_per_device(std::atomic<uint64_t>& done, F&& set) {
  int dev = 0;
  if (cudaError_t e = cudaGetDevice(&dev)) return e;
  const uint64_t bit = dev < 64 ? (uint64_t(1) << dev) : 0;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  const cudaError_t e = set();
  if (e == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

constexpr int kF32 = 0, kBF16 = 1, kF16 = 2;  // WMOE_F32/BF16/F16
constexpr int kGgmlQ4K = 12, kGgmlQ6K = 14;

// Where a layer's routed experts live: a slab of fixed-size slots and a [layers, experts] slot table
// (-1: not resident). The shared expert (id == experts) comes from its own pointers.
struct ExpertSource {
  const uint8_t* slab;
  const int32_t* slot_of;
  uint64_t slot_bytes;
  uint64_t gate_up_bytes;  // offset of down within a slot
  int experts;
  int n_slots;             // slots in the slab
  const uint8_t* shared_gate_up;
  const uint8_t* shared_down;
  int down_type;           // ggml type of the layer's down matrices, routed and shared: 14 Q6_K or 12 Q4_K
};

// Result of dispatch for T tokens with top-k routing, plus the shared expert as an extra segment.
// Positions 0..T*k-1 hold the routed (token, slot) pairs grouped by expert (ascending id, tokens ascending
// within an expert); positions T*k..T*k+T-1 are the shared expert's rows, one per token.
struct PairMap {
  int T, k, E;
  const int32_t* perm;    // [T*k] pair id (token*k + slot) at each position
  const int32_t* pos;     // [T*k] inverse: position of pair id
  const int32_t* used;    // [E+1] expert id of segment u; the last used segment is the shared expert (id E)
  const int32_t* seg;     // [E+2] first position of segment u; seg[n_used] = T*(k+1)
  const int32_t* n_used;  // [1]
};

__device__ __forceinline__ int pair_token(const PairMap& m, int p) {
  return p < m.T * m.k ? m.perm[p] / m.k : p - m.T * m.k;
}

// dequant.cu
cudaError_t dequant(int type, const uint8_t* blocks, size_t nblocks, void* out, int out_dtype, cudaStream_t st);

// norm.cu: x_out = x + y (y optional), xn = x_out * rsqrt(mean(x_out^2) + eps), per token row (H % 4 == 0)
cudaError_t add_rmsnorm(const float* x, const void* y, int y_dtype, int T, int H, float eps, float* x_out, void* xn,
                        int xn_dtype, cudaStream_t st, int* launches);

// route.cu: at most 8 tokens, logits [T, E+1] (column E = shared gate); then top-k
cudaError_t router_logits(const void* x, int x_dtype, int T, int H, int E, const float* router_w,
                          const float* shared_gate, float* logits, cudaStream_t st, int* launches);
cudaError_t router_topk(const float* logits, int T, int E, int k, const float* bias, float* topk_w,
                        int32_t* topk_idx, float* shared_s, float* logits_out, cudaStream_t st, int* launches);
cudaError_t router_topk_split(const float* logits, int splits, int T, int E, int k, const float* bias, float* topk_w,
                              int32_t* topk_idx, float* shared_s, float* logits_out, const void* x, int x_dtype,
                              const float* g, int H, cudaStream_t st, int* launches);

// willow's skip_small_experts on topk_w [T, k] in place (no-op for min_w <= 0): each token keeps its top pick and
// the picks of weight >= min_w, rescaled to the former total; dropped picks get weight 0 (their ids are kept).
cudaError_t skip_small_experts(float* topk_w, int T, int k, float min_w, cudaStream_t st, int* launches);
// out = idx with -1 where w == 0 (the picks skip_small_experts dropped)
cudaError_t mark_dropped(const int32_t* idx, const float* w, int32_t* out, int n, cudaStream_t st, int* launches);

// More than 8 tokens: float32 logits without the shared gate as router_slice_outputs(T, H) partial sums [n][T][E]
// over 128-wide K slices (one sum of all slices for large T), added in order by router_topk_split, which also forms
// the shared-gate logit. A token's logits do not depend on the other tokens of the call. H a multiple of 128.
int router_slice_outputs(int T, int H);
cudaError_t router_logits_sliced(const void* x, int x_dtype, int T, int H, int E, const float* R, float* out,
                                 cudaStream_t st, int* launches);

// router_sm100.cu: bf16 tokens x (float32 router as three bf16 terms) on the tensor cores, K split kRouterKSplit
// ways into partial logits [kRouterKSplit][T][E]
constexpr int kRouterKSplit = 4;
bool router_tc_supported(int T, int H, int E);
cudaError_t router_split(const float* router_w, int E, int H, void* out, cudaStream_t st);
cudaError_t router_logits_tc(const void* x_bf16, int T, int H, int E, const void* router_split3, float* partial,
                             int* status, cudaStream_t st, int* launches);

// dispatch.cu
size_t dispatch_scratch_bytes(int T, int E);
cudaError_t dispatch(const int32_t* topk_idx, int T, int k, int E, void* scratch, int32_t* counts,
                     int32_t* offsets, int32_t* perm, int32_t* pos, int32_t* used, int32_t* seg, int32_t* n_used,
                     int64_t* usage, int* status, cudaStream_t st, int* launches);
// The same with a shared-expert segment of shared_rows rows (instead of T) after the T * k routed positions.
cudaError_t dispatch_rows(const int32_t* topk_idx, int T, int k, int E, int shared_rows, void* scratch,
                          int32_t* counts, int32_t* offsets, int32_t* perm, int32_t* pos, int32_t* used,
                          int32_t* seg, int32_t* n_used, int64_t* usage, int* status, cudaStream_t st,
                          int* launches);

// The residual epilogue of a combine: between layers willow computes x + moe(rms_norm(x))
// (engines/qwen36/model.py:17-22, engines/base.py:27-32 with weight 1). With h set the combine adds its output to the
// residual row (h[t] += out[t], float32) instead of writing out, and when xn is set also writes the next layer's
// input xn[t] = h[t] / sqrt(mean(h[t]^2) + eps) in xn_dtype. xn may be the call's own input x: every kernel that
// reads x runs before the combine on the same stream.
struct AddNorm {
  float* h = nullptr;
  void* xn = nullptr;
  int xn_dtype = 0;
  float eps = 0.f;
};

// gemv.cu (small token counts per expert)
cudaError_t quant_rows(const void* x, int x_dtype, int rows, int K, int16_t* q, float* scale, int32_t* sum16,
                       cudaStream_t st, int* launches);
cudaError_t gate_up_gemv(const ExpertSource& src, int layer, const PairMap& pm, int H, int F, const int16_t* xq,
                         const float* xs, const int32_t* xsum16, float* h, int* status, cudaStream_t st,
                         int* launches);
cudaError_t down_gemv(const ExpertSource& src, int layer, const PairMap& pm, int H, int F, const int16_t* hq,
                      const float* hs, const int32_t* hsum16, float* y, int* status, cudaStream_t st,
                      int* launches);
cudaError_t combine(const PairMap& pm, int H, const float* topk_w, const float* shared_s, const float* y, void* out,
                    int out_dtype, const AddNorm& an, cudaStream_t st, int* launches);

// gemm_sm100.cu: tcgen05 grouped GEMMs for many tokens per expert (gate_up + SwiGLU, down) and the fp16 combine
size_t prefill_scratch_bytes(int T, int k, int E, int H, int F);
size_t prefill_gemm_scratch_bytes(size_t P, int E, int H, int F);
// The whole multi-token expert stage: gather, both GEMMs, combine. marks: 4 events recorded after gather, gate_up,
// down, combine (or null).
cudaError_t prefill_experts(const ExpertSource& src, int layer, const PairMap& pm, const int32_t* topk_idx, int H,
                            int F, const void* x, int x_dtype, const float* topk_w, const float* shared_s, void* out,
                            int out_dtype, const AddNorm& an, void* scratch, int num_sms, int* status,
                            const cudaEvent_t* marks, cudaStream_t st, int* launches);
// The two GEMMs over P gathered fp16 rows xg (run-of-8 order): y [P][H] fp16 (= down output / 32); routed pair
// positions p < n_routed are written at row out_rows[p] when out_rows is given. marks: 2 events (or null).
cudaError_t prefill_gemms(const ExpertSource& src, int layer, const PairMap& pm, size_t P, int H, int F,
                          const __half* xg, __half* y, const int32_t* out_rows, int n_routed, void* scratch,
                          int num_sms, int* status, const cudaEvent_t* marks, cudaStream_t st, int* launches);
// out[t] = sum over picks in ascending expert id of w * 32 * y_routed[rows[t][j]] + s_t * 32 * y_shared[t]
// (or the residual epilogue an, when an.h is set)
cudaError_t combine_rows(int T, int k, int H, const int32_t* topk_idx, const float* topk_w, const int32_t* rows,
                         const float* shared_s, const __half* y_routed, const __half* y_shared, void* out,
                         int out_dtype, const AddNorm& an, cudaStream_t st, int* launches);

// ep.cu: expert parallelism over up to kMaxRanks ranks (contiguous expert blocks)
constexpr int kMaxRanks = 8;
constexpr int kMaxEpChunks = 16;
constexpr int kCountWords = 1 + 2 * kMaxEpChunks;  // per rank in the EP count exchange: chunks, then rows / pairs
// SMs the persistent GEMMs leave free while exchanges overlap them, so that NCCL's kernels find room
constexpr int kEpCommSms = 16;
// the same on the copy-engine exchange path, where only the barriers' one-CTA all-reduces run beside the GEMMs
constexpr int kEpBarrierSms = 4;
size_t ep_plan_scratch_bytes(int T, int world);
cudaError_t ep_count_header(int32_t* cnt, int world, int words, int chunks, cudaStream_t st, int* launches);
// send_rows[d * count_stride], send_pairs[d * count_stride]: rows and pairs to rank d
cudaError_t ep_plan(const int32_t* topk_idx, int T, int k, int E, int world, int32_t* send_rows, int32_t* send_pairs,
                    int count_stride, int32_t* send_tok, int32_t* pair_list, int32_t* ret_index, void* scratch,
                    int* status, cudaStream_t st, int* launches);
cudaError_t ep_pack(const void* x, int x_dtype, int H, const int32_t* send_tok, const int32_t* send_rows,
                    int count_stride, int world, int max_rows, void* send_buf, cudaStream_t st, int* launches);
cudaError_t ep_fixup(const int32_t* pair_list, int P, int world, const int32_t* recv_rows, const int32_t* recv_pairs,
                     int32_t* pair_row, int32_t* pair_expert, cudaStream_t st, int* launches);
cudaError_t ep_gather(const int32_t* perm, const int32_t* pair_row, int P_r, const void* recv, const void* x,
                      int x_dtype, int T, int H, void* xg, cudaStream_t st, int* launches);

// decode.cu: persistent one-token decode (one layer or a stack)
struct DecodeLayer {
  const float* router_w;
  const float* router_bias;
  const float* shared_gate;
  const uint8_t* shared_gate_up;
  const uint8_t* shared_down;
  const float* router_packed;  // [H][kRouterStride] or null
  const void* router_split;    // bf16 [3][E][H] (router as three bf16 terms) or null
};
constexpr int kRouterStride = 264;
cudaError_t pack_router(const float* router_w, const float* shared_gate, int E, int H, float* out, cudaStream_t st);
size_t decode_scratch_bytes(int H, int F, int E, int num_ctas);
size_t static_scratch_bytes();
cudaError_t static_scratch(int device, void** ptr);  // the no-allocation entry point's scratch on a device
int decode_num_ctas(int device);
// down_types[i]: ggml type of layer layer_begin + i's down matrices (kGgmlQ6K or kGgmlQ4K). The scratch holds
// decode_scratch_bytes; each launch clears what it needs first.
cudaError_t decode_persistent(const ExpertSource& src, const int* down_types, int layer_begin, int n_layers,
                              const DecodeLayer* layers, int H, int F, int E, int k, float eps, bool stack,
                              const void* x_in, int x_dtype, void* out, int out_dtype, int32_t* topk_idx_out,
                              float* topk_w_out, void* scratch, int num_ctas, int* status, uint64_t* trace,
                              size_t trace_entries, cudaStream_t st, int* launches, float min_w = 0.f);

// store.cu: device generator
cudaError_t fill_synthetic(uint8_t* dst, uint64_t seed, const int32_t* layer_expert /*[n][2]*/, int n,
                           uint64_t dst_stride, int hidden, int ffn, cudaStream_t st);
cudaError_t fill_synthetic_one(uint8_t* dst, uint64_t seed, int layer, int expert, int hidden, int ffn,
                               cudaStream_t st);

// Typed expert kernels over ggml blocks (ggml_gemv.cu). Types: 6 Q5_0, 8 Q8_0, 12 Q4_K, 14 Q6_K, 18 IQ3_XXS,
// 20 IQ4_NL, 21 IQ3_S, 22 IQ2_S, 23 IQ4_XS, 42 Q2_0. ggml_row_bytes is 0 for another type or a k that is not a
// whole number of blocks.
size_t ggml_row_bytes(int type, int k);
cudaError_t ggml_dequant(int type, const uint8_t* blocks, size_t nblocks, void* out, int out_dtype, cudaStream_t st);
// y[(pos_i * tokens + t) * rows + r] = W_i[r] . x[t]; W_i = weights[i] (device array) or `single` when weights is
// null; pos_i = positions[i] (device, < n_out) or i
cudaError_t ggml_gemv(int type, const uint8_t* const* weights, const uint8_t* single, const int64_t* positions, int n,
                      int n_out, int rows, int k, const void* x, int x_dtype, int tokens, void* y, int y_dtype,
                      int* status, cudaStream_t st);
// y[r] = sum_i route_w[perm[i]] * (W_i[r] . x[i]) in order of i; dtype kBF16 rounds each product, scaled product
// and running sum to bf16 (engines/base.py:431-443), kF32 keeps float32. gated (kBF16 only): x holds bf16 gate_up
// rows [n][2k] and x[i] is willow's expert_gate of row i (engines/base.py:99-102), as swiglu_bf16 computes it
// willow's expert_gate on bf16 [n][2F] gate_up rows -> bf16 [n][F], rounded as torch's bf16 silu and product
cudaError_t swiglu_bf16(const void* gate_up, int n, int F, void* out, cudaStream_t st);
cudaError_t ggml_combine(int type, const uint8_t* const* weights, const int64_t* perm, int n, int n_route, int rows,
                         int k, const void* x, const void* route_w, int dtype, void* y, int* status,
                         cudaStream_t st,
                         bool gated = false);

}  // namespace wmoe
