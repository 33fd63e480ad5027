/*
 * wmoe.h - C ABI of libwmoe.so, the B200 (sm_100a) MoE block of willow's qwen35moe engine.
 *
 * Plain C: device pointers, sizes and a CUDA stream passed as void*. Every function returns WMOE_OK (0) or a
 * negative WMOE_ERR_* code; wmoe_last_error() gives the message of the last failure on a context. Nothing
 * aborts or exits. A context is used from one host thread.
 *
 * Each entry point names the willow interface it replaces (paths within the willow-v2 project):
 *   wmoe_dequant             gguf/quants.py:207-227 dequantize (Q4_K 73-92, Q6_K 104-116, the other types
 *                            27-195);
 *                            gguf/metal.py:217-228,357-363 dequant_<type> / dequantize_gpu
 *   wmoe_route               engines/base.py:91-97 route (+ the router linear, base.py:305-306,448,
 *                            and the shared-expert gate of base.py:104-107)
 *   wmoe_dispatch            engines/base.py:456-467,555-566 (selected.cpu / unique / nonzero grouping),
 *                            gguf/store.py:482-484 record_usage
 *   wmoe_moe_forward         engines/base.py:445-490 Engine.moe (each_expert 534-591,
 *                            batched_decode_experts 492-532, combine_decode_experts 431-443)
 *   wmoe_decode_stack        engines/qwen36/model.py:17-22 MoEEngine.forward's per-layer
 *                            x + moe(rms_norm(x)) for one decode token, all layers in one launch
 *   wmoe_prefill_stack       the same layer loop for a prompt of T tokens, residual + RMSNorm in each
 *                            layer's combine
 *   wmoe_store_*             gguf/store.py:41-536 ExpertStore (slabs, LRU, load_batches, prefetch,
 *                            record_usage) and gguf/mps_shared.mm:10-20 shared_empty (host staging)
 *   wmoe_ggml_row_bytes      gguf/metal.py:323-325 row_bytes
 *   wmoe_gemv                gguf/metal.py:189-215,327-334 gemv_<type> / gemv (GGMLWeight.linear, 365-408)
 *   wmoe_gemv_batch          gguf/metal.py:239-261,336-343 gemv_batch (several experts x one token)
 *   wmoe_gemv_combine        gguf/metal.py:263-291,345-355 gemv_combine (down + routing-weighted sum,
 *                            engines/base.py:492-532 batched_decode_experts)
 *   wmoe_expert_gate         engines/base.py:99-102 expert_gate (silu(gate) * up)
 *   wmoe_batched_decode_experts  engines/base.py:492-532 batched_decode_experts in one call (gemv_batch,
 *                            expert_gate, gemv_combine)
 */
#ifndef WMOE_H
#define WMOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define WMOE_OK 0
#define WMOE_ERR_INVALID (-1)     /* bad argument (null pointer, shape, dtype, alignment) */
#define WMOE_ERR_CUDA (-2)        /* a CUDA runtime call failed */
#define WMOE_ERR_CAPACITY (-3)    /* the expert store's cap cannot hold what one call needs */
#define WMOE_ERR_DEVICE (-4)      /* a kernel reported a bad index or a wait that ran out (device status) */
#define WMOE_ERR_UNSUPPORTED (-5) /* shape or type this build has no kernel for */
#define WMOE_ERR_IO (-6)          /* a host-side copy into the store failed or was short */
#define WMOE_ERR_NCCL (-7)        /* an NCCL call of the expert-parallel path failed */

/* element types of activations */
#define WMOE_F32 0
#define WMOE_BF16 1
#define WMOE_F16 2

/* ggml type ids (gguf/reader.py:14-48). The MoE block runs Q4_K gate_up with Q6_K or Q4_K down; wmoe_dequant and
 * the typed kernels (wmoe_gemv*) run every type of willow's Metal path (gguf/metal.py:295). */
#define WMOE_GGML_Q5_0 6
#define WMOE_GGML_Q8_0 8
#define WMOE_GGML_Q4_K 12
#define WMOE_GGML_Q6_K 14
#define WMOE_GGML_IQ3_XXS 18
#define WMOE_GGML_IQ4_NL 20
#define WMOE_GGML_IQ3_S 21
#define WMOE_GGML_IQ2_S 22
#define WMOE_GGML_IQ4_XS 23
#define WMOE_GGML_Q2_0 42

typedef struct wmoe_ctx wmoe_ctx;
typedef struct wmoe_store wmoe_store;

/* ---- context ---------------------------------------------------------------------------------------- */

/* Creates a context on a CUDA device (made current). Owns scratch buffers, grown on demand. */
int wmoe_init(int device, wmoe_ctx** out);
void wmoe_destroy(wmoe_ctx* ctx);
const char* wmoe_last_error(const wmoe_ctx* ctx);
/* Number of kernels this context has launched so far (for benchmark accounting). */
uint64_t wmoe_launch_count(const wmoe_ctx* ctx);
/* enable = 1 (default): wmoe_moe_forward runs single-token calls on an uncapped store with the persistent
 * decode kernel; 0: with the multi-launch GEMV path. Returns the previous setting. */
int wmoe_set_decode_kernel(wmoe_ctx* ctx, int enable);
/* wmoe_moe_forward runs calls of at least this many tokens (default 16) with the tcgen05 grouped GEMMs (fp16
 * weight tiles dequantised into TMEM, fp32 accumulation), fewer with the dequant-GEMV kernels. (Measured: at 16 and
 * 64 Zipf-routed tokens the GEMMs take 0.63x / 0.30x the time of the GEMV kernels, which re-read an expert's
 * weights for each of its tokens.)
 * Returns the previous value (or WMOE_ERR_INVALID for tokens < 1). */
int wmoe_set_prefill_threshold(wmoe_ctx* ctx, int tokens);
/* willow's --min-expert-weight (Engine.skip_small_experts, engines/base.py:413-429; main.py:37,108): with
 * weight > 0 every routing of this context keeps each token's top pick and its picks of renormalised weight >=
 * weight, scaled back up to the picks' former total; the others are dropped. Dropped picks come back as -1 in
 * topk_idx_out and with weight 0 in topk_w_out (wmoe_route: weight 0, id kept); their experts' outputs are added
 * with weight 0, which leaves the block's output what it is without them. weight in [0, 1); 0 (default) is off. */
int wmoe_set_min_expert_weight(wmoe_ctx* ctx, float weight);
/* Phase tracing of the persistent decode kernel (the role of willow's per-section Engine.tick timings,
 * engines/base.py:384-390): with trace non-null, each CTA writes %globaltimer nanoseconds at WMOE_TRACE_POINTS
 * points of every layer into trace[(layer * WMOE_TRACE_POINTS + point) * ctas + cta] (device memory of at least
 * layers * WMOE_TRACE_POINTS * ctas entries; ctas from wmoe_decode_ctas). Null turns it off. */
#define WMOE_TRACE_POINTS 16
int wmoe_set_trace(wmoe_ctx* ctx, uint64_t* trace, size_t entries);
int wmoe_decode_ctas(const wmoe_ctx* ctx);
/* Reads and clears the device status word: 0, or the first WMOE_ERR_DEVICE cause a kernel recorded
 * (1 = expert id out of range, 2 = expert not resident, 3 = grid barrier timed out, 4 = bad segment). */
int wmoe_device_status(wmoe_ctx* ctx, int* status, void* stream);

/* ---- quantised weights ------------------------------------------------------------------------------ */

/* Dequantises nblocks ggml blocks of any WMOE_GGML_* type (Q4_K: 144 B, Q6_K: 210 B, IQ2_S: 82 B ... per block of
 * 256 values; Q5_0, Q8_0, IQ4_NL: 32 values; Q2_0: 64) to out_dtype, nblocks x elements values.
 * F32 output is bit-identical to gguf/quants.py:dequantize; BF16/F16 are that value rounded to nearest even. */
int wmoe_dequant(wmoe_ctx* ctx, int ggml_type, const uint8_t* blocks, size_t nblocks, void* out, int out_dtype,
                 void* stream);

/* ---- router ----------------------------------------------------------------------------------------- */

/* logits = x . router_w^T (+ router_bias); softmax over experts, top_k largest, renormalised to sum 1
 * (norm_topk_prob); shared_s = sigmoid(x . shared_gate) when shared_gate is not null.
 * x: [T, hidden] of x_dtype. router_w: f32 [experts, hidden]. Outputs: topk_w f32 [T, top_k],
 * topk_idx int32 [T, top_k] (descending weight), shared_s f32 [T] (nullable), logits f32 [T, experts]
 * (nullable). */
int wmoe_route(wmoe_ctx* ctx, const void* x, int x_dtype, int T, int hidden, int experts, int top_k,
               const float* router_w, const float* router_bias, const float* shared_gate, float* topk_w,
               int32_t* topk_idx, float* shared_s, float* logits, void* stream);

/* Groups the T*top_k (token, slot) picks by expert, stably in token order: counts int32 [experts],
 * offsets int32 [experts + 1], perm int32 [T*top_k] (token*top_k + slot, expert-major), usage (nullable)
 * int64 [experts] += counts. */
int wmoe_dispatch(wmoe_ctx* ctx, const int32_t* topk_idx, int T, int top_k, int experts, int32_t* counts,
                  int32_t* offsets, int32_t* perm, int64_t* usage, void* stream);

/* ---- expert store ----------------------------------------------------------------------------------- */

/* An HBM store of layers x experts expert blobs (gate_up bytes then down bytes, the pack layout of
 * gguf/compiler.py:139-197). cap_bytes = 0: every blob resident. Otherwise at most cap_bytes of device slots;
 * blobs live in pinned host memory and are copied in on a side stream, least recently used evicted first.
 * gate_up is Q4_K [2*ffn, hidden]; down is Q6_K [hidden, ffn]. */
int wmoe_store_create(wmoe_ctx* ctx, int layers, int experts, int hidden, int ffn, size_t cap_bytes,
                      wmoe_store** out);
/* A store holding only experts [expert_begin, expert_end) of each layer (the block one rank owns under expert
 * parallelism); the others are never resident and are refused by upload / prepare / download. cap_bytes as above,
 * over the held blobs only (so is the pinned host copy). wmoe_store_create is the range [0, experts). */
int wmoe_store_create_range(wmoe_ctx* ctx, int layers, int experts, int expert_begin, int expert_end, int hidden,
                            int ffn, size_t cap_bytes, wmoe_store** out);
void wmoe_store_destroy(wmoe_store* store);
/* Copies one blob (gate_up then down, size wmoe_store_blob_bytes) from host memory into the store. */
int wmoe_store_upload(wmoe_store* store, int layer, int expert, const void* host_src, void* stream);
/* Generates every blob of layers [layer_begin, layer_end) on the device from a seed (the generator of
 * willow_v2_b200/synth.py), in the store's resident slots or its host copy when capped. */
int wmoe_store_fill_synthetic(wmoe_store* store, uint64_t seed, int layer_begin, int layer_end, void* stream);
size_t wmoe_store_blob_bytes(const wmoe_store* store);
/* Sets a layer's down-matrix type (routed experts and the shared expert): 14 Q6_K (the default) or 12 Q4_K, as
 * llama.cpp's Q4_K_M files store some layers (gguf/compiler.py:42-44 records the type per layer). Set it before
 * uploading the layer: a Q4_K layer's blob is gate_up then H rows of 288 bytes (wmoe_store_layer_blob_bytes).  Every
 * kernel runs both: the grouped GEMMs, the dequant-GEMV kernels and the persistent decode kernel (stacks may mix
 * the two types layer by layer). */
int wmoe_store_set_down_type(wmoe_store* store, int layer, int ggml_type);
size_t wmoe_store_layer_blob_bytes(const wmoe_store* store, int layer);
/* Makes the given experts of a layer resident (copies misses from the host copy on the store's side stream;
 * the compute stream waits for them). Returns WMOE_ERR_CAPACITY if they cannot all fit at once. */
int wmoe_store_prepare(wmoe_store* store, int layer, const int32_t* experts, int n, void* stream);
/* Starts copying the given experts of a coming layer without making the compute stream wait; the call that uses
 * them waits for those copies only. experts null: the experts this layer has been routed to before, most used
 * first (every expert of the layer the store holds when there is no history yet). Takes only slots that neither
 * the last call nor a pending prefetch holds, and copies as many as fit, in the order given; unused ones become
 * ordinary cached slots once their layer runs. Replaces ExpertStore.prefetch and collect_prefetches
 * (gguf/store.py:204-232). No-op on an uncapped store. */
int wmoe_store_prefetch(wmoe_store* store, int layer, const int32_t* experts, int n, void* stream);
/* Picks the hot set: the `share` of the slots (0..1) that go to the experts routed the most tokens so far (counted
 * by every call on a capped store); they are evicted only when no other slot can go. Replaces
 * ExpertStore.choose_hot and record_usage (gguf/store.py:464-484). */
int wmoe_store_choose_hot(wmoe_store* store, double share);
/* Counters: experts copied by prefetches, and how many of those a call read before they were evicted. */
int wmoe_store_prefetch_stats(const wmoe_store* store, uint64_t* prefetched, uint64_t* prefetch_used);
/* Copies one blob back to host memory (from its slot, or the host copy of a capped store); synchronous. */
int wmoe_store_download(wmoe_store* store, int layer, int expert, void* host_dst, void* stream);
/* Device address of a resident blob, or null. */
const uint8_t* wmoe_store_blob(const wmoe_store* store, int layer, int expert);
/* Counters: hits, misses (copies), bytes copied host->device, evictions. */
int wmoe_store_stats(const wmoe_store* store, uint64_t* hits, uint64_t* misses, uint64_t* bytes_in,
                     uint64_t* evictions);

/* Per-phase device time of the multi-token MoE block, by CUDA events (opt-in, for benchmarks and profiling; no
 * counterpart in willow, whose engine times phases on the host with Engine.tick, engines/base.py:445-491). After
 * wmoe_set_profiling(ctx, calls), every wmoe_moe_forward(_layer) call with more than one token records its phase
 * boundaries on its own stream into slot (call number % calls); calls = 0 turns it off and frees the events.
 * wmoe_phase_ms gives phase `phase` of the call `ago` calls back (0 = the latest): 0 router + top-k, 1 dispatch,
 * 2 gather (GEMM path) or activation quantisation (GEMV path), 3 gate_up, 4 down, 5 combine. It waits for that
 * call's events. wmoe_moe_forward_ep records its own six on the caller's stream: 0 route + plan + rows, 1 count
 * exchange and read-back, 2 wait for the first chunk's rows, 3 expert stages (the other exchanges overlap them),
 * 4 wait for the last results, 5 combine. */
#define WMOE_PHASES 6
int wmoe_set_profiling(wmoe_ctx* ctx, int calls);
int wmoe_phase_ms(wmoe_ctx* ctx, int ago, int phase, float* ms);

/* ---- the MoE block ---------------------------------------------------------------------------------- */

/* One MoE block on T tokens: out = sum over each token's top_k experts (ascending expert id) of
 * w * down(silu(gate x) * up x), plus sigmoid(x . shared_gate) * shared(x).
 * x: [T, hidden] (x_dtype F32 or BF16). router_w f32 [experts, hidden]; router_bias f32 [experts] (nullable);
 * shared_gate f32 [hidden]; shared_gate_up / shared_down: the shared expert's Q4_K / Q6_K bytes on the device.
 * out: [T, hidden] of out_dtype (F32 or BF16). topk_idx_out int32 [T, top_k] and topk_w_out f32 [T, top_k]
 * are optional copies of the routing. Routed experts come from the store (all must be resident, or the store
 * must be able to stream them: capped stores synchronise on the routing once per call). */
int wmoe_moe_forward(wmoe_ctx* ctx, wmoe_store* store, int layer, const void* x, int x_dtype, int T, int top_k,
                     const float* router_w, const float* router_bias, const float* shared_gate,
                     const uint8_t* shared_gate_up, const uint8_t* shared_down, void* out, int out_dtype,
                     int32_t* topk_idx_out, float* topk_w_out, void* stream);

/* Per-layer weights of a decode stack (device pointers): one entry per layer. */
typedef struct wmoe_layer_weights {
    const float* router_w;          /* f32 [experts, hidden] */
    const float* router_bias;       /* f32 [experts] or null */
    const float* shared_gate;       /* f32 [hidden] */
    const uint8_t* shared_gate_up;  /* Q4_K [2*ffn, hidden] */
    const uint8_t* shared_down;     /* Q6_K [hidden, ffn] */
    const float* router_packed;     /* f32 [hidden, WMOE_ROUTER_STRIDE] from wmoe_pack_router, or null */
    const uint16_t* router_split;   /* bf16 [3, experts, hidden] from wmoe_split_router, or null */
} wmoe_layer_weights;

/* The router and the shared-expert gate transposed into one [hidden, WMOE_ROUTER_STRIDE] f32 matrix: column e < experts
 * is router row e, column experts is the shared gate, the rest zero. A layout transform done once at load (like
 * willow's pack step, gguf/compiler.py:90-137); with it every CTA of the decode kernel reads its slice of rows as one
 * contiguous block. out: device memory of hidden * WMOE_ROUTER_STRIDE floats. experts <= 263. */
#define WMOE_ROUTER_STRIDE 264
int wmoe_pack_router(wmoe_ctx* ctx, const float* router_w, const float* shared_gate, int experts, int hidden,
                     float* out, void* stream);

/* The router as three bf16 terms, R = R1 + R2 + R3 (R1 = bf16(R), R2 = bf16(R - R1), R3 = bf16(R - R1 - R2)),
 * stored [3, experts, hidden]: a layout transform done once at load, like wmoe_pack_router. With it,
 * wmoe_moe_forward_layer computes the router logits of bf16 tokens on the tensor cores with float32 accuracy
 * (bf16 x R_i products are exact in the float32 accumulator); without it the router runs in float32 on the CUDA
 * cores. out: device memory of 3 * experts * hidden bf16 values. */
int wmoe_split_router(wmoe_ctx* ctx, const float* router_w, int experts, int hidden, uint16_t* out, void* stream);

/* wmoe_moe_forward with the layer's weights as one wmoe_layer_weights (device pointers), so that prepared forms
 * (router_split) can be used. Same semantics, arguments and errors as wmoe_moe_forward, which it generalises:
 * the MoE block of engines/base.py:445-491 reads all of a layer's weights under one name prefix in the same way. */
int wmoe_moe_forward_layer(wmoe_ctx* ctx, wmoe_store* store, int layer, const void* x, int x_dtype, int T, int top_k,
                           const wmoe_layer_weights* weights, void* out, int out_dtype, int32_t* topk_idx_out,
                           float* topk_w_out, void* stream);

/* ---- expert parallelism --------------------------------------------------------------
 * willow runs on one device and has no counterpart; these replace its single-device MoE block
 * (engines/base.py:445-491) when `world` ranks share the experts. Rank r owns experts
 * [r * experts / world, (r + 1) * experts / world) of every layer, in a store from wmoe_store_create_range, and
 * routes its own T tokens. One layer on every rank:
 *   1. wmoe_ep_route_plan: route, then for each rank d the tokens with a pick on d (send_rows[d] rows, each token
 *      once) and those picks (send_pairs[d] pairs, (row within d's block, expert id) int32 pairs).
 *   2. all-to-all of the counts, then of the rows (fp16 [rows][hidden], send_buf) and pair lists, blocks in rank order.
 *   3. wmoe_ep_experts on what arrived: y rows 0 .. P_r - 1 (one fp16 row per received pair, in arrival order) and
 *      y rows P_r .. P_r + T - 1 (the shared expert on this rank's own tokens).
 *   4. all-to-all of y rows 0 .. P_r - 1 back to their senders (send_pairs[d] rows from rank d, in rank order).
 *   5. wmoe_ep_combine: out[t] = sum of the token's picks in ascending expert id + the shared expert, the same
 *      arithmetic in the same order as wmoe_moe_forward, so the output does not depend on `world`.
 * The transfers are the caller's (willow_v2_b200.moe.moe_forward_ep uses torch.distributed over NCCL). Rows are fp16
 * in the library's internal layout (elements permuted within runs of 8; results scaled by 1/32). */
#define WMOE_MAX_RANKS 8
int wmoe_ep_route_plan(wmoe_ctx* ctx, int world, const void* x, int x_dtype, int T, int top_k, int experts,
                       int hidden, const wmoe_layer_weights* weights, float* topk_w /* [T, top_k] */,
                       int32_t* topk_idx /* [T, top_k] */, float* shared_s /* [T] */,
                       int32_t* send_rows /* [world] */, int32_t* send_pairs /* [world] */,
                       int32_t* send_tok /* [T * min(top_k, world)] */, int32_t* pair_list /* [T * top_k, 2] */,
                       int32_t* ret_index /* [T, top_k] */, uint16_t* send_buf /* fp16 [T * min(top_k, world), hidden] */,
                       void* stream);
/* The same layer in one call over the library's own NCCL communicator: each rank passes its own tokens and gets
 * their outputs, identical to wmoe_moe_forward on one GPU. Per layer one all-gather of every rank's transfer counts
 * (one bounded host read of them); the rows, pair lists and result rows are copied by the copy engines straight
 * into the destination rank's exchange window (device memory every rank maps through CUDA IPC; made on first use
 * and grown together by every rank), one stream per destination, each exchange closed by a one-int all-reduce as
 * barrier. No kernel reads another GPU's memory. With WMOE_EP_NCCL_ROWS set in the environment at wmoe_ep_init
 * the rows go through grouped ncclSend/ncclRecv instead. wmoe_ep_unique_id (one rank) makes the id every rank passes to
 * wmoe_ep_init(ctx, id, rank, world), which creates the communicator (collectively); wmoe_ep_finalize (or
 * wmoe_destroy) frees it. NCCL is loaded at run time (libnccl.so.2); without it wmoe_ep_init returns
 * WMOE_ERR_UNSUPPORTED. Arguments of wmoe_moe_forward_ep as in wmoe_moe_forward_layer; store from
 * wmoe_store_create_range holding this rank's block. */
int wmoe_ep_unique_id(void* out /* WMOE_EP_ID_BYTES */);
#define WMOE_EP_ID_BYTES 128
int wmoe_ep_init(wmoe_ctx* ctx, const void* unique_id, int rank, int world);
int wmoe_ep_finalize(wmoe_ctx* ctx);
/* Failure handling: the communicator is non-blocking, and every host wait on it (the creation, the count read-back
 * of each wmoe_moe_forward_ep, the exchange windows' set-up) is bounded by this many milliseconds (default 30000)
 * while the communicator is watched for asynchronous errors. A rank that left, or any NCCL error, aborts the
 * communicator (its kernels in flight return) and the call returns WMOE_ERR_NCCL; every later EP call of the context
 * does so too until wmoe_ep_finalize and a new wmoe_ep_init. Returns the previous value. No counterpart in willow,
 * which runs on one device. */
int wmoe_ep_set_timeout(wmoe_ctx* ctx, int ms);
/* wmoe_moe_forward_ep runs the rank's tokens in this many chunks (1..16; wmoe_ep_init sets 1 below four ranks and 2
 * from four) so that the exchanges of one chunk overlap the expert stage of another (the exchanges then run on a
 * stream of the context, and the GEMMs leave SMs free for them). Every rank must use the same value: the count exchange carries it, and a mismatch makes every
 * rank's call return WMOE_ERR_INVALID. The result does not depend on it. Chunks pay off when each expert still gets
 * ~256 tokens per chunk (the tensor cores' cost per instruction is fixed up to N = 192). Returns the previous value. */
int wmoe_ep_set_chunks(wmoe_ctx* ctx, int chunks);
/* 1 when the context's exchanges copy the rows with the copy engines into the peers' windows, 0 when they go through
 * NCCL send/recv (WMOE_EP_NCCL_ROWS set at wmoe_ep_init), -1 without a communicator. */
int wmoe_ep_uses_copy_engines(const wmoe_ctx* ctx);
int wmoe_moe_forward_ep(wmoe_ctx* ctx, wmoe_store* store, int layer, const void* x, int x_dtype, int T, int top_k,
                        const wmoe_layer_weights* weights, void* out, int out_dtype, int32_t* topk_idx_out,
                        float* topk_w_out, void* stream);

/* recv_rows / recv_pairs: HOST arrays [world] (what each rank sent here); recv_buf fp16 [sum recv_rows, hidden];
 * recv_pair_list [sum recv_pairs, 2]; x [T, hidden] this rank's own tokens; y fp16 [sum recv_pairs + T, hidden]. */
int wmoe_ep_experts(wmoe_ctx* ctx, wmoe_store* store, int layer, int world, const int32_t* recv_rows,
                    const int32_t* recv_pairs, const uint16_t* recv_buf, const int32_t* recv_pair_list,
                    const void* x, int x_dtype, int T, const wmoe_layer_weights* weights, uint16_t* y, void* stream);
/* y_returned fp16 [sum send_pairs, hidden] (blocks in rank order); y_shared fp16 [T, hidden] (rows P_r.. of y). */
int wmoe_ep_combine(wmoe_ctx* ctx, int T, int top_k, int hidden, const int32_t* topk_idx, const float* topk_w,
                    const int32_t* ret_index, const float* shared_s, const uint16_t* y_returned,
                    const uint16_t* y_shared, void* out, int out_dtype, void* stream);

/* One decode token through layers [layer_begin, layer_begin + n_layers) of the store:
 * h <- h + moe_l(rms_norm(h)) per layer (eps, unit weight), in one persistent launch per 64 layers.
 * h_in / h_out: f32 [hidden] on the device (may alias). layers: HOST array of n_layers entries whose pointers
 * are device pointers. topk_idx_out: optional int32 [n_layers, top_k]. Needs every routed expert resident
 * (cap 0). */
int wmoe_decode_stack(wmoe_ctx* ctx, wmoe_store* store, int layer_begin, int n_layers,
                      const wmoe_layer_weights* layers, float eps, const float* h_in, float* h_out,
                      int32_t* topk_idx_out, void* stream);

/* wmoe_decode_stack for callers that cannot allocate device memory: it has no counterpart in willow. It calls no
 * cudaMalloc/cudaFree and no allocating library routine. Its scratch is a fixed file-scope device array of
 * WMOE_NOALLOC_SCRATCH_BYTES that every GPU loading the library holds until the process exits. Shapes needing more
 * scratch are refused with WMOE_ERR_CAPACITY.
 *
 * Who needs it: code that runs where allocation is not allowed or not safe, for example
 *   - a caller issuing work while a CUDA graph is being captured on its stream (cudaMalloc there fails or breaks
 *     the capture);
 *   - an engine whose device memory is owned by a pool allocator it must not bypass;
 *   - a latency-critical decode loop that must never hit a growing scratch buffer (wmoe_decode_stack grows the
 *     context's scratch with cudaMalloc on first use).
 *
 * The first call on each device looks up the array's device address (cudaGetSymbolAddress); make that first call
 * before any stream capture. Every call on a device shares the one array, which keeps the last call's contents (the
 * kernel zeroes what must start at zero), so calls that overlap on the GPU - on different streams, or from
 * different contexts of one process on the same device - race and must be serialised by the caller. */
#define WMOE_NOALLOC_SCRATCH_BYTES (160u * 1024u)
int wmoe_decode_stack_noalloc(wmoe_ctx* ctx, wmoe_store* store, int layer_begin, int n_layers,
                              const wmoe_layer_weights* layers, float eps, const float* h_in, float* h_out,
                              int32_t* topk_idx_out, void* stream);

/* T tokens through layers [layer_begin, layer_begin + n_layers) of the store: h <- h + moe_l(rms_norm(h)) per layer
 * (eps, unit weight), MoEEngine.forward's layer loop (engines/qwen36/model.py:17-22) for a prompt. One residual +
 * RMSNorm launch before the first layer; after it every layer's combine kernel adds the block output to h and
 * writes the next layer's normalised input (no separate residual + RMSNorm pass between layers). Each block takes
 * its input in x_dtype (WMOE_BF16: tensor-core router when layers[i].router_split is set, and the grouped GEMMs; or
 * WMOE_F32) and computes as wmoe_moe_forward_layer does, min_expert_weight included. h_in / h_out: f32 [T, hidden]
 * on the device, 16-byte aligned, may alias. layers: HOST array of n_layers entries of device pointers.
 *   - After wmoe_ep_init every layer runs as wmoe_moe_forward_ep does, over the context's communicator: the store
 *     holds this rank's block of the experts (wmoe_store_create_range) and every rank calls with its own tokens
 *     (T may be 0: the rank still takes part in every layer's exchanges).
 *   - A capped store starts copying the next layer's experts (wmoe_store_prefetch with its guess) once a layer is
 *     issued, and the first layer's after the last.
 *   - One f32 token on a resident store runs wmoe_decode_stack.
 * The context keeps the T x hidden rows passed between layers (grown on first use). */
int wmoe_prefill_stack(wmoe_ctx* ctx, wmoe_store* store, int layer_begin, int n_layers,
                       const wmoe_layer_weights* layers, float eps, const float* h_in, int T, int x_dtype,
                       float* h_out, void* stream);

/* Residual add + RMS normalisation between MoE layers (engines/qwen36/model.py:17-22, engines/base.py:27-32,
 * weight 1): x_out = x + y (y optional, f32 or bf16), xn_out = x_out / sqrt(mean(x_out^2) + eps) as f32 or bf16.
 * x, x_out f32 [T, hidden]; x_out may be x. 16-byte aligned buffers, hidden % 4 == 0. */
int wmoe_add_rmsnorm(wmoe_ctx* ctx, const float* x, const void* y, int y_dtype, int T, int hidden, float eps,
                     float* x_out, void* xn_out, int xn_dtype, void* stream);

/* ---- typed expert kernels (gguf/metal.py) ----------------------------------------------------------- */
/* Matrices are [rows, k] ggml blocks, rows back to back (a row is wmoe_ggml_row_bytes(type, k) bytes) at an even
 * address; k is a multiple of 32 and of the type's block. Sums are float32; x, y, route_w are f32 or bf16 (16-byte
 * aligned). An out-of-range position or perm entry, or an odd matrix address, sets the device status
 * (wmoe_device_status) and that matrix is skipped. A CTA holds its activations (about 2.3 bytes per value: tokens x k
 * for gemv, n x k for the combine) and a tile of rows in at most 200 KB of shared memory; calls beyond that return
 * WMOE_ERR_UNSUPPORTED. */

/* Bytes of one row of k values; 0 for a type these kernels do not run or a k that is not a whole number of blocks. */
size_t wmoe_ggml_row_bytes(int ggml_type, int k);

/* y [tokens, rows] = x [tokens, k] . W^T for 1 <= tokens <= 8 (gguf/metal.py:189-215 gemv_<type>). */
int wmoe_gemv(wmoe_ctx* ctx, int ggml_type, const uint8_t* w, int rows, int k, const void* x, int x_dtype,
              int tokens, void* y, int y_dtype, void* stream);

/* Several matrices times one token: y[positions[i]] = W_i x for i < n (gguf/metal.py:239-261 gemv_batch_<type>).
 * weights: device array of n device pointers; positions: device int64 [n] with entries < n_out, or null for i
 * (n_out >= n); x [k]; y [n_out, rows]. */
int wmoe_gemv_batch(wmoe_ctx* ctx, int ggml_type, const uint8_t* const* weights, const int64_t* positions, int n,
                    int n_out, int rows, int k, const void* x, int x_dtype, void* y, int y_dtype, void* stream);

/* y [rows] = sum over i < n, in order, of route_w[perm[i]] * (W_i x_i) (gguf/metal.py:263-291 gemv_combine_<type>).
 * dtype WMOE_BF16: x [n, k], route_w and y are bf16, and each W_i x_i, each scaled product and the running sum are
 * rounded to bf16 as engines/base.py:431-443 combine_decode_experts does; WMOE_F32: all float32, no rounding.
 * weights: device array of n device pointers; perm: device int64 [n] with entries < n_route. */
int wmoe_gemv_combine(wmoe_ctx* ctx, int ggml_type, const uint8_t* const* weights, const int64_t* perm, int n,
                      int n_route, int rows, int k, const void* x, const void* route_w, int dtype, void* y,
                      void* stream);

/* willow's expert_gate (engines/base.py:99-102) on bf16 rows: out [n, ffn] = silu(gate) * up for gate_up [n, 2 * ffn]
 * ([gate | up] per row), each step rounded to bf16 as torch's bf16 F.silu and product round it. */
int wmoe_expert_gate(wmoe_ctx* ctx, const void* gate_up, int n, int ffn, void* out, void* stream);

/* One decode token's routed experts in one call, as engines/base.py:492-532 batched_decode_experts runs them when
 * every down matrix sits in one buffer: gate_up for all n experts (wmoe_gemv_batch: [2 * ffn, hidden] matrices of
 * gate_up_type), willow's expert_gate silu(gate) * up in bf16 (engines/base.py:99-102), then the down matrices
 * ([hidden, ffn] of down_type) and the routing-weighted sum in bf16 (wmoe_gemv_combine, perm[i] the slot of expert
 * i's weight in route_w). gate_up_ptrs, down_ptrs, perm: HOST arrays of n (1..256) device addresses / slots, staged
 * to the GPU by the context without a host synchronisation; x bf16 [hidden] (16-byte aligned), route_w bf16
 * [n_route], y bf16 [hidden]. Two launches on stream: the combine applies expert_gate as it loads the gate_up rows. */
int wmoe_batched_decode_experts(wmoe_ctx* ctx, int gate_up_type, int down_type, int hidden, int ffn,
                                const uint64_t* gate_up_ptrs, const uint64_t* down_ptrs, const int64_t* perm, int n,
                                int n_route, const void* x, const void* route_w, void* y, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* WMOE_H */
