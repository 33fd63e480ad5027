// Persistent one-token decode of the MoE block: one cooperative launch (one CTA per SM, all co-resident) runs
// every layer of a stack, h <- h + moe_l(rms_norm(h)) (engines/qwen36/model.py:17-22), or a single MoE block.
//
// A layer has two grid-wide exchanges, the minimum its data flow allows (every logit needs all of x; every down
// row needs all of an expert's h):
//   S1  x_l is complete in global memory, and so are the router sums S_l[e] = sum_r R_l[e, r] x_l[r] (plus the
//       shared-expert gate row), accumulated in float64 by the CTAs that produced the rows of x_l, into 4
//       replicas (CTA c adds into replica c % 4; measured against 1, 2, 8 and 16 replicas, 4 balances the atomics'
//       contention against the reads after S1).
//   B   every CTA reads x_l (its own RMS scale r = 1/sqrt(mean(x^2) + eps) from it), sums the replicas in a
//       fixed order and quantises x to int16; warp 0 forms logits r*S + bias and the same top-k routing on every
//       CTA and its lanes at once issue TMA bulk copies (cp.async.bulk, mbarrier completion) of this CTA's 32
//       gate/up row pairs in two chunks; right after the routing barrier warp 1 issues its slice of down rows of
//       all k+1 experts (off warp 0's path), so that the layer's whole expert stream is in flight together.
//       CTA c < 144 owns h block c: 32 consecutive h values of one expert slot. Warps compute gate and up rows
//       (dp2a on the 4-bit codes) -> SwiGLU; warp 0 quantises the block's 32 h values to int16 once and writes
//       them to global memory in the order the down lanes read; the other warps unpack their down codes (Q6_K, or
//       Q4_K on a layer whose down matrices are Q4_K) into registers (independent of h).
//   S2  all h blocks complete.
//   C   every CTA copies the quantised h into shared memory, finishes its rows of the k+1 down products (dp2a on
//       the unpacked codes), combines them in ascending expert id plus the gated shared expert (+ the residual),
//       writes x_{l+1} rows, and adds its rows' share of the next layer's router sums S_{l+1}.
// The router is linear in x, so the RMS normalisation is applied to the sums afterwards (logits = r * S).
// Data written by other CTAs is read through L2 (ld.global.cg). The float64 replicas keep the logits
// independent of the order in which CTAs add their parts (to far below float32 resolution).
// Barrier and mbarrier waits are bounded (1 s of %globaltimer): a timeout sets the device status word and
// every CTA returns instead of hanging (by then every copy it issued has long completed).
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"

namespace wmoe {

namespace {

constexpr int kH = 2048, kF = 512, kE = 256, kK = 8;
constexpr int kSlots = kK + 1;  // routed experts + the shared one
constexpr int kThreads = 512, kWarps = kThreads / 32;
constexpr int kMaxLayers = 64;
constexpr int kMaxRows = 32;                      // output rows per CTA
constexpr int kRowBytesQ4 = kH / 256 * Q4K_BYTES;  // 1152
constexpr int kRowBytesQ6 = kF / 256 * Q6K_BYTES;  // 420: a Q6_K down row
constexpr int kRowBytesQ4d = kF / 256 * Q4K_BYTES;  // 288: a Q4_K down row
constexpr int kHBlocks = kSlots * kF / 32;        // 144 h blocks of 32 values: one per CTA
constexpr int kChunkBytes = 16 * 2 * kRowBytesQ4;  // 16 gate rows + 16 up rows
constexpr int kReplicas = 4;
constexpr int kSaccStride = 264;                  // doubles per replica (>= kE + 1)
constexpr int kSaccRot = kReplicas * kSaccStride;  // doubles per rotation buffer
constexpr int kMaxPairs = 2;                      // (row, slot) down pairs per 8-lane group
constexpr unsigned long long kTimeoutNs = 1000000000ull;
constexpr int kTracePoints = 16;  // WMOE_TRACE_POINTS

struct DecodeParams {
  ExpertSource src;
  int layer_begin, n_layers;
  float eps;
  int stack;
  const void* x_in;
  int x_dtype;
  void* out;
  int out_dtype;
  int32_t* topk_idx_out;
  float* topk_w_out;
  float* xbuf;      // [2][H] residual stream between layers
  double* sacc;     // [3][kReplicas][kSaccStride] router sums, rotating by layer
  int16_t* hq;      // [kSlots][F] quantised h, down lane order
  float* hs;        // [kSlots][F / 32] its scales
  int32_t* hsum;    // [kSlots][F / 16] its per-16 sums
  unsigned* bar;    // grid barrier counter (own 128-byte line)
  int* status;
  int dn_chunk;     // bytes reserved per slot for this CTA's down rows
  unsigned long long* trace;  // phase timestamps [layer][point][cta], or null
  unsigned char down_q4[kMaxLayers];  // 1: the layer's down matrices are Q4_K (else Q6_K)
  float min_w;      // willow's min_expert_weight (0: off)
  DecodeLayer layers[kMaxLayers];
};

// ---------------------------------------------------------------- synchronisation primitives

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Monotonic-counter grid barrier: the epoch-th barrier of this launch completes when the counter reaches
// epoch * gridDim.x. Split into arrive (one thread, after the CTA's writes that others will read; the fence
// makes them visible first) and wait (every thread), so that independent work can run in between.
__device__ __forceinline__ void grid_arrive(unsigned* counter) {
  asm volatile("fence.acq_rel.gpu;" ::: "memory");
  asm volatile("red.relaxed.gpu.global.add.u32 [%0], 1;" ::"l"(counter) : "memory");
}

// Returns false on every thread of the CTA if the wait ran out.
__device__ bool grid_wait(unsigned* counter, unsigned epoch, int* status, volatile int* abort_flag) {
  if (threadIdx.x == 0) {
    const unsigned target = epoch * gridDim.x;
    const unsigned long long t0 = globaltimer();
    while (int(ld_acquire(counter) - target) < 0) {
      if (globaltimer() - t0 > kTimeoutNs) {
        set_status(status, kStatusBarrierTimeout);
        *abort_flag = 1;
        break;
      }
    }
  }
  __syncthreads();
  return *abort_flag == 0;
}

__device__ bool grid_barrier(unsigned* counter, unsigned epoch, int* status, volatile int* abort_flag) {
  __syncthreads();
  if (threadIdx.x == 0) grid_arrive(counter);
  return grid_wait(counter, epoch, status, abort_flag);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity; false if it ran out (status and abort flag set).
__device__ bool mbar_wait(uint64_t* bar, unsigned parity, int* status, volatile int* abort_flag) {
  if (!mbar_try_wait(bar, parity)) {
    const unsigned long long t0 = globaltimer();
    while (!mbar_try_wait(bar, parity)) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > kTimeoutNs) {
        set_status(status, kStatusBarrierTimeout);
        *abort_flag = 1;
        return false;
      }
    }
  }
  return true;
}

// global -> shared bulk copy (16-byte aligned addresses, size a multiple of 16), completing on an mbarrier. The
// destination's earlier readers have all passed a CTA barrier before the copy is issued (their loads are
// complete), so the copy's async-proxy writes cannot overtake them.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// An L2 prefetch of one line: used to have an address translation cached before a bulk copy needs it.
__device__ __forceinline__ void touch(const void* ptr) { asm volatile("prefetch.global.L2 [%0];" ::"l"(ptr)); }

// ---------------------------------------------------------------- shared memory layout

struct Small {
  uint64_t mbar_gu[2], mbar_dn, mbar_rs;
  DecodeLayer layers[kMaxLayers];  // the layer table, copied once (parameter reads by layer index miss the cache)
  unsigned char down_q4[kMaxLayers];
  alignas(16) float x[kH];        // x_l as read (raw residual for a stack)
  alignas(16) int16_t xq[kH];     // quantised x, in gate_up lane order (see xq_offset)
  float xs[kH / 32];
  int32_t xsum[kH / 16];
  alignas(16) int16_t hq[kSlots][kF];  // quantised h, in down lane order (see hq_offset)
  float hs[kSlots][kF / 32];
  int32_t hsum[kSlots][kF / 16];
  float ys[kMaxRows][kSlots];
  float xn[kMaxRows];             // this CTA's rows of x_{l+1}
  alignas(16) float rs[kMaxRows][kRouterStride];  // packed router rows r0..r1-1 of the next layer
  float logit[kE + 1];            // summed router sums S (before the RMS factor)
  int slot_row[2][kE];            // the store slot of each expert, by layer parity
  float bias[2][kE];              // the routing bias (zero without one), by layer parity
  float hblk[32];                 // this CTA's 32 h values
  float red[kWarps];
  int sel[kSlots];
  float w[kSlots];
  int order[kK];
  const uint8_t* dn_ptr[kSlots];
  float rscale;
  int abort_flag;
};

// Scale and min of sub-blocks j = 2g and 2g + 1 of a Q4_K super-block (6-bit values packed in the 12 bytes s0..s2,
// ggml's get_scale_min_k4 layout), without a branch on g: byte k = j % 4 of each word, and for j >= 4 the high two
// bits of the first eight bytes complete the 4-bit halves of the last four.
__device__ __forceinline__ void q4k_scales_pair(uint32_t s0, uint32_t s1, uint32_t s2, int g, int& sc0, int& mn0,
                                                int& sc1, int& mn1) {
  const int k = (2 * g) & 3;
  const bool hi = g >= 2;
  const uint32_t a = __byte_perm(s0, 0, 0x4440 + k) | (__byte_perm(s0, 0, 0x4440 + k + 1) << 16);  // b[k], b[k+1]
  const uint32_t b = __byte_perm(s1, 0, 0x4440 + k) | (__byte_perm(s1, 0, 0x4440 + k + 1) << 16);
  const uint32_t c = __byte_perm(s2, 0, 0x4440 + k) | (__byte_perm(s2, 0, 0x4440 + k + 1) << 16);
  // two 16-bit lanes at once: (sub-block 2g, sub-block 2g + 1)
  const uint32_t sc = hi ? ((c & 0x000F000Fu) | ((a >> 2) & 0x00300030u)) : (a & 0x003F003Fu);
  const uint32_t mn = hi ? (((c >> 4) & 0x000F000Fu) | ((b >> 2) & 0x00300030u)) : (b & 0x003F003Fu);
  sc0 = int(sc & 0xFFFF), sc1 = int(sc >> 16), mn0 = int(mn & 0xFFFF), mn1 = int(mn >> 16);
}

// One lane's share of a gate row and an up row: 64 weights of each (super-block sb, nibble group g = sub-blocks 2g
// and 2g + 1) against the int16 x codes in xw, with four independent accumulators per row.
__device__ __forceinline__ float2 q4_dot_pair(const uint8_t* gate, const uint8_t* up, int g, const uint32_t* xw,
                                              float sx0, float sx1, float sum0, float sum1) {
  const uint4 hg = *reinterpret_cast<const uint4*>(gate), hu = *reinterpret_cast<const uint4*>(up);
  const uint4 g0 = *reinterpret_cast<const uint4*>(gate + 16 + 32 * g);
  const uint4 g1 = *reinterpret_cast<const uint4*>(gate + 32 + 32 * g);
  const uint4 u0 = *reinterpret_cast<const uint4*>(up + 16 + 32 * g);
  const uint4 u1 = *reinterpret_cast<const uint4*>(up + 32 + 32 * g);
  const uint32_t gw[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
  const uint32_t uw[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
  int ga0 = 0, ga1 = 0, gb0 = 0, gb1 = 0, ua0 = 0, ua1 = 0, ub0 = 0, ub1 = 0;  // a: runs m even, b: m odd
#pragma unroll
  for (int m = 0; m < 8; m += 2) {
#pragma unroll
    for (int o = 0; o < 2; ++o) {
      const int mm = m + o;
      const uint32_t glo = gw[mm] & 0x0F0F0F0Fu, ghi = (gw[mm] >> 4) & 0x0F0F0F0Fu;
      const uint32_t ulo = uw[mm] & 0x0F0F0F0Fu, uhi = (uw[mm] >> 4) & 0x0F0F0F0Fu;
      int& g_lo = o ? gb0 : ga0;
      int& g_hi = o ? gb1 : ga1;
      int& u_lo = o ? ub0 : ua0;
      int& u_hi = o ? ub1 : ua1;
      g_lo = dp2a_hi(xw[2 * mm + 1], glo, dp2a_lo(xw[2 * mm], glo, g_lo));
      u_lo = dp2a_hi(xw[2 * mm + 1], ulo, dp2a_lo(xw[2 * mm], ulo, u_lo));
      g_hi = dp2a_hi(xw[17 + 2 * mm], ghi, dp2a_lo(xw[16 + 2 * mm], ghi, g_hi));
      u_hi = dp2a_hi(xw[17 + 2 * mm], uhi, dp2a_lo(xw[16 + 2 * mm], uhi, u_hi));
    }
  }
  int gsc0, gmn0, gsc1, gmn1, usc0, umn0, usc1, umn1;
  q4k_scales_pair(hg.y, hg.z, hg.w, g, gsc0, gmn0, gsc1, gmn1);
  q4k_scales_pair(hu.y, hu.z, hu.w, g, usc0, umn0, usc1, umn1);
  const float gd = f16_to_f32(uint16_t(hg.x & 0xFFFF)), gdm = f16_to_f32(uint16_t(hg.x >> 16));
  const float ud = f16_to_f32(uint16_t(hu.x & 0xFFFF)), udm = f16_to_f32(uint16_t(hu.x >> 16));
  const int gs0 = ga0 + gb0, gs1 = ga1 + gb1, us0 = ua0 + ub0, us1 = ua1 + ub1;
  return make_float2(sx0 * ((gd * float(gsc0)) * float(gs0) - (gdm * float(gmn0)) * sum0) +
                         sx1 * ((gd * float(gsc1)) * float(gs1) - (gdm * float(gmn1)) * sum1),
                     sx0 * ((ud * float(usc0)) * float(us0) - (udm * float(umn0)) * sum0) +
                         sx1 * ((ud * float(usc1)) * float(us1) - (udm * float(umn1)) * sum1));
}

// Where x position pos lives in sm.xq: the gate_up lane (super-block pos/256, nibble group (pos%256)/64) reads its
// 64 values as 8 runs of 8, run m of every lane adjacent (conflict-free 16-byte loads).
__device__ __forceinline__ int xq_offset(int pos) {
  const int lanex = (pos / 256) * 4 + (pos % 256) / 64, k = pos % 64;
  return ((k / 8) * 32 + lanex) * 8 + k % 8;
}

// Where h position pos lives within a slot's quantised h: the down lane task t8 = (super-block, half, 16-run)
// reads quarter s of its positions as two runs of 8, the eight tasks' runs adjacent.
__device__ __forceinline__ int hq_offset(int pos) {
  const int sb = pos / 256, hh = (pos % 256) / 128, r = pos % 128, s = r / 32, p = r % 32;
  const int t8 = sb * 4 + hh * 2 + p / 16, e16 = p % 16;
  return ((s * 2 + e16 / 8) * 8 + t8) * 8 + e16 % 8;
}
// Start of run (quarter s, half-run j) of down lane task t8 within a slot's quantised h.
__device__ __forceinline__ int hq_run(int s, int j, int t8) { return ((s * 2 + j) * 8 + t8) * 8; }

// Warp-cooperative int16 quantisation of 32 values (lane i holds value i of the block): q[offset], the block's
// scale and its two per-16 sums, with single-instruction warp reductions (redux.sync).
__device__ __forceinline__ void quant32_warp(float v, int lane, int16_t* q, int offset, float* scale,
                                             int32_t* sum16) {
  const float amax = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v))));
  const float inv = amax > 0.f ? 32767.f / amax : 0.f;
  int a = __float2int_rn(v * inv);
  a = max(-32767, min(32767, a));
  q[offset] = int16_t(a);
  const int all = __reduce_add_sync(0xffffffffu, a);
  const int lo = __reduce_add_sync(0xffffffffu, lane < 16 ? a : 0);
  if (lane == 0) {
    *scale = amax / 32767.f;
    sum16[0] = lo;
    sum16[1] = all - lo;
  }
}

// This CTA's rows [r0, r1) of x (in sm.xn) times the packed router slice in sm.rs, added into its float64 replica.
__device__ void add_router_part(Small& sm, double* replica, int nrows) {
  const int e = threadIdx.x;
  if (e <= kE) {
    float acc = 0.f;
    for (int i = 0; i < nrows; ++i) acc = fmaf(sm.rs[i][e], sm.xn[i], acc);
    atomicAdd(replica + e, double(acc));
  }
}

// Router rows r0..r1-1 (transposed: [row][expert], shared gate at column kE) of layer L into sm.rs: one bulk copy
// of the packed router (thread 0 issues; mbar_rs completes), or plain loads from the [E, H] router when no packed
// copy exists (every thread; then the caller's __syncthreads completes it). Returns true if a copy was issued.
__device__ bool fetch_router_slice(Small& sm, const DecodeLayer& L, int r0, int nrows) {
  if (L.router_packed) {
    if (threadIdx.x == 0) {
      const unsigned bytes = unsigned(nrows) * kRouterStride * 4;
      mbar_arrive_expect_tx(&sm.mbar_rs, bytes);
      bulk_g2s(&sm.rs[0][0], L.router_packed + size_t(r0) * kRouterStride, bytes, &sm.mbar_rs);
    }
    return true;
  }
  for (int idx = threadIdx.x; idx < (kE + 1) * nrows; idx += kThreads) {
    const int e = idx / nrows, i = idx % nrows;
    const float* row = e < kE ? L.router_w + size_t(e) * kH : L.shared_gate;
    sm.rs[i][e] = __ldg(row + r0 + i);
  }
  return false;
}

// Layer li's slot-table row and routing bias into shared memory (buffer li % 2, read by that layer's top-k).
__device__ void fetch_layer_meta(Small& sm, const DecodeParams& p, int li) {
  const int t = threadIdx.x, layer = p.layer_begin + li;
  if (t < kE)
    sm.slot_row[li % 2][t] = p.src.slot_of[size_t(layer) * kE + t];
  else if (t < 2 * kE)
    sm.bias[li % 2][t - kE] = sm.layers[li].router_bias ? sm.layers[li].router_bias[t - kE] : 0.f;
}

// int16 quantisation of 2048 values by 512 threads, 4 each (thread t holds positions 4t..4t+3 in v): a 32-value
// block is 8 adjacent threads (amax and per-16 sums by xor shuffles within the group). q written in xq_offset
// order (4 adjacent positions stay adjacent).
__device__ __forceinline__ void quant_x(float4 v, int16_t* q, float* scale, int32_t* sum16) {
  const int t = threadIdx.x;
  float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
  const float inv = amax > 0.f ? 32767.f * __frcp_rn(amax) : 0.f;
  const int a = max(-32767, min(32767, __float2int_rn(v.x * inv)));
  const int b = max(-32767, min(32767, __float2int_rn(v.y * inv)));
  const int cc = max(-32767, min(32767, __float2int_rn(v.z * inv)));
  const int d = max(-32767, min(32767, __float2int_rn(v.w * inv)));
  *reinterpret_cast<uint2*>(q + xq_offset(4 * t)) =
      make_uint2((uint32_t(a) & 0xFFFFu) | (uint32_t(b) << 16), (uint32_t(cc) & 0xFFFFu) | (uint32_t(d) << 16));
  int s = a + b + cc + d;
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  s += __shfl_xor_sync(0xffffffffu, s, 2);  // sum of 16 values (4 threads)
  if ((t & 7) == 0) scale[t / 8] = amax / 32767.f;
  if ((t & 3) == 0) sum16[t / 4] = s;
}

// Order-preserving map of a float onto unsigned (larger float -> larger integer); 0 is below every float.
__device__ __forceinline__ uint32_t ordered(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float unordered(uint32_t u) {
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u);
}

// Down codes of one (row, slot) pair for one lane, unpacked while the h exchange (S2) completes.
// Q6_K: lane task t8 = (super-block t8/4, half (t8/2)%2, 16-run t8%2); q[s][m] holds quarter s, positions 4m..4m+3
// of the run as 6-bit codes, D[s] = d * scale of the quarter's 16 values.
// Q4_K: lane task t8 = (super-block t8/4, nibble group g = t8%4); q[0..1][*] hold the 8 words of quant bytes
// 32g..32g+31 (low nibbles: sub-block 2g, high: 2g + 1), D = {d*sc0, dmin*mn0, d*sc1, dmin*mn1}.
struct DownPair {
  uint32_t q[4][4];
  float D[4];
};

__device__ __forceinline__ void down_unpack_q6(const uint8_t* blk, int hh, int pq, DownPair& dp) {
  const uint4 ql0 = lds_u2_16(blk + hh * 64 + pq), ql1 = lds_u2_16(blk + hh * 64 + 32 + pq);
  const uint4 qh = lds_u2_16(blk + 128 + hh * 32 + pq), sc = lds_u2_16(blk + 192);
  const float d = f16_to_f32(*reinterpret_cast<const uint16_t*>(blk + 208));
  const uint32_t scw[4] = {sc.x, sc.y, sc.z, sc.w};
  const uint32_t l0[4] = {ql0.x, ql0.y, ql0.z, ql0.w}, l1[4] = {ql1.x, ql1.y, ql1.z, ql1.w};
  const uint32_t hw[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    const int si = hh * 8 + 2 * s + pq / 16;
    dp.D[s] = d * float(int8_t((scw[si / 4] >> (8 * (si % 4))) & 0xFF));
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const uint32_t lw = (s % 2 == 0) ? l0[m] : l1[m];
      dp.q[s][m] = ((lw >> (4 * (s / 2))) & 0x0F0F0F0Fu) | (((hw[m] >> (2 * s)) & 0x03030303u) << 4);
    }
  }
}

__device__ __forceinline__ void down_unpack_q4(const uint8_t* blk, int g, DownPair& dp) {
  const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
  const uint4 q0 = *reinterpret_cast<const uint4*>(blk + 16 + 32 * g);
  const uint4 q1 = *reinterpret_cast<const uint4*>(blk + 32 + 32 * g);
  int sc0, mn0, sc1, mn1;
  q4k_scales_pair(hdr.y, hdr.z, hdr.w, g, sc0, mn0, sc1, mn1);
  const float d = f16_to_f32(uint16_t(hdr.x & 0xFFFF)), dm = f16_to_f32(uint16_t(hdr.x >> 16));
  dp.q[0][0] = q0.x, dp.q[0][1] = q0.y, dp.q[0][2] = q0.z, dp.q[0][3] = q0.w;
  dp.q[1][0] = q1.x, dp.q[1][1] = q1.y, dp.q[1][2] = q1.z, dp.q[1][3] = q1.w;
  dp.D[0] = d * float(sc0), dp.D[1] = dm * float(mn0), dp.D[2] = d * float(sc1), dp.D[3] = dm * float(mn1);
}

// One pair's down product for one lane, from the unpacked codes and the slot's quantised h in shared memory.
__device__ __forceinline__ float down_dot_q6(const DownPair& dp, const Small& sm, int slot, int t8, int base) {
  float t[4];
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    // runs of 8 of this lane task: (s, 0) and (s, 1), each group's eight tasks adjacent
    const uint4 xa = *reinterpret_cast<const uint4*>(&sm.hq[slot][hq_run(s, 0, t8)]);
    const uint4 xb = *reinterpret_cast<const uint4*>(&sm.hq[slot][hq_run(s, 1, t8)]);
    const uint32_t xw[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
    int acc0 = 0, acc1 = 0;
#pragma unroll
    for (int m = 0; m < 4; m += 2) {
      acc0 = dp2a_hi(xw[2 * m + 1], dp.q[s][m], dp2a_lo(xw[2 * m], dp.q[s][m], acc0));
      acc1 = dp2a_hi(xw[2 * m + 3], dp.q[s][m + 1], dp2a_lo(xw[2 * m + 2], dp.q[s][m + 1], acc1));
    }
    const int pos = base + 32 * s;
    t[s] = sm.hs[slot][pos / 32] * (dp.D[s] * float(acc0 + acc1 - 32 * sm.hsum[slot][pos / 16]));
  }
  return (t[0] + t[1]) + (t[2] + t[3]);
}

// Q4_K: sub-block 2g is positions sb*256 + 64g + [0, 32) and lies in quarter s = 2 (g % 2) of half g / 2, tasks
// t8b and t8b + 1 of the Q6_K lane layout (16 positions each); sub-block 2g + 1 is quarter s + 1 of the same tasks.
__device__ __forceinline__ float down_dot_q4(const DownPair& dp, const Small& sm, int slot, int sb, int g) {
  const int t8b = sb * 4 + (g >> 1) * 2, s = 2 * (g & 1);
  int acc[2] = {0, 0};
#pragma unroll
  for (int half = 0; half < 2; ++half) {  // 0: low nibbles (sub-block 2g), 1: high nibbles (2g + 1)
#pragma unroll
    for (int j = 0; j < 4; ++j) {  // run j: positions 8j..8j+7 of the sub-block = quant words 2j, 2j + 1
      const int t8 = t8b + (j >> 1), jr = j & 1;
      const uint4 xa = *reinterpret_cast<const uint4*>(&sm.hq[slot][hq_run(s + half, jr, t8)]);
      const uint32_t w0 = dp.q[j >> 1][2 * (j & 1)], w1 = dp.q[j >> 1][2 * (j & 1) + 1];
      const uint32_t n0 = (w0 >> (4 * half)) & 0x0F0F0F0Fu, n1 = (w1 >> (4 * half)) & 0x0F0F0F0Fu;
      acc[half] = dp2a_hi(xa.y, n0, dp2a_lo(xa.x, n0, acc[half]));
      acc[half] = dp2a_hi(xa.w, n1, dp2a_lo(xa.z, n1, acc[half]));
    }
  }
  const int b0 = sb * 8 + 2 * g;  // 32-value block of sub-block 2g in h
  const float h0 = float(sm.hsum[slot][2 * b0] + sm.hsum[slot][2 * b0 + 1]);
  const float h1 = float(sm.hsum[slot][2 * b0 + 2] + sm.hsum[slot][2 * b0 + 3]);
  return sm.hs[slot][b0] * (dp.D[0] * float(acc[0]) - dp.D[1] * h0) +
         sm.hs[slot][b0 + 1] * (dp.D[2] * float(acc[1]) - dp.D[3] * h1);
}

__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const __grid_constant__ DecodeParams p) {
  extern __shared__ __align__(128) uint8_t dyn[];
  Small& sm = *reinterpret_cast<Small*>(dyn);
  uint8_t* gu_buf = dyn + (sizeof(Small) + 127) / 128 * 128;  // [chunk][gate rows 16][up rows 16]
  uint8_t* dn_buf = gu_buf + 2 * kChunkBytes;
  const int dn_chunk = p.dn_chunk;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int nc = gridDim.x, c = blockIdx.x;
  const int r0 = int((long long)c * kH / nc), r1 = int((long long)(c + 1) * kH / nc), nrows = r1 - r0;
  const bool has_block = c < kHBlocks;  // h block c: slot c / 16, h indices 32 (c % 16) .. + 31
  const int blk_slot = c / 16, blk_j0 = 32 * (c % 16);
  const int replica = c % kReplicas;
  unsigned epoch = 0;
  unsigned rs_phase = 0;  // parity of the next mbar_rs phase
#define WMOE_TRACE(li, pt)                                                                        \
  do {                                                                                            \
    if (p.trace && tid == 0) p.trace[(size_t(li) * kTracePoints + (pt)) * nc + c] = globaltimer(); \
  } while (0)
  if (tid == 0) {
    sm.abort_flag = 0;
    mbar_init(&sm.mbar_gu[0], 1);
    mbar_init(&sm.mbar_gu[1], 1);
    mbar_init(&sm.mbar_dn, 1);
    mbar_init(&sm.mbar_rs, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  {
    constexpr int kWords = int(sizeof(DecodeLayer) / sizeof(uint64_t));
    static_assert(sizeof(DecodeLayer) % sizeof(uint64_t) == 0, "DecodeLayer holds pointers only");
    for (int i = tid; i < p.n_layers * kWords; i += kThreads)
      reinterpret_cast<uint64_t*>(sm.layers)[i] = reinterpret_cast<const uint64_t*>(p.layers)[i];
    if (tid < kMaxLayers) sm.down_q4[tid] = p.down_q4[tid];
  }
  __syncthreads();

  // ---------------- prologue: the first layer's router sums from the input rows of this CTA
  {
    const DecodeLayer& L = sm.layers[0];
    for (int i = tid; i < nrows; i += kThreads) {
      float v;
      if (p.x_dtype == kF32)
        v = __ldcg(static_cast<const float*>(p.x_in) + r0 + i);
      else
        v = __bfloat162float(static_cast<const __nv_bfloat16*>(p.x_in)[r0 + i]);
      sm.xn[i] = v;
    }
    fetch_layer_meta(sm, p, 0);
    if (fetch_router_slice(sm, L, r0, nrows)) {
      if (!mbar_wait(&sm.mbar_rs, rs_phase, p.status, &sm.abort_flag)) return;
      rs_phase ^= 1u;
    }
    __syncthreads();
    add_router_part(sm, p.sacc + replica * kSaccStride, nrows);
  }
  if (!grid_barrier(p.bar, ++epoch, p.status, &sm.abort_flag)) return;

  for (int li = 0; li < p.n_layers; ++li) {
    const int layer = p.layer_begin + li;
    const DecodeLayer& L = sm.layers[li];
    const unsigned parity = unsigned(li & 1);
    const double* S = p.sacc + (li % 3) * kSaccRot;
    const bool last = li + 1 == p.n_layers;
    const bool dq4 = sm.down_q4[li] != 0;
    const int rb = dq4 ? kRowBytesQ4d : kRowBytesQ6;  // down row bytes of this layer

    // ---------------- phase B: x_l, RMS scale, router sums, routing, copies, gate_up
    WMOE_TRACE(li, 0);
    {
      float4 v;
      if (li == 0 && p.x_dtype != kF32) {
        const uint2 b = reinterpret_cast<const uint2*>(p.x_in)[tid];
        v = make_float4(__uint_as_float(b.x << 16), __uint_as_float(b.x & 0xFFFF0000u), __uint_as_float(b.y << 16),
                        __uint_as_float(b.y & 0xFFFF0000u));
      } else {
        const float* xi = li == 0 ? static_cast<const float*>(p.x_in) : p.xbuf + (li % 2) * kH;
        v = __ldcg(reinterpret_cast<const float4*>(xi) + tid);
      }
      // the router-sum replicas are read while x is in flight (one L2 round trip for both) and summed first
      if (tid <= kE) {
        double acc = 0.0;
#pragma unroll
        for (int r = 0; r < kReplicas; ++r) acc += __ldcg(S + r * kSaccStride + tid);
        sm.logit[tid] = float(acc);
      }
      reinterpret_cast<float4*>(sm.x)[tid] = v;
      float ss = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      ss = warp_sum(ss);
      if (lane == 0) sm.red[warp] = ss;
      quant_x(v, sm.xq, sm.xs, sm.xsum);  // the RMS factor is applied to the scales later
      if (c == 0)  // this rotation buffer is next added into two layers on
        for (int i = tid; i < kSaccRot; i += kThreads) p.sacc[((li + 2) % 3) * kSaccRot + i] = 0.0;
    }
    __syncthreads();
    WMOE_TRACE(li, 1);
    // the next layer's slot row and bias, loaded now into a register and stored in phase C
    int next_meta = 0;
    if (!last) {
      const int layer1 = layer + 1;
      if (tid < kE)
        next_meta = p.src.slot_of[size_t(layer1) * kE + tid];
      else if (tid < 2 * kE && sm.layers[li + 1].router_bias)
        next_meta = __float_as_int(sm.layers[li + 1].router_bias[tid - kE]);
    }
    if (warp == 0) {
      const float t = warp_sum(lane < kWarps ? sm.red[lane] : 0.f);
      const float rsc = p.stack ? 1.0f / sqrtf(t / float(kH) + p.eps) : 1.0f;
      // top-k by k rounds of two single-instruction warp reductions: the largest logit, then the smallest expert
      // id holding it (ties go to the lower id)
      uint32_t key[kE / 32];
#pragma unroll
      for (int i = 0; i < kE / 32; ++i) {
        const int e = lane + 32 * i;
        key[i] = ordered(sm.logit[e] * rsc + sm.bias[li % 2][e]);
      }
      uint32_t my_key = 0;
      int my_e = kE;  // lane kK keeps the shared expert's id
      for (int r = 0; r < kK; ++r) {
        // local maximum as a tree; ties keep the lower expert id (smaller i)
        uint32_t m01 = key[0] >= key[1] ? key[0] : key[1], m23 = key[2] >= key[3] ? key[2] : key[3];
        uint32_t m45 = key[4] >= key[5] ? key[4] : key[5], m67 = key[6] >= key[7] ? key[6] : key[7];
        int i01 = key[0] >= key[1] ? 0 : 1, i23 = key[2] >= key[3] ? 2 : 3;
        int i45 = key[4] >= key[5] ? 4 : 5, i67 = key[6] >= key[7] ? 6 : 7;
        const uint32_t ma = m01 >= m23 ? m01 : m23, mb = m45 >= m67 ? m45 : m67;
        const int ia = m01 >= m23 ? i01 : i23, ib = m45 >= m67 ? i45 : i67;
        const uint32_t lm = ma >= mb ? ma : mb;
        const int le = lane + 32 * (ma >= mb ? ia : ib);
        const uint32_t m = __reduce_max_sync(0xffffffffu, lm);
        const int be = int(__reduce_min_sync(0xffffffffu, lm == m ? uint32_t(le) : 0xffffffffu));
#pragma unroll
        for (int i = 0; i < kE / 32; ++i)
          if (lane + 32 * i == be) key[i] = 0u;
        if (lane == r) {
          my_key = m;
          my_e = be;
        }
      }
      WMOE_TRACE(li, 2);
      // expert addresses of the k+1 slots (lane s holds slot s)
      const uint8_t *gu = nullptr, *dn = nullptr;
      if (lane < kSlots) {
        if (my_e == kE) {
          gu = L.shared_gate_up;
          dn = L.shared_down;
        } else {
          const int s = sm.slot_row[li % 2][my_e];
          if (s >= 0) {
            gu = p.src.slab + size_t(s) * p.src.slot_bytes;
            dn = gu + p.src.gate_up_bytes;
          } else {
            set_status(p.status, kStatusNotResident);
          }
        }
        sm.sel[lane] = my_e;
      }
      // this CTA's 32 gate/up row pairs: lanes 0-3 issue the four copies at once (chunk = 16 pairs)
      const unsigned long long gu_blk =
          __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(gu), has_block ? blk_slot : 0);
      if (lane < 2) mbar_arrive_expect_tx(&sm.mbar_gu[lane], has_block && gu_blk ? kChunkBytes : 0u);
      __syncwarp();
      if (has_block && gu_blk && lane < 4) {
        const int ch = lane / 2, up = lane % 2;
        const uint8_t* src = reinterpret_cast<const uint8_t*>(gu_blk) +
                             size_t(up * kF + blk_j0 + 16 * ch) * kRowBytesQ4;
        bulk_g2s(gu_buf + ch * kChunkBytes + up * (kChunkBytes / 2), src, kChunkBytes / 2, &sm.mbar_gu[ch]);
      }
      if (lane < kSlots) sm.dn_ptr[lane] = dn;  // the down rows are issued by warp 1 after the routing barrier
      WMOE_TRACE(li, 3);
      // renormalised weights of the k picks: exp(l_i - l_0) / sum_j exp(l_j - l_0)
      const float top0 = unordered(__shfl_sync(0xffffffffu, my_key, 0));
      const float my_ex = lane < kK ? expf(unordered(my_key) - top0) : 0.f;
      float sum = my_ex;
#pragma unroll
      for (int o = 4; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);  // lanes 0..7
      // willow's skip_small_experts (engines/base.py:413-429): keep the top pick (lane 0) and the picks >= min_w,
      // scaled back up to the former total; a dropped pick keeps its expert with weight 0
      float my_w = lane < kK ? my_ex / sum : 0.f;
      if (p.min_w > 0.f) {
        const bool keep = lane == 0 || my_w >= p.min_w;
        float total = my_w, kept = keep ? my_w : 0.f;
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) {
          total += __shfl_xor_sync(0xffffffffu, total, o);
          kept += __shfl_xor_sync(0xffffffffu, kept, o);
        }
        my_w = keep ? my_w * (total / kept) : 0.f;
      }
      if (lane < kK) {
        sm.w[lane] = my_w;
        if (c == 0 && p.topk_idx_out) p.topk_idx_out[li * kK + lane] = my_w == 0.f ? -1 : my_e;
        if (c == 0 && p.topk_w_out) p.topk_w_out[li * kK + lane] = my_w;
        int rank = 0;
        for (int o = 0; o < kK; ++o) rank += __shfl_sync(0x000000ffu, my_e, o) < my_e ? 1 : 0;
        sm.order[rank] = lane;
      }
      if (lane == 0) {
        sm.rscale = rsc;
        sm.w[kK] = 1.0f / (1.0f + expf(-sm.logit[kE] * rsc));
      }
    }
    __syncthreads();
    WMOE_TRACE(li, 4);
    if (warp == 1) {  // down rows [r0, r1) of every slot (aligned outward to 16 bytes), off warp 0's critical path
      const uint8_t* dn = lane < kSlots ? sm.dn_ptr[lane] : nullptr;
      const unsigned lo = unsigned(r0) * unsigned(rb) / 16 * 16;
      const unsigned hi = (unsigned(r1) * unsigned(rb) + 15) / 16 * 16;
      const unsigned present = __popc(__ballot_sync(0xffffffffu, dn != nullptr));
      if (lane == 0) mbar_arrive_expect_tx(&sm.mbar_dn, present * (hi - lo));
      __syncwarp();
      if (dn) bulk_g2s(dn_buf + size_t(lane) * dn_chunk, dn + lo, hi - lo, &sm.mbar_dn);
    }
    // the next layer's router slice, overlapping the copies (waited for before it is used in phase C)
    const bool rs_copy = p.stack && !last && fetch_router_slice(sm, sm.layers[li + 1], r0, nrows);
    if (!mbar_wait(&sm.mbar_gu[0], parity, p.status, &sm.abort_flag)) return;
    WMOE_TRACE(li, 5);
    if (has_block) {
      const int sb = lane / 4, g = lane % 4;
      uint32_t xw[32];
      const uint4* xp = reinterpret_cast<const uint4*>(sm.xq) + lane;  // run m of this lane at (m * 32 + lane)
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint4 v = xp[i * 32];
        xw[4 * i] = v.x, xw[4 * i + 1] = v.y, xw[4 * i + 2] = v.z, xw[4 * i + 3] = v.w;
      }
      const float rsc = sm.rscale;
      const float sx0 = sm.xs[sb * 8 + 2 * g] * rsc, sx1 = sm.xs[sb * 8 + 2 * g + 1] * rsc;
      const float sum0 = float(sm.xsum[sb * 16 + 4 * g] + sm.xsum[sb * 16 + 4 * g + 1]);
      const float sum1 = float(sm.xsum[sb * 16 + 4 * g + 2] + sm.xsum[sb * 16 + 4 * g + 3]);
#pragma unroll
      for (int ch = 0; ch < 2; ++ch) {
        if (ch == 1) {
          WMOE_TRACE(li, 6);
          if (!mbar_wait(&sm.mbar_gu[1], parity, p.status, &sm.abort_flag)) return;
          WMOE_TRACE(li, 7);
        }
        const uint8_t* gate = gu_buf + ch * kChunkBytes + warp * kRowBytesQ4 + sb * Q4K_BYTES;
        const uint8_t* up = gate + kChunkBytes / 2;
        const float2 gu = q4_dot_pair(gate, up, g, xw, sx0, sx1, sum0, sum1);
        float gs = gu.x, us = gu.y;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          gs += __shfl_xor_sync(0xffffffffu, gs, o);
          us += __shfl_xor_sync(0xffffffffu, us, o);
        }
        if (lane == 0) sm.hblk[16 * ch + warp] = silu(gs) * us;
      }
    }
    if (!has_block) {
      WMOE_TRACE(li, 6);
      WMOE_TRACE(li, 7);
    }
    __syncthreads();
    WMOE_TRACE(li, 8);
    // the block's h, quantised once, in the order the down lanes read it; then this CTA arrives at S2
    if (warp == 0) {
      if (has_block) {
        const int pos = blk_j0 + lane, blk = blk_j0 / 32;
        quant32_warp(sm.hblk[lane], lane, p.hq + blk_slot * kF, hq_offset(pos), p.hs + blk_slot * (kF / 32) + blk,
                     p.hsum + blk_slot * (kF / 16) + 2 * blk);
      }
      __syncwarp();
      if (lane == 0) grid_arrive(p.bar);
    }
    ++epoch;
    // down codes of this thread's (row, slot) pairs, unpacked while S2 completes
    const int grp = tid / 8, t8 = tid % 8;
    DownPair dp[kMaxPairs];
    WMOE_TRACE(li, 9);
    if (!mbar_wait(&sm.mbar_dn, parity, p.status, &sm.abort_flag)) return;
    WMOE_TRACE(li, 10);
    {
      const int dn_off = (r0 * rb) % 16;  // row r0 within each slot's down chunk
#pragma unroll
      for (int k = 0; k < kMaxPairs; ++k) {
        const int pr = grp + k * (kThreads / 8);
        if (pr < nrows * kSlots) {
          const int rl = pr / kSlots, slot = pr % kSlots;
          const uint8_t* row = dn_buf + size_t(slot) * dn_chunk + dn_off + rl * rb;
          if (dq4)
            down_unpack_q4(row + (t8 / 4) * Q4K_BYTES, t8 % 4, dp[k]);
          else
            down_unpack_q6(row + (t8 / 4) * Q6K_BYTES, (t8 / 2) % 2, 16 * (t8 % 2), dp[k]);
        } else {
          dp[k] = DownPair{};  // past the CTA's rows: computed on, never stored
        }
      }
    }
    // while S2 completes: the address translations of the next layer's experts. A layer's copies come from 9 of
    // 20 GB of expert pages, and a translation miss delays a bulk copy at issue and again at completion; each CTA
    // touches both pages that each expert blob of its share (expert e on CTA e % nc) can span, and the shared
    // expert's.
    if (!last) {
      if (tid < kE && tid % nc == c && next_meta >= 0) {
        const uint8_t* b = p.src.slab + size_t(next_meta) * p.src.slot_bytes;
        touch(b);
        touch(b + p.src.slot_bytes - 1);
      }
      if (tid == kE && c == nc - 1) {
        const DecodeLayer& N = sm.layers[li + 1];
        touch(N.shared_gate_up);
        touch(N.shared_gate_up + 2 * kF * kRowBytesQ4 - 1);
        touch(N.shared_down);
        touch(N.shared_down + kH * (sm.down_q4[li + 1] ? kRowBytesQ4d : kRowBytesQ6) - 1);
      }
    }
    WMOE_TRACE(li, 11);
    if (!grid_wait(p.bar, epoch, p.status, &sm.abort_flag)) return;
    WMOE_TRACE(li, 12);

    // ---------------- phase C: h, down rows of this CTA, combine, next layer's router sums
    if (!last) {  // the next layer's slot row and bias (read by its top-k after S1)
      if (tid < kE)
        sm.slot_row[(li + 1) % 2][tid] = next_meta;
      else if (tid < 2 * kE)
        sm.bias[(li + 1) % 2][tid - kE] = __int_as_float(next_meta);
    }
    {
      // every load issued before any store: one L2 round trip
      constexpr int kVec = kSlots * kF / 8, kScales = kSlots * kF / 32, kSums = kSlots * kF / 16;
      static_assert(kVec > kThreads && kVec <= 2 * kThreads && kScales <= kThreads && kSums <= kThreads, "h sizes");
      const uint4* src = reinterpret_cast<const uint4*>(p.hq);
      uint4* dst = reinterpret_cast<uint4*>(&sm.hq[0][0]);
      const bool two = tid + kThreads < kVec;
      const uint4 v0 = __ldcg(src + tid);
      const uint4 v1 = two ? __ldcg(src + tid + kThreads) : make_uint4(0u, 0u, 0u, 0u);
      const float hs = tid < kScales ? __ldcg(p.hs + tid) : 0.f;
      const int hsum = tid < kSums ? __ldcg(p.hsum + tid) : 0;
      dst[tid] = v0;
      if (two) dst[tid + kThreads] = v1;
      if (tid < kScales) (&sm.hs[0][0])[tid] = hs;
      if (tid < kSums) (&sm.hsum[0][0])[tid] = hsum;
    }
    __syncthreads();
    WMOE_TRACE(li, 13);
    {
      // both pairs of the thread at once (a pair past the CTA's rows computes on unused codes and is not stored);
      // the four quarters of a pair summed as a tree
      const unsigned gmask = 0xFFu << (8 * (lane / 8));
      float part[kMaxPairs];
#pragma unroll
      for (int k = 0; k < kMaxPairs; ++k) {
        const int slot = (grp + k * (kThreads / 8)) % kSlots;
        if (dq4)
          part[k] = down_dot_q4(dp[k], sm, slot, t8 / 4, t8 % 4);
        else
          part[k] = down_dot_q6(dp[k], sm, slot, t8, (t8 / 4) * 256 + ((t8 / 2) % 2) * 128 + 16 * (t8 % 2));
      }
#pragma unroll
      for (int o = 4; o > 0; o >>= 1)
#pragma unroll
        for (int k = 0; k < kMaxPairs; ++k) part[k] += __shfl_xor_sync(gmask, part[k], o);
#pragma unroll
      for (int k = 0; k < kMaxPairs; ++k) {
        const int pr = grp + k * (kThreads / 8);
        if (t8 == 0 && pr < nrows * kSlots) sm.ys[pr / kSlots][pr % kSlots] = part[k];
      }
    }
    __syncthreads();
    WMOE_TRACE(li, 14);
    if (tid < nrows) {
      const int r = r0 + tid;
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < kK; ++i) {
        const int slot = sm.order[i];
        acc = __fadd_rn(acc, __fmul_rn(sm.ys[tid][slot], sm.w[slot]));
      }
      acc = __fadd_rn(acc, __fmul_rn(sm.w[kK], sm.ys[tid][kK]));
      if (p.stack) acc = __fadd_rn(sm.x[r], acc);
      sm.xn[tid] = acc;
      if (!last) {
        p.xbuf[((li + 1) % 2) * kH + r] = acc;
      } else if (p.out_dtype == kF32) {
        static_cast<float*>(p.out)[r] = acc;
      } else {
        static_cast<__nv_bfloat16*>(p.out)[r] = __float2bfloat16_rn(acc);
      }
    }
    if (!last) {
      if (rs_copy && !mbar_wait(&sm.mbar_rs, rs_phase, p.status, &sm.abort_flag)) return;
      if (rs_copy) rs_phase ^= 1u;
      __syncthreads();
      add_router_part(sm, p.sacc + ((li + 1) % 3) * kSaccRot + replica * kSaccStride, nrows);
      WMOE_TRACE(li, 15);
      if (!grid_barrier(p.bar, ++epoch, p.status, &sm.abort_flag)) return;
    }
  }
#undef WMOE_TRACE
}

// one slot's down rows of a CTA, aligned outward to 16 bytes, plus the 4 bytes a funnel-shift load may read past
int down_chunk_bytes(int nc) { return ((kH + nc - 1) / nc * kRowBytesQ6 + 32 + 15) / 16 * 16; }

size_t smem_bytes(int nc) {
  return (sizeof(Small) + 127) / 128 * 128 + 2 * size_t(kChunkBytes) + size_t(kSlots) * down_chunk_bytes(nc) + 64;
}

}  // namespace

// Scratch of the no-allocation entry point (wmoe_decode_stack_noalloc): file-scope device memory of a fixed size,
// one copy on every GPU that loads the library, held until the process exits. Host code cannot use the symbol as
// a device address (it is a host-side stand-in); static_scratch() looks the address up per device.
constexpr size_t kStaticScratchBytes = 160u * 1024u;  // WMOE_NOALLOC_SCRATCH_BYTES
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

size_t static_scratch_bytes() { return kStaticScratchBytes; }

// Device address of g_static_scratch on the current device, looked up once per (device, primary context) pair:
// after a cudaDeviceReset the context is a new one and the address is looked up again. The first call on a device
// must come before any stream capture. Returns the CUDA error of the lookup.
cudaError_t static_scratch(int device, void** ptr) {
  constexpr int kMaxDevices = 64;
  static std::mutex mu;
  static void* addr[kMaxDevices] = {};
  static void* owner[kMaxDevices] = {};  // the context the address belongs to
  using GetCtx = int (*)(void**);        // cuCtxGetCurrent, reached through the runtime (no link to libcuda)
  static GetCtx get_ctx = nullptr;
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (!get_ctx) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_ctx = reinterpret_cast<GetCtx>(fn);
  }
  void* cur = nullptr;
  if (get_ctx) {
    cudaFree(nullptr);  // makes the device's primary context current if it is not yet
    if (get_ctx(&cur) != 0) cur = nullptr;
  }
  if (!addr[device] || owner[device] != cur) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return e;
    addr[device] = p;
    owner[device] = cur;
  }
  *ptr = addr[device];
  return cudaSuccess;
}

size_t decode_scratch_bytes(int H, int F, int E, int) {
  // barrier line, x ping-pong, router sums, then quantised h with its scales and per-16 sums
  return 256 + size_t(2 * H) * sizeof(float) + 3 * size_t(kSaccRot) * sizeof(double) +
         size_t(kSlots * F) * sizeof(int16_t) + size_t(kSlots * F / 32) * sizeof(float) +
         size_t(kSlots * F / 16) * sizeof(int32_t) + 256;
}

int decode_num_ctas(int device) {
  int coop = 0, sms = 0, per_sm = 0;
  if (cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device) != cudaSuccess || !coop) return 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
  // one h block per CTA; every CTA at most kMaxRows output rows and kMaxPairs (row, slot) pairs per 8-lane group
  if (sms < kHBlocks || (kH + sms - 1) / sms > kMaxRows || (kH + sms - 1) / sms * kSlots > kMaxPairs * (kThreads / 8))
    return 0;
  const size_t smem = smem_bytes(sms);
  if (cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
    return 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_kernel, kThreads, smem) != cudaSuccess) return 0;
  return per_sm >= 1 ? sms : 0;
}

cudaError_t decode_persistent(const ExpertSource& src, const int* down_types, int layer_begin, int n_layers,
                              const DecodeLayer* layers, int H, int F, int E, int k, float eps, bool stack,
                              const void* x_in, int x_dtype, void* out, int out_dtype, int32_t* topk_idx_out,
                              float* topk_w_out, void* scratch, int num_ctas, int* status, uint64_t* trace,
                              size_t trace_entries, cudaStream_t st, int* launches, float min_w) {
  if (H != kH || F != kF || E != kE || k != kK || num_ctas < kHBlocks) return cudaErrorInvalidValue;
  for (int i = 0; i < n_layers; ++i) {
    if (down_types[i] != kGgmlQ6K && down_types[i] != kGgmlQ4K) return cudaErrorInvalidValue;
    // a packed router is bulk-copied: 16-byte aligned
    if (reinterpret_cast<uintptr_t>(layers[i].router_packed) & 15u) return cudaErrorMisalignedAddress;
  }
  // the trace covers the first launch's layers when it is large enough, else it is off
  if (trace && trace_entries < size_t(std::min(n_layers, kMaxLayers)) * kTracePoints * size_t(num_ctas))
    trace = nullptr;
  char* base = static_cast<char*>(scratch);
  unsigned* bar = reinterpret_cast<unsigned*>(base);
  float* xbuf = reinterpret_cast<float*>(base + 256);
  double* sacc = reinterpret_cast<double*>(xbuf + 2 * kH);
  int16_t* hq = reinterpret_cast<int16_t*>(sacc + 3 * kSaccRot);
  float* hs = reinterpret_cast<float*>(hq + kSlots * kF);
  int32_t* hsum = reinterpret_cast<int32_t*>(hs + kSlots * kF / 32);
  const size_t smem = smem_bytes(num_ctas);
  cudaError_t e = cudaSuccess;
  for (int l0 = 0; l0 < n_layers; l0 += kMaxLayers) {
    DecodeParams p{};
    p.src = src;
    p.layer_begin = layer_begin + l0;
    p.n_layers = std::min(kMaxLayers, n_layers - l0);
    p.eps = eps;
    p.stack = stack ? 1 : 0;
    p.x_in = l0 == 0 ? x_in : out;
    p.x_dtype = l0 == 0 ? x_dtype : out_dtype;
    p.out = out;
    p.out_dtype = out_dtype;
    p.topk_idx_out = topk_idx_out ? topk_idx_out + l0 * kK : nullptr;
    p.topk_w_out = topk_w_out ? topk_w_out + l0 * kK : nullptr;
    p.xbuf = xbuf;
    p.sacc = sacc;
    p.hq = hq;
    p.hs = hs;
    p.hsum = hsum;
    p.bar = bar;
    p.status = status;
    p.dn_chunk = down_chunk_bytes(num_ctas);
    p.min_w = min_w;
    p.trace = l0 == 0 ? reinterpret_cast<unsigned long long*>(trace) : nullptr;
    for (int i = 0; i < p.n_layers; ++i) {
      p.layers[i] = layers[l0 + i];
      p.down_q4[i] = down_types[l0 + i] == kGgmlQ4K ? 1 : 0;
    }
    // barrier counter and the router sums start at zero for every launch
    e = cudaMemsetAsync(base, 0, 256, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(sacc, 0, 3 * size_t(kSaccRot) * sizeof(double), st);
    if (e != cudaSuccess) return e;
    void* args[] = {&p};
    e = cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(decode_kernel), dim3(num_ctas), dim3(kThreads),
                                    args, smem, st);
    if (e != cudaSuccess) return e;
    ++*launches;
  }
  return cudaSuccess;
}

}  // namespace wmoe
