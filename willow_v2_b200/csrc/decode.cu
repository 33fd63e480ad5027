// Persistent one-token decode of the MoE block: one cooperative launch (one CTA per SM, all co-resident) runs
// every layer of a stack, h <- h + moe_l(rms_norm(h)) (engines/qwen36/model.py:17-22), or a single MoE block.
//
// Per layer, three phases separated by grid barriers:
//   A  x (the residual stream, or the caller's normalised input) -> shared memory, RMS-normalised for a stack,
//      quantised to int16 per 32 values; the E router rows and the shared-expert gate row are split over the
//      CTAs (fp32 dot products, 16 warps per row) -> logits in global memory.
//   B  every CTA reads the E+1 logits and forms the same top-k routing (softmax over the picks, renormalised);
//      the (k routed + 1 shared) x F SwiGLU outputs are split over CTAs and warps: each warp computes a gate row
//      and its up row from the Q4_K blocks (dp2a on the 4-bit codes, layout of gemv.cu) -> h in global memory.
//   C  every CTA quantises all k+1 h vectors into shared memory and owns a slice of the H output rows: for each
//      of its rows, the k+1 Q6_K down dot products (8 lanes each), then the combine in ascending expert id plus
//      the shared expert times its sigmoid gate, plus the residual for a stack.
// Data written by other CTAs is read with ld.global.cg (L2), never from a possibly stale L1 line.
// The barrier spins are bounded (1 s of %globaltimer); a timeout sets the device status word and every CTA
// returns early instead of hanging.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace wmoe {

namespace {

constexpr int kH = 2048, kF = 512, kE = 256, kK = 8;
constexpr int kSlots = kK + 1;  // routed experts + the shared one
constexpr int kThreads = 512, kWarps = kThreads / 32;
constexpr int kMaxLayers = 64;
constexpr unsigned long long kBarrierTimeoutNs = 1000000000ull;

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
  float* xbuf;     // [2][H] residual stream between layers
  float* logits;   // [E+1]
  float* hbuf;     // [kSlots][F]
  unsigned* bar;   // [64]: count at 0, generation at 32 (separate 128-byte lines)
  int* status;
  DecodeLayer layers[kMaxLayers];
};

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release(unsigned* p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Returns false (for every thread of the CTA) when the wait ran out.
__device__ bool grid_barrier(unsigned* bar, int* status, int* abort_flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned* count = bar;
    unsigned* gen = bar + 32;
    const unsigned g = ld_acquire(gen);
    __threadfence();
    const unsigned arrived = atomicAdd(count, 1u);
    if (arrived == gridDim.x - 1) {
      atomicExch(count, 0u);
      st_release(gen, g + 1);
    } else {
      const unsigned long long t0 = globaltimer();
      while (ld_acquire(gen) == g) {
        if (globaltimer() - t0 > kBarrierTimeoutNs) {
          set_status(status, kStatusBarrierTimeout);
          *abort_flag = 1;
          break;
        }
      }
    }
    __threadfence();
  }
  __syncthreads();
  return *abort_flag == 0;
}

struct Smem {
  float x[kH];                 // input row (normalised for a stack)
  float resid[kH];             // residual (stack)
  int16_t xq[kH];              // quantised x
  float xs[kH / 32];           // per-32 scales
  int32_t xsum[kH / 16];       // per-16 sums of xq
  int16_t hq[kSlots][kF];      // quantised h of each slot
  float hs[kSlots][kF / 32];
  int32_t hsum[kSlots][kF / 16];
  float ys[32][kSlots];        // down outputs of this CTA's rows (at most 32: needs >= 64 CTAs)
  float red[kWarps];
  float red2[kWarps][2];
  int sel[kSlots];             // expert id of each slot (slot kK: shared = kE)
  float w[kSlots];             // routing weight of each slot (slot kK: sigmoid gate)
  int order[kK];               // routed slots in ascending expert id
  float norm;
  int abort_flag;
};

// Quantise 32 floats (shared memory) to int16 with their scale and per-16 sums.
__device__ __forceinline__ void quant32(const float* v, int16_t* q, float* scale, int32_t* sum16) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  const float inv = amax > 0.f ? 32767.f / amax : 0.f;
  int s0 = 0, s1 = 0;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    int a = __float2int_rn(v[i] * inv);
    a = max(-32767, min(32767, a));
    q[i] = int16_t(a);
    if (i < 16) s0 += a; else s1 += a;
  }
  *scale = amax / 32767.f;
  sum16[0] = s0;
  sum16[1] = s1;
}

struct Q4L {
  float A0, B0, A1, B1;
  uint4 q0, q1;
};

__device__ __forceinline__ Q4L q4_load(const uint8_t* block, int g) {
  Q4L r;
  const uint4 hd = ldg_nc_v4(block);
  r.q0 = ldg_nc_v4(block + 16 + 32 * g);
  r.q1 = ldg_nc_v4(block + 32 + 32 * g);
  const float d = f16_to_f32(uint16_t(hd.x & 0xFFFF)), dmin = f16_to_f32(uint16_t(hd.x >> 16));
  int sc0, mn0, sc1, mn1;
  q4k_scale_min_w(hd.y, hd.z, hd.w, 2 * g, sc0, mn0);
  q4k_scale_min_w(hd.y, hd.z, hd.w, 2 * g + 1, sc1, mn1);
  r.A0 = d * float(sc0);
  r.B0 = dmin * float(mn0);
  r.A1 = d * float(sc1);
  r.B1 = dmin * float(mn1);
  return r;
}

__device__ __forceinline__ float q4_dot(const Q4L& w, const uint32_t* xw, float sx0, float sx1, float sum0,
                                        float sum1) {
  const uint32_t qw[8] = {w.q0.x, w.q0.y, w.q0.z, w.q0.w, w.q1.x, w.q1.y, w.q1.z, w.q1.w};
  int a0 = 0, a1 = 0;
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const uint32_t lo = qw[m] & 0x0F0F0F0Fu, hi = (qw[m] >> 4) & 0x0F0F0F0Fu;
    a0 = dp2a_lo(xw[2 * m], lo, a0);
    a0 = dp2a_hi(xw[2 * m + 1], lo, a0);
    a1 = dp2a_lo(xw[16 + 2 * m], hi, a1);
    a1 = dp2a_hi(xw[17 + 2 * m], hi, a1);
  }
  return sx0 * (w.A0 * float(a0) - w.B0 * sum0) + sx1 * (w.A1 * float(a1) - w.B1 * sum1);
}

__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const __grid_constant__ DecodeParams p) {
  __shared__ Smem sm;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int nc = gridDim.x, c = blockIdx.x;
  if (tid == 0) sm.abort_flag = 0;
  __syncthreads();

  for (int li = 0; li < p.n_layers; ++li) {
    const int layer = p.layer_begin + li;
    const DecodeLayer& L = p.layers[li];

    // ---------------- phase A: input row, normalisation, quantisation, router logits
    if (li == 0) {
      if (p.x_dtype == kF32) {
        const float* xi = static_cast<const float*>(p.x_in);
        for (int i = tid; i < kH; i += kThreads) sm.resid[i] = __ldcg(xi + i);
      } else {
        const __nv_bfloat16* xi = static_cast<const __nv_bfloat16*>(p.x_in);
        for (int i = tid; i < kH; i += kThreads) sm.resid[i] = __bfloat162float(xi[i]);
      }
    } else {
      const float* xi = p.xbuf + (li % 2) * kH;
      for (int i = tid; i < kH; i += kThreads) sm.resid[i] = __ldcg(xi + i);
    }
    __syncthreads();
    if (p.stack) {
      float ss = 0.f;
      for (int i = tid; i < kH; i += kThreads) ss = fmaf(sm.resid[i], sm.resid[i], ss);
      ss = warp_sum(ss);
      if (lane == 0) sm.red[warp] = ss;
      __syncthreads();
      if (tid == 0) {
        float t = 0.f;
        for (int i = 0; i < kWarps; ++i) t += sm.red[i];
        sm.norm = 1.0f / sqrtf(t / float(kH) + p.eps);
      }
      __syncthreads();
      for (int i = tid; i < kH; i += kThreads) sm.x[i] = sm.resid[i] * sm.norm;
    } else {
      for (int i = tid; i < kH; i += kThreads) sm.x[i] = sm.resid[i];
    }
    __syncthreads();
    if (tid < kH / 32) quant32(sm.x + 32 * tid, sm.xq + 32 * tid, sm.xs + tid, sm.xsum + 2 * tid);
    // router rows r = c, c + nc, ... of [R; g]: 16 warps split K, one float4 per lane
    for (int r = c; r <= kE; r += nc) {
      const float* row = r < kE ? L.router_w + size_t(r) * kH : L.shared_gate;
      const int k0 = warp * (kH / kWarps) + lane * 4;
      const float4 wv = __ldg(reinterpret_cast<const float4*>(row + k0));
      float acc = wv.x * sm.x[k0];
      acc = fmaf(wv.y, sm.x[k0 + 1], acc);
      acc = fmaf(wv.z, sm.x[k0 + 2], acc);
      acc = fmaf(wv.w, sm.x[k0 + 3], acc);
      acc = warp_sum(acc);
      __syncthreads();  // sm.red is reused across rows
      if (lane == 0) sm.red[warp] = acc;
      __syncthreads();
      if (tid == 0) {
        float t = 0.f;
        for (int i = 0; i < kWarps; ++i) t += sm.red[i];
        p.logits[r] = t;
      }
    }
    if (!grid_barrier(p.bar, p.status, &sm.abort_flag)) return;

    // ---------------- phase B: routing (every CTA), gate_up + SwiGLU
    if (warp == 0) {
      float v[kE / 32];
#pragma unroll
      for (int i = 0; i < kE / 32; ++i) {
        const int e = lane + 32 * i;
        float l = __ldcg(p.logits + e);
        if (L.router_bias) l += L.router_bias[e];
        v[i] = l;
      }
      float top0 = 0.f, sum = 0.f, my_ex = 0.f;
      int my_e = 0;
      for (int r = 0; r < kK; ++r) {
        float best = -INFINITY;
        int be = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < kE / 32; ++i) {
          const int e = lane + 32 * i;
          if (v[i] > best || (v[i] == best && e < be)) {
            best = v[i];
            be = e;
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ob = __shfl_xor_sync(0xffffffffu, best, o);
          const int oe = __shfl_xor_sync(0xffffffffu, be, o);
          if (ob > best || (ob == best && oe < be)) {
            best = ob;
            be = oe;
          }
        }
#pragma unroll
        for (int i = 0; i < kE / 32; ++i)
          if (lane + 32 * i == be) v[i] = -INFINITY;
        if (r == 0) top0 = best;
        const float ex = expf(best - top0);
        sum += ex;
        if (lane == r) {
          my_ex = ex;
          my_e = be;
        }
      }
      if (lane < kK) {
        sm.sel[lane] = my_e;
        sm.w[lane] = my_ex / sum;
        if (c == 0 && p.topk_idx_out) p.topk_idx_out[li * kK + lane] = my_e;
        if (c == 0 && p.topk_w_out) p.topk_w_out[li * kK + lane] = my_ex / sum;
        // rank of this slot in ascending expert id
        int rank = 0;
        for (int o = 0; o < kK; ++o) {
          const int oe = __shfl_sync(0x000000ffu, my_e, o);
          rank += oe < my_e ? 1 : 0;
        }
        sm.order[rank] = lane;
      }
      if (lane == 0) {
        sm.sel[kK] = kE;
        sm.w[kK] = 1.0f / (1.0f + expf(-__ldcg(p.logits + kE)));
      }
    }
    __syncthreads();
    {
      // the lane's 64 activations (super-block lane/4, nibble group lane%4) stay in registers
      const int sb = lane / 4, g = lane % 4;
      uint32_t xw[32];
      const uint4* xp = reinterpret_cast<const uint4*>(sm.xq + sb * 256 + 64 * g);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint4 v = xp[i];
        xw[4 * i] = v.x, xw[4 * i + 1] = v.y, xw[4 * i + 2] = v.z, xw[4 * i + 3] = v.w;
      }
      const float sx0 = sm.xs[sb * 8 + 2 * g], sx1 = sm.xs[sb * 8 + 2 * g + 1];
      const float sum0 = float(sm.xsum[sb * 16 + 4 * g] + sm.xsum[sb * 16 + 4 * g + 1]);
      const float sum1 = float(sm.xsum[sb * 16 + 4 * g + 2] + sm.xsum[sb * 16 + 4 * g + 3]);
      constexpr int kUnits = kSlots * kF, kRowBytes = kH / 256 * Q4K_BYTES;
      const int u0 = int((long long)c * kUnits / nc), u1 = int((long long)(c + 1) * kUnits / nc);
      for (int u = u0 + warp; u < u1; u += kWarps) {
        const int slot = u / kF, j = u % kF;
        const int e = sm.sel[slot];
        const uint8_t* w;
        if (e == kE) {
          w = L.shared_gate_up;
        } else {
          const int s = p.src.slot_of[size_t(layer) * kE + e];
          if (s < 0) {
            set_status(p.status, kStatusNotResident);
            continue;
          }
          w = p.src.slab + size_t(s) * p.src.slot_bytes;
        }
        const Q4L gw = q4_load(w + size_t(j) * kRowBytes + sb * Q4K_BYTES, g);
        const Q4L uw = q4_load(w + size_t(kF + j) * kRowBytes + sb * Q4K_BYTES, g);
        float gs = q4_dot(gw, xw, sx0, sx1, sum0, sum1);
        float us = q4_dot(uw, xw, sx0, sx1, sum0, sum1);
        gs = warp_sum(gs);
        us = warp_sum(us);
        if (lane == 0) p.hbuf[slot * kF + j] = silu(gs) * us;
      }
    }
    if (!grid_barrier(p.bar, p.status, &sm.abort_flag)) return;

    // ---------------- phase C: down for this CTA's rows, combine, residual
    for (int b = tid; b < kSlots * kF / 32; b += kThreads) {
      const int slot = b / (kF / 32), blk = b % (kF / 32);
      float v[32];
      const float4* hp = reinterpret_cast<const float4*>(p.hbuf + slot * kF + 32 * blk);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 f = __ldcg(hp + i);
        v[4 * i] = f.x, v[4 * i + 1] = f.y, v[4 * i + 2] = f.z, v[4 * i + 3] = f.w;
      }
      quant32(v, &sm.hq[slot][32 * blk], &sm.hs[slot][blk], &sm.hsum[slot][2 * blk]);
    }
    __syncthreads();
    const int r0 = int((long long)c * kH / nc), r1 = int((long long)(c + 1) * kH / nc);
    const int nrows = r1 - r0;
    {
      const int grp = tid / 8, t8 = tid % 8;
      const unsigned gmask = 0xFFu << (8 * (lane / 8));
      const int sb = t8 / 4, hh = (t8 / 2) % 2, pq = 16 * (t8 % 2);
      const int base = sb * 256 + hh * 128 + pq;
      for (int pr = grp; pr < nrows * kSlots; pr += kThreads / 8) {
        const int rl = pr / kSlots, slot = pr % kSlots;
        const int e = sm.sel[slot];
        const uint8_t* w;
        bool ok = true;
        if (e == kE) {
          w = L.shared_down;
        } else {
          const int s = p.src.slot_of[size_t(layer) * kE + e];
          ok = s >= 0;
          w = p.src.slab + size_t(ok ? s : 0) * p.src.slot_bytes + p.src.gate_up_bytes;
        }
        float part = 0.f;
        if (ok) {
          const uint8_t* blk = w + size_t(r0 + rl) * (kF / 256 * Q6K_BYTES) + sb * Q6K_BYTES;
          const uint4 ql0 = ldg_u2_16(blk + hh * 64 + pq), ql1 = ldg_u2_16(blk + hh * 64 + 32 + pq);
          const uint4 qh = ldg_u2_16(blk + 128 + hh * 32 + pq), sc = ldg_u2_16(blk + 192);
          const float d = f16_to_f32(__ldg(reinterpret_cast<const unsigned short*>(blk + 208)));
          const uint32_t scw[4] = {sc.x, sc.y, sc.z, sc.w};
          const uint32_t l0[4] = {ql0.x, ql0.y, ql0.z, ql0.w}, l1[4] = {ql1.x, ql1.y, ql1.z, ql1.w};
          const uint32_t hw[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
          for (int s = 0; s < 4; ++s) {
            const int si = hh * 8 + 2 * s + pq / 16;
            const float D = d * float(int8_t((scw[si / 4] >> (8 * (si % 4))) & 0xFF));
            const uint4* xp = reinterpret_cast<const uint4*>(&sm.hq[slot][base + 32 * s]);
            const uint4 xa = xp[0], xb = xp[1];
            const uint32_t xw[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
            int acc = 0;
#pragma unroll
            for (int m = 0; m < 4; ++m) {
              const uint32_t lw = (s % 2 == 0) ? l0[m] : l1[m];
              const uint32_t q = ((lw >> (4 * (s / 2))) & 0x0F0F0F0Fu) | (((hw[m] >> (2 * s)) & 0x03030303u) << 4);
              acc = dp2a_lo(xw[2 * m], q, acc);
              acc = dp2a_hi(xw[2 * m + 1], q, acc);
            }
            const int pos = base + 32 * s;
            part += sm.hs[slot][pos / 32] * (D * float(acc - 32 * sm.hsum[slot][pos / 16]));
          }
        } else {
          set_status(p.status, kStatusNotResident);
        }
        part += __shfl_xor_sync(gmask, part, 4);
        part += __shfl_xor_sync(gmask, part, 2);
        part += __shfl_xor_sync(gmask, part, 1);
        if (t8 == 0) sm.ys[rl][slot] = part;
      }
    }
    __syncthreads();
    if (tid < nrows) {
      const int r = r0 + tid;
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < kK; ++i) {
        const int slot = sm.order[i];
        acc = __fadd_rn(acc, __fmul_rn(sm.ys[tid][slot], sm.w[slot]));
      }
      acc = __fadd_rn(acc, __fmul_rn(sm.w[kK], sm.ys[tid][kK]));
      if (p.stack) acc = __fadd_rn(sm.resid[r], acc);
      if (li + 1 < p.n_layers) {
        p.xbuf[((li + 1) % 2) * kH + r] = acc;
      } else if (p.out_dtype == kF32) {
        static_cast<float*>(p.out)[r] = acc;
      } else {
        static_cast<__nv_bfloat16*>(p.out)[r] = __float2bfloat16_rn(acc);
      }
    }
    if (li + 1 < p.n_layers)
      if (!grid_barrier(p.bar, p.status, &sm.abort_flag)) return;
  }
}

}  // namespace

size_t decode_scratch_bytes(int H, int F, int E, int) {
  return size_t(2 * H + (E + 1) + kSlots * F) * sizeof(float) + 64 * sizeof(unsigned) + 1024;
}

int decode_num_ctas(int device) {
  int coop = 0, sms = 0, per_sm = 0;
  if (cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device) != cudaSuccess || !coop) return 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_kernel, kThreads, 0) != cudaSuccess) return 0;
  return per_sm >= 1 && sms >= 64 ? sms : 0;
}

cudaError_t decode_persistent(const ExpertSource& src, int layer_begin, int n_layers, const DecodeLayer* layers,
                              int H, int F, int E, int k, float eps, bool stack, const void* x_in, int x_dtype,
                              void* out,
                              int out_dtype, int32_t* topk_idx_out, float* topk_w_out, void* scratch,
                              int num_ctas, int* status, cudaStream_t st, int* launches) {
  if (H != kH || F != kF || E != kE || k != kK || num_ctas <= 0) return cudaErrorInvalidValue;
  char* base = static_cast<char*>(scratch);
  unsigned* bar = reinterpret_cast<unsigned*>(base);
  float* xbuf = reinterpret_cast<float*>(base + 256);
  float* logits = xbuf + 2 * kH;
  float* hbuf = logits + (kE + 1 + 63) / 64 * 64;
  cudaError_t e = cudaMemsetAsync(bar, 0, 64 * sizeof(unsigned), st);
  if (e != cudaSuccess) return e;
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
    p.logits = logits;
    p.hbuf = hbuf;
    p.bar = bar;
    p.status = status;
    for (int i = 0; i < p.n_layers; ++i) p.layers[i] = layers[l0 + i];
    void* args[] = {&p};
    e = cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(decode_kernel), dim3(num_ctas), dim3(kThreads),
                                    args, 0, st);
    if (e != cudaSuccess) return e;
    ++*launches;
  }
  return cudaSuccess;
}

}  // namespace wmoe
