// Grouped dequant-GEMV for few tokens per expert (decode and small batches): the expert products run straight
// from the Q4_K / Q6_K super-blocks with no tensor cores (gguf/metal.py:189-291 gemv/gemv_batch/gemv_combine).
//
// Arithmetic. Activations are quantised per 32 values to int16 (scale = absmax / 32767, relative error ~1e-5),
// so a super-block's inner products are exact integer sums formed with dp2a (two int16 x uint8 products per
// instruction) on the raw 4-bit / 6-bit codes:
//   Q4_K sub-block j (32 values):  sum_i (A_j q_i - B_j) x_i = sx (A_j * sum_i q_i xq_i - B_j * sum_i xq_i)
//   Q6_K 16-value group g:          sum_i D_g (q_i - 32) x_i = sx D_g (sum_i q_i xq_i - 32 sum_i xq_i)
// with A_j = d*sc_j, B_j = dmin*mn_j, D_g = d*sc_g exactly as the reference forms them (exact float32 products
// of an fp16 and a small integer), sx the block's activation scale, and the per-16 sums of xq precomputed once
// per activation row. Sub-block results are accumulated in float32 and reduced with warp shuffles.
//
// Lane layout. Q4_K row of H = 2048 (8 super-blocks x 144 B): lane l takes super-block l/4 and nibble group
// l%4 (32 quant bytes = sub-blocks 2g and 2g+1, 64 values), every load a 16-byte aligned 128-bit load.
// Q6_K row of F = 512 (2 super-blocks x 210 B): 8 lanes per row, lane task t takes super-block t/4, half
// (t/2)%2 and positions 16(t%2)..+15 of all four quarters (48 bytes: two ql runs and one qh run, 64 values);
// Q6_K super-blocks start on 2-byte boundaries, so those loads are aligned 32-bit loads and funnel shifts.
#include "common.cuh"
#include "kernels.cuh"

#include <algorithm>

namespace wmoe {

// ---------------------------------------------------------------- activation quantisation (one thread / 32 values)

template <typename XT>
__global__ void __launch_bounds__(256) quant_rows_kernel(const XT* __restrict__ x, size_t nblocks,
                                                         int16_t* __restrict__ q, float* __restrict__ scale,
                                                         int32_t* __restrict__ sum16) {
  const size_t b = blockIdx.x * size_t(blockDim.x) + threadIdx.x;
  if (b >= nblocks) return;
  float v[32];
  if constexpr (sizeof(XT) == 4) {
    const float4* p = reinterpret_cast<const float4*>(x) + b * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 f = p[i];
      v[4 * i] = f.x, v[4 * i + 1] = f.y, v[4 * i + 2] = f.z, v[4 * i + 3] = f.w;
    }
  } else {
    const uint4* p = reinterpret_cast<const uint4*>(x) + b * 4;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 u = p[i];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[8 * i + 2 * j] = __uint_as_float(w[j] << 16);
        v[8 * i + 2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
      }
    }
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  const float inv = amax > 0.f ? 32767.f / amax : 0.f;
  uint32_t packed[16];
  int s0 = 0, s1 = 0;
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    int a = __float2int_rn(v[i] * inv), c = __float2int_rn(v[i + 1] * inv);
    a = max(-32767, min(32767, a));
    c = max(-32767, min(32767, c));
    if (i < 16) s0 += a + c; else s1 += a + c;
    packed[i / 2] = (uint32_t(a) & 0xFFFFu) | (uint32_t(c) << 16);
  }
  uint4* qo = reinterpret_cast<uint4*>(q) + b * 4;
#pragma unroll
  for (int i = 0; i < 4; ++i) qo[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
  scale[b] = amax / 32767.f;
  sum16[2 * b] = s0;
  sum16[2 * b + 1] = s1;
}

cudaError_t quant_rows(const void* x, int x_dtype, int rows, int K, int16_t* q, float* scale, int32_t* sum16,
                       cudaStream_t st, int* launches) {
  const size_t nblocks = size_t(rows) * (K / XQ_BLOCK);
  if (nblocks == 0) return cudaSuccess;
  const unsigned grid = unsigned((nblocks + 255) / 256);
  if (x_dtype == kF32)
    quant_rows_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(x), nblocks, q, scale, sum16);
  else
    quant_rows_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), nblocks, q, scale,
                                                           sum16);
  ++*launches;
  return cudaGetLastError();
}

// ---------------------------------------------------------------- expert addresses

__device__ __forceinline__ const uint8_t* expert_blob(const ExpertSource& s, int layer, int e, int* status) {
  const int slot = s.slot_of[size_t(layer) * s.experts + e];
  if (slot < 0) {
    set_status(status, kStatusNotResident);
    return nullptr;
  }
  return s.slab + size_t(slot) * s.slot_bytes;
}

__device__ __forceinline__ const uint8_t* gate_up_of(const ExpertSource& s, int layer, int e, int* status) {
  if (e == s.experts) return s.shared_gate_up;
  const uint8_t* b = expert_blob(s, layer, e, status);
  return b;
}

__device__ __forceinline__ const uint8_t* down_of(const ExpertSource& s, int layer, int e, int* status) {
  if (e == s.experts) return s.shared_down;
  const uint8_t* b = expert_blob(s, layer, e, status);
  return b ? b + s.gate_up_bytes : nullptr;
}

// ---------------------------------------------------------------- Q4_K row slice of one lane

struct Q4Lane {
  float A0, B0, A1, B1;  // d*sc and dmin*mn of sub-blocks 2g and 2g+1
  uint4 q0, q1;          // the 32 quant bytes of nibble group g
};

__device__ __forceinline__ Q4Lane q4_lane_load(const uint8_t* block, int g) {
  Q4Lane r;
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

// x: the lane's 64 int16 activations (sub-block 2g in words 0..15, 2g+1 in 16..31), as 8 uint4
__device__ __forceinline__ void q4_lane_dot(const Q4Lane& w, const uint4* x, int& acc0, int& acc1) {
  const uint32_t qw[8] = {w.q0.x, w.q0.y, w.q0.z, w.q0.w, w.q1.x, w.q1.y, w.q1.z, w.q1.w};
  const uint32_t* xw = reinterpret_cast<const uint32_t*>(x);
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const uint32_t lo = qw[m] & 0x0F0F0F0Fu, hi = (qw[m] >> 4) & 0x0F0F0F0Fu;
    acc0 = dp2a_lo(xw[2 * m], lo, acc0);
    acc0 = dp2a_hi(xw[2 * m + 1], lo, acc0);
    acc1 = dp2a_lo(xw[16 + 2 * m], hi, acc1);
    acc1 = dp2a_hi(xw[17 + 2 * m], hi, acc1);
  }
}

// ---------------------------------------------------------------- gate_up + SwiGLU

template <int H>
__global__ void __launch_bounds__(256) gate_up_gemv_kernel(ExpertSource src, int layer, PairMap pm, int F,
                                                           const int16_t* __restrict__ xq,
                                                           const float* __restrict__ xs,
                                                           const int32_t* __restrict__ xsum16,
                                                           float* __restrict__ h, int* status) {
  static_assert(H / 256 * 4 == 32, "one lane per (super-block, nibble group)");
  const int u = blockIdx.y;
  if (u >= *pm.n_used) return;
  const int e = pm.used[u], p0 = pm.seg[u], p1 = pm.seg[u + 1];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int j = blockIdx.x * 8 + warp;
  if (j >= F) return;
  const uint8_t* w = gate_up_of(src, layer, e, status);
  if (w == nullptr) return;
  constexpr int kRowBytes = H / 256 * Q4K_BYTES;
  const int sb = lane / 4, g = lane % 4;
  const Q4Lane gw = q4_lane_load(w + size_t(j) * kRowBytes + sb * Q4K_BYTES, g);
  const Q4Lane uw = q4_lane_load(w + size_t(F + j) * kRowBytes + sb * Q4K_BYTES, g);
  for (int p = p0; p < p1; ++p) {
    const int t = pair_token(pm, p);
    const uint4* xr = reinterpret_cast<const uint4*>(xq + size_t(t) * H + sb * 256 + 64 * g);
    uint4 x[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = xr[i];
    const int xb = t * (H / 32) + sb * 8 + 2 * g;
    const float sx0 = xs[xb], sx1 = xs[xb + 1];
    const int* s16 = xsum16 + size_t(t) * (H / 16) + sb * 16 + 4 * g;
    const float sum0 = float(s16[0] + s16[1]), sum1 = float(s16[2] + s16[3]);
    int ga0 = 0, ga1 = 0, ua0 = 0, ua1 = 0;
    q4_lane_dot(gw, x, ga0, ga1);
    q4_lane_dot(uw, x, ua0, ua1);
    float gs = sx0 * (gw.A0 * float(ga0) - gw.B0 * sum0) + sx1 * (gw.A1 * float(ga1) - gw.B1 * sum1);
    float us = sx0 * (uw.A0 * float(ua0) - uw.B0 * sum0) + sx1 * (uw.A1 * float(ua1) - uw.B1 * sum1);
    gs = warp_sum(gs);
    us = warp_sum(us);
    if (lane == 0) h[size_t(p) * F + j] = silu(gs) * us;
  }
}

cudaError_t gate_up_gemv(const ExpertSource& src, int layer, const PairMap& pm, int H, int F, const int16_t* xq,
                         const float* xs, const int32_t* xsum16, float* h, int* status, cudaStream_t st,
                         int* launches) {
  if (H != 2048) return cudaErrorInvalidValue;
  const dim3 grid(unsigned((F + 7) / 8), unsigned(std::min(pm.E, pm.T * pm.k) + 1));
  gate_up_gemv_kernel<2048><<<grid, 256, 0, st>>>(src, layer, pm, F, xq, xs, xsum16, h, status);
  ++*launches;
  return cudaGetLastError();
}

// ---------------------------------------------------------------- Q6_K row slice of one lane

struct Q6Lane {
  float D[4];        // d*sc of the four 16-value groups (quarters 0..3)
  uint32_t q[4][4];  // unsigned 6-bit codes (0..63) of quarter s, positions 4m..4m+3, one per byte
};

// block: one Q6_K super-block (2-byte aligned); hh: half; pq: 0 or 16
template <bool kShared>
__device__ __forceinline__ Q6Lane q6_lane_load(const uint8_t* block, int hh, int pq) {
  Q6Lane r;
  uint4 ql0, ql1, qh, sc;
  uint32_t dbits;
  if constexpr (kShared) {
    ql0 = lds_u2_16(block + hh * 64 + pq);
    ql1 = lds_u2_16(block + hh * 64 + 32 + pq);
    qh = lds_u2_16(block + 128 + hh * 32 + pq);
    sc = lds_u2_16(block + 192);
    dbits = *reinterpret_cast<const uint16_t*>(block + 208);
  } else {
    ql0 = ldg_u2_16(block + hh * 64 + pq);
    ql1 = ldg_u2_16(block + hh * 64 + 32 + pq);
    qh = ldg_u2_16(block + 128 + hh * 32 + pq);
    sc = ldg_u2_16(block + 192);
    dbits = __ldg(reinterpret_cast<const unsigned short*>(block + 208));
  }
  const float d = f16_to_f32(uint16_t(dbits));
  const uint32_t scw[4] = {sc.x, sc.y, sc.z, sc.w};
  const uint32_t l0[4] = {ql0.x, ql0.y, ql0.z, ql0.w}, l1[4] = {ql1.x, ql1.y, ql1.z, ql1.w};
  const uint32_t hw[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    const int si = hh * 8 + 2 * s + pq / 16;  // scale index of quarter s's positions pq..pq+15
    const int8_t s8 = int8_t((scw[si / 4] >> (8 * (si % 4))) & 0xFF);
    r.D[s] = d * float(s8);
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const uint32_t lw = (s % 2 == 0) ? l0[m] : l1[m];
      const uint32_t nib = (lw >> (4 * (s / 2))) & 0x0F0F0F0Fu;
      const uint32_t hb = (hw[m] >> (2 * s)) & 0x03030303u;
      r.q[s][m] = nib | (hb << 4);
    }
  }
  return r;
}

// x: the lane's activations for quarter s (16 int16 as 2 uint4); returns sum q*x
__device__ __forceinline__ int q6_quarter_dot(const Q6Lane& w, int s, uint4 xa, uint4 xb) {
  const uint32_t xw[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
  int acc = 0;
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    acc = dp2a_lo(xw[2 * m], w.q[s][m], acc);
    acc = dp2a_hi(xw[2 * m + 1], w.q[s][m], acc);
  }
  return acc;
}

// ---------------------------------------------------------------- down

template <int F>
__global__ void __launch_bounds__(256) down_gemv_kernel(ExpertSource src, int layer, PairMap pm, int H,
                                                        const int16_t* __restrict__ hq,
                                                        const float* __restrict__ hs,
                                                        const int32_t* __restrict__ hsum16,
                                                        float* __restrict__ y, int* status) {
  constexpr int S2 = F / 256, LPR = 4 * S2, RPW = 32 / LPR, kRowBytes = S2 * Q6K_BYTES;
  const int u = blockIdx.y;
  if (u >= *pm.n_used) return;
  const int e = pm.used[u], p0 = pm.seg[u], p1 = pm.seg[u + 1];
  const uint8_t* w = down_of(src, layer, e, status);
  if (w == nullptr) return;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int r = (blockIdx.x * 8 + warp) * RPW + lane / LPR;
  const int task = lane % LPR, sb = task / 4, hh = (task / 2) % 2, pq = 16 * (task % 2);
  const bool valid = r < H;
  const Q6Lane wl = q6_lane_load<false>(w + size_t(valid ? r : 0) * kRowBytes + sb * Q6K_BYTES, hh, pq);
  const int base = sb * 256 + hh * 128 + pq;
  for (int p = p0; p < p1; ++p) {
    const int16_t* hr = hq + size_t(p) * F + base;
    float part = 0.f;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const uint4* xp = reinterpret_cast<const uint4*>(hr + 32 * s);
      const int acc = q6_quarter_dot(wl, s, xp[0], xp[1]);
      const int pos = base + 32 * s;
      const int sum = hsum16[size_t(p) * (F / 16) + pos / 16];
      part += hs[size_t(p) * (F / 32) + pos / 32] * (wl.D[s] * float(acc - 32 * sum));
    }
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    if (task == 0 && valid) y[size_t(p) * H + r] = part;
  }
}

// Q4_K down rows (F = 512: 2 super-blocks x 144 B, as some layers of llama.cpp's Q4_K_M files store them): 8 lanes
// per row, lane task t = (super-block t / 4, nibble group t % 4), the Q4_K lane arithmetic of gate_up.
template <int F>
__global__ void __launch_bounds__(256) down_q4k_gemv_kernel(ExpertSource src, int layer, PairMap pm, int H,
                                                            const int16_t* __restrict__ hq,
                                                            const float* __restrict__ hs,
                                                            const int32_t* __restrict__ hsum16,
                                                            float* __restrict__ y, int* status) {
  constexpr int LPR = F / 256 * 4, RPW = 32 / LPR, kRowBytes = F / 256 * Q4K_BYTES;
  const int u = blockIdx.y;
  if (u >= *pm.n_used) return;
  const int e = pm.used[u], p0 = pm.seg[u], p1 = pm.seg[u + 1];
  const uint8_t* w = down_of(src, layer, e, status);
  if (w == nullptr) return;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int r = (blockIdx.x * 8 + warp) * RPW + lane / LPR;
  const int task = lane % LPR, sb = task / 4, g = task % 4;
  const bool valid = r < H;
  const Q4Lane wl = q4_lane_load(w + size_t(valid ? r : 0) * kRowBytes + sb * Q4K_BYTES, g);
  for (int p = p0; p < p1; ++p) {
    const uint4* xr = reinterpret_cast<const uint4*>(hq + size_t(p) * F + sb * 256 + 64 * g);
    uint4 x[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = xr[i];
    const int xb = p * (F / 32) + sb * 8 + 2 * g;
    const float sx0 = hs[xb], sx1 = hs[xb + 1];
    const int* s16 = hsum16 + size_t(p) * (F / 16) + sb * 16 + 4 * g;
    const float sum0 = float(s16[0] + s16[1]), sum1 = float(s16[2] + s16[3]);
    int a0 = 0, a1 = 0;
    q4_lane_dot(wl, x, a0, a1);
    float part = sx0 * (wl.A0 * float(a0) - wl.B0 * sum0) + sx1 * (wl.A1 * float(a1) - wl.B1 * sum1);
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    if (task == 0 && valid) y[size_t(p) * H + r] = part;
  }
}

cudaError_t down_gemv(const ExpertSource& src, int layer, const PairMap& pm, int H, int F, const int16_t* hq,
                      const float* hs, const int32_t* hsum16, float* y, int* status, cudaStream_t st,
                      int* launches) {
  if (F != 512) return cudaErrorInvalidValue;
  constexpr int rows_per_cta = 8 * (32 / 8);
  if (src.down_type == kGgmlQ4K) {
    const dim3 grid(unsigned((H + rows_per_cta - 1) / rows_per_cta), unsigned(std::min(pm.E, pm.T * pm.k) + 1));
    down_q4k_gemv_kernel<512><<<grid, 256, 0, st>>>(src, layer, pm, H, hq, hs, hsum16, y, status);
    ++*launches;
    return cudaGetLastError();
  }
  const dim3 grid(unsigned((H + rows_per_cta - 1) / rows_per_cta), unsigned(std::min(pm.E, pm.T * pm.k) + 1));
  down_gemv_kernel<512><<<grid, 256, 0, st>>>(src, layer, pm, H, hq, hs, hsum16, y, status);
  ++*launches;
  return cudaGetLastError();
}

// ---------------------------------------------------------------- combine

// out[t] = sum over t's k picks in ascending expert id of w * y[pick] (engines/base.py:580-586: index_add_ in
// expert order), then + s_t * shared(x_t) (base.py:481-489). With the residual epilogue (an.h set; the grid is then
// one CTA per token) h[t] += out[t] and, when an.xn is set, xn[t] = rms_norm(h[t]) (engines/qwen36/model.py:17-22).
template <int K>
__global__ void __launch_bounds__(256) combine_kernel(PairMap pm, int H, const float* __restrict__ topk_w,
                                                      const float* __restrict__ shared_s,
                                                      const float* __restrict__ y, void* __restrict__ out,
                                                      int out_dtype, AddNorm an) {
  __shared__ float red[32];
  const int t = blockIdx.y;
  int ps[K];
  float ws[K];
#pragma unroll
  for (int s = 0; s < K; ++s) {
    ps[s] = pm.pos[size_t(t) * K + s];
    ws[s] = topk_w[size_t(t) * K + s];
  }
#pragma unroll
  for (int i = 1; i < K; ++i)
#pragma unroll
    for (int j = i; j > 0; --j)
      if (ps[j] < ps[j - 1]) {
        const int tp = ps[j];
        ps[j] = ps[j - 1];
        ps[j - 1] = tp;
        const float tw = ws[j];
        ws[j] = ws[j - 1];
        ws[j - 1] = tw;
      }
  const float s = shared_s[t];
  const size_t shared_row = size_t(pm.T) * K + t;
  auto value = [&](int r) {
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < K; ++i) acc = __fadd_rn(acc, __fmul_rn(y[size_t(ps[i]) * H + r], ws[i]));
    return __fadd_rn(acc, __fmul_rn(s, y[shared_row * H + r]));
  };
  if (!an.h) {
    for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < H; r += gridDim.x * blockDim.x) {
      const float acc = value(r);
      if (out_dtype == kF32)
        static_cast<float*>(out)[size_t(t) * H + r] = acc;
      else
        static_cast<__nv_bfloat16*>(out)[size_t(t) * H + r] = __float2bfloat16_rn(acc);
    }
    return;
  }
  // the residual epilogue: the CTA holds the whole row, 8 consecutive values per thread (the partition and
  // summation order of add_rmsnorm_kernel)
  float ss = 0.f;
  float* hrow = an.h + size_t(t) * H;
  for (int r = threadIdx.x * 8; r < H; r += blockDim.x * 8) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float v = __fadd_rn(hrow[r + j], value(r + j));
      hrow[r + j] = v;
      ss = fmaf(v, v, ss);
    }
  }
  if (an.xn) {  // uniform over the CTA
    const float rs = rsqrtf(block_sum(ss, red) / float(H) + an.eps);
    for (int r = threadIdx.x * 8; r < H; r += blockDim.x * 8) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = hrow[r + j] * rs;
      store8(an.xn, an.xn_dtype == kF32, size_t(t) * H + r, v);
    }
  }
}

cudaError_t combine(const PairMap& pm, int H, const float* topk_w, const float* shared_s, const float* y, void* out,
                    int out_dtype, const AddNorm& an, cudaStream_t st, int* launches) {
  if (pm.k != 8) return cudaErrorInvalidValue;
  if (an.h && (H % 8 || reinterpret_cast<uintptr_t>(an.xn) % 16)) return cudaErrorInvalidValue;
  // the epilogue's norm needs the whole row in one CTA
  const dim3 grid(an.h ? 1u : unsigned((H + 255) / 256), unsigned(pm.T));
  combine_kernel<8><<<grid, 256, 0, st>>>(pm, H, topk_w, shared_s, y, out, out_dtype, an);
  ++*launches;
  return cudaGetLastError();
}

}  // namespace wmoe
