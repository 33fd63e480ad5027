// Router: logits = x . [R; g]^T in float32 (R [E, H] router, g [H] shared-expert gate as row E), then per token
// the top-k of softmax(logits + bias), renormalised to sum 1 (engines/base.py:91-97 with norm_topk_prob), and
// sigmoid(x . g) (engines/base.py:104-107).
//
// The renormalised weights are exp(l_i - l_0) / sum_j exp(l_j - l_0) over the k selected logits (l_0 the largest):
// the full softmax denominator cancels in p_i / sum_j p_j, so it is never formed.
#include "common.cuh"
#include "kernels.cuh"

namespace wmoe {

template <typename XT>
__device__ __forceinline__ float4 load4(const XT* p);
template <>
__device__ __forceinline__ float4 load4<float>(const float* p) { return *reinterpret_cast<const float4*>(p); }
template <>
__device__ __forceinline__ float4 load4<__nv_bfloat16>(const __nv_bfloat16* p) {
  const uint2 v = *reinterpret_cast<const uint2*>(p);
  return make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xFFFF0000u), __uint_as_float(v.y << 16),
                     __uint_as_float(v.y & 0xFFFF0000u));
}

// Few tokens: one warp per router row, every token at once (T <= 8). Grid covers E + 1 rows.
template <typename XT, int TMAX>
__global__ void __launch_bounds__(256) router_gemv_kernel(const XT* __restrict__ x, int T, int H, int E,
                                                          const float* __restrict__ R,
                                                          const float* __restrict__ g,
                                                          float* __restrict__ logits) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int e = blockIdx.x * 8 + warp;
  if (e > E || (e == E && g == nullptr)) return;
  const float* row = e < E ? R + size_t(e) * H : g;
  float acc[TMAX];
#pragma unroll
  for (int t = 0; t < TMAX; ++t) acc[t] = 0.f;
  for (int k = lane * 4; k < H; k += 128) {
    const float4 w = __ldg(reinterpret_cast<const float4*>(row + k));
#pragma unroll
    for (int t = 0; t < TMAX; ++t) {
      if (t < T) {
        const float4 v = load4<XT>(x + size_t(t) * H + k);
        acc[t] = fmaf(w.x, v.x, acc[t]);
        acc[t] = fmaf(w.y, v.y, acc[t]);
        acc[t] = fmaf(w.z, v.z, acc[t]);
        acc[t] = fmaf(w.w, v.w, acc[t]);
      }
    }
  }
#pragma unroll
  for (int t = 0; t < TMAX; ++t) {
    if (t < T) {
      const float s = warp_sum(acc[t]);
      if (lane == 0) logits[size_t(t) * (E + 1) + e] = s;
    }
  }
}

// Many tokens: a 64 x 64 tile of logits per CTA (256 threads, 4 x 4 each), K in steps of 32 through shared memory.
template <typename XT>
__global__ void __launch_bounds__(256) router_gemm_kernel(const XT* __restrict__ x, int T, int H, int E,
                                                          const float* __restrict__ R,
                                                          const float* __restrict__ g,
                                                          float* __restrict__ logits) {
  constexpr int BM = 64, BN = 64, BK = 32;
  __shared__ float xs[BK][BM + 4];
  __shared__ float ws[BK][BN + 4];
  const int t0 = blockIdx.x * BM, e0 = blockIdx.y * BN;
  const int tid = threadIdx.x;
  const int rows = E + (g != nullptr ? 1 : 0);
  const int ty = tid / 16, tx = tid % 16;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < H; k0 += BK) {
    // 64 rows x 32 columns of x and of the weights: 2048 values each, 8 per thread (two float4)
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int idx = tid + i * 256;  // 0..511 float4 slots
      const int r = idx / 8, c = (idx % 8) * 4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (t0 + r < T) v = load4<XT>(x + size_t(t0 + r) * H + k0 + c);
      xs[c + 0][r] = v.x;
      xs[c + 1][r] = v.y;
      xs[c + 2][r] = v.z;
      xs[c + 3][r] = v.w;
      float4 w = make_float4(0.f, 0.f, 0.f, 0.f);
      const int e = e0 + r;
      if (e < E)
        w = __ldg(reinterpret_cast<const float4*>(R + size_t(e) * H + k0 + c));
      else if (e < rows)
        w = __ldg(reinterpret_cast<const float4*>(g + k0 + c));
      ws[c + 0][r] = w.x;
      ws[c + 1][r] = w.y;
      ws[c + 2][r] = w.z;
      ws[c + 3][r] = w.w;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = xs[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = ws[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = t0 + ty * 4 + i;
    if (t >= T) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = e0 + tx * 4 + j;
      if (e < rows) logits[size_t(t) * (E + 1) + e] = acc[i][j];
    }
  }
}

cudaError_t router_logits(const void* x, int x_dtype, int T, int H, int E, const float* R, const float* g,
                          float* logits, cudaStream_t st, int* launches) {
  if (T <= 8) {
    const unsigned grid = unsigned((E + 1 + 7) / 8);
    if (x_dtype == kF32)
      router_gemv_kernel<float, 8><<<grid, 256, 0, st>>>(static_cast<const float*>(x), T, H, E, R, g, logits);
    else
      router_gemv_kernel<__nv_bfloat16, 8><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), T, H, E, R,
                                                                   g, logits);
  } else {
    const dim3 grid(unsigned((T + 63) / 64), unsigned((E + 1 + 63) / 64));
    if (x_dtype == kF32)
      router_gemm_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(x), T, H, E, R, g, logits);
    else
      router_gemm_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), T, H, E, R, g,
                                                               logits);
  }
  ++*launches;
  return cudaGetLastError();
}

// One warp per token: k rounds of warp arg-max (larger value first, then the smaller expert id).
// splits == 0: logits [T][E + 1], column E the shared-expert gate logit. splits > 0: `splits` partial sums
// [splits][T][E] added in order, and the shared-expert gate logit is x[t] . g computed here.
template <int PER_LANE>
__global__ void __launch_bounds__(256) topk_kernel(const float* __restrict__ logits, int splits, int T, int E, int k,
                                                   const float* __restrict__ bias, float* __restrict__ topk_w,
                                                   int32_t* __restrict__ topk_idx, float* __restrict__ shared_s,
                                                   float* __restrict__ logits_out, const void* __restrict__ x,
                                                   int x_dtype, const float* __restrict__ g, int H) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int t = blockIdx.x * 8 + warp;
  if (t >= T) return;
  const float* row = logits + size_t(t) * (E + 1);
  float v[PER_LANE];
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i) {
    const int e = lane + 32 * i;
    float l = -INFINITY;
    if (e < E) {
      if (splits == 0) {
        l = row[e];
      } else {
        l = logits[size_t(t) * E + e];
        for (int s = 1; s < splits; ++s) l += logits[(size_t(s) * T + t) * E + e];
      }
      if (bias) l += bias[e];
      if (logits_out) logits_out[size_t(t) * E + e] = l;
    }
    v[i] = l;
  }
  float top0 = 0.f, sum = 0.f;
  float sel_l = 0.f;
  int sel_e = 0;
  for (int r = 0; r < k; ++r) {
    float best = -INFINITY;
    int best_e = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) {
      const int e = lane + 32 * i;
      if (e < E && (v[i] > best || (v[i] == best && e < best_e))) {
        best = v[i];
        best_e = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oe = __shfl_xor_sync(0xffffffffu, best_e, o);
      if (ob > best || (ob == best && oe < best_e)) {
        best = ob;
        best_e = oe;
      }
    }
    // remove the winner from its lane
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i)
      if (lane + 32 * i == best_e) v[i] = -INFINITY;
    if (r == 0) top0 = best;
    const float ex = expf(best - top0);
    sum += ex;
    if (lane == r) {
      sel_l = ex;
      sel_e = best_e;
    }
  }
  if (lane < k) {
    topk_w[size_t(t) * k + lane] = sel_l / sum;
    topk_idx[size_t(t) * k + lane] = sel_e;
  }
  if (shared_s) {
    float sl;
    if (splits == 0) {
      sl = row[E];
    } else {
      float acc = 0.f;
      for (int h = lane * 4; h < H; h += 128) {
        const float4 w = __ldg(reinterpret_cast<const float4*>(g + h));
        const float4 xv = x_dtype == kF32 ? load4<float>(static_cast<const float*>(x) + size_t(t) * H + h)
                                          : load4<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(x) + size_t(t) * H + h);
        acc = fmaf(w.x, xv.x, acc);
        acc = fmaf(w.y, xv.y, acc);
        acc = fmaf(w.z, xv.z, acc);
        acc = fmaf(w.w, xv.w, acc);
      }
      sl = warp_sum(acc);
    }
    if (lane == 0) shared_s[t] = 1.0f / (1.0f + expf(-sl));
  }
}

// out[h][e] = R[e][h] for e < E, out[h][E] = g[h], zero up to the stride: 32 x 32 tiles through shared memory.
__global__ void pack_router_kernel(const float* __restrict__ R, const float* __restrict__ g, int E, int H,
                                   float* __restrict__ out) {
  __shared__ float tile[32][33];
  const int e0 = blockIdx.y * 32, h0 = blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int e = e0 + i, h = h0 + threadIdx.x;
    float v = 0.f;
    if (h < H) v = e < E ? R[size_t(e) * H + h] : (e == E ? g[h] : 0.f);
    tile[i][threadIdx.x] = v;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int h = h0 + i, e = e0 + threadIdx.x;
    if (h < H && e < kRouterStride) out[size_t(h) * kRouterStride + e] = tile[threadIdx.x][i];
  }
}

cudaError_t pack_router(const float* router_w, const float* shared_gate, int E, int H, float* out, cudaStream_t st) {
  const dim3 grid(unsigned((H + 31) / 32), unsigned((kRouterStride + 31) / 32));
  pack_router_kernel<<<grid, dim3(32, 8), 0, st>>>(router_w, shared_gate, E, H, out);
  return cudaGetLastError();
}

cudaError_t router_topk_split(const float* logits, int splits, int T, int E, int k, const float* bias, float* topk_w,
                              int32_t* topk_idx, float* shared_s, float* logits_out, const void* x, int x_dtype,
                              const float* g, int H, cudaStream_t st, int* launches) {
  const unsigned grid = unsigned((T + 7) / 8);
  if (E <= 256)
    topk_kernel<8><<<grid, 256, 0, st>>>(logits, splits, T, E, k, bias, topk_w, topk_idx, shared_s, logits_out, x,
                                         x_dtype, g, H);
  else
    topk_kernel<16><<<grid, 256, 0, st>>>(logits, splits, T, E, k, bias, topk_w, topk_idx, shared_s, logits_out, x,
                                          x_dtype, g, H);
  ++*launches;
  return cudaGetLastError();
}

cudaError_t router_topk(const float* logits, int T, int E, int k, const float* bias, float* topk_w,
                        int32_t* topk_idx, float* shared_s, float* logits_out, cudaStream_t st, int* launches) {
  return router_topk_split(logits, 0, T, E, k, bias, topk_w, topk_idx, shared_s, logits_out, nullptr, kF32, nullptr,
                           0, st, launches);
}

}  // namespace wmoe
