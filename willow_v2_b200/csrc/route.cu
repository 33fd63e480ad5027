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

// More than 8 tokens: the router logits without the shared gate (the top-k kernel forms that one from x). Every logit
// is a sequential fma chain over each kRouterSlice-wide K slice, and the slices are added in ascending order, whether
// one CTA walks all of them (`slices_per_cta` = H / kRouterSlice, one output [T][E]) or each CTA takes one slice and
// writes it as a partial sum ([H / kRouterSlice][T][E], added in order by the top-k kernel). A token's logits are
// therefore the same bits whatever other tokens share its call.
// CTA: 64 tokens x 64 router rows, 256 threads with 4 x 4 logits each; K in steps of 32 through two shared-memory
// buffers, the next step's global loads held in registers while the current step computes.
constexpr int kRouterSlice = 128, kRouterSplitMaxT = 1024;

template <typename XT>
__global__ void __launch_bounds__(256) router_slices_kernel(const XT* __restrict__ x, int T, int H, int E,
                                                            const float* __restrict__ R, int slices_per_cta,
                                                            float* __restrict__ out) {
  constexpr int BM = 64, BN = 64, BK = 32, kSteps = kRouterSlice / BK;
  __shared__ __align__(16) float xs[2][BK][BM + 4];
  __shared__ __align__(16) float ws[2][BK][BN + 4];
  const int t0 = blockIdx.x * BM, e0 = blockIdx.y * BN;
  const int k_begin = blockIdx.z * slices_per_cta * kRouterSlice;
  const int nsteps = slices_per_cta * kSteps;
  const int tid = threadIdx.x, ty = tid / 16, tx = tid % 16;
  float4 xv[2], wv[2];
  auto fetch = [&](int k0) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int idx = tid + i * 256, r = idx / 8, c = (idx % 8) * 4;
      xv[i] = t0 + r < T ? load4<XT>(x + size_t(t0 + r) * H + k0 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      wv[i] = e0 + r < E ? __ldg(reinterpret_cast<const float4*>(R + size_t(e0 + r) * H + k0 + c))
                         : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  auto stash = [&](int b) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int idx = tid + i * 256, r = idx / 8, c = (idx % 8) * 4;
      xs[b][c][r] = xv[i].x, xs[b][c + 1][r] = xv[i].y, xs[b][c + 2][r] = xv[i].z, xs[b][c + 3][r] = xv[i].w;
      ws[b][c][r] = wv[i].x, ws[b][c + 1][r] = wv[i].y, ws[b][c + 2][r] = wv[i].z, ws[b][c + 3][r] = wv[i].w;
    }
  };
  float acc[4][4], total[4][4];
  fetch(k_begin);
  stash(0);
  __syncthreads();
  for (int s = 0; s < nsteps; ++s) {
    const int b = s & 1;
    if (s + 1 < nsteps) fetch(k_begin + (s + 1) * BK);
    if (s % kSteps == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
    }
#pragma unroll 8
    for (int kk = 0; kk < BK; ++kk) {
      const float4 a = *reinterpret_cast<const float4*>(&xs[b][kk][ty * 4]);
      const float4 w = *reinterpret_cast<const float4*>(&ws[b][kk][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, wv4[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], wv4[j], acc[i][j]);
    }
    if (s % kSteps == kSteps - 1) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) total[i][j] = s < kSteps ? acc[i][j] : total[i][j] + acc[i][j];
    }
    if (s + 1 < nsteps) stash(b ^ 1);
    __syncthreads();
  }
  float* o = out + size_t(blockIdx.z) * T * E;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = t0 + ty * 4 + i;
    if (t >= T) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = e0 + tx * 4 + j;
      if (e < E) o[size_t(t) * E + e] = total[i][j];
    }
  }
}

int router_slice_outputs(int T, int H) { return T <= kRouterSplitMaxT ? H / kRouterSlice : 1; }

cudaError_t router_logits_sliced(const void* x, int x_dtype, int T, int H, int E, const float* R, float* out,
                                 cudaStream_t st, int* launches) {
  if (T <= 0 || H % kRouterSlice) return cudaErrorInvalidValue;
  const int outputs = router_slice_outputs(T, H);
  const dim3 grid(unsigned((T + 63) / 64), unsigned((E + 63) / 64), unsigned(outputs));
  const int per_cta = H / kRouterSlice / outputs;
  if (x_dtype == kF32)
    router_slices_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(x), T, H, E, R, per_cta, out);
  else
    router_slices_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), T, H, E, R,
                                                              per_cta, out);
  ++*launches;
  return cudaGetLastError();
}

cudaError_t router_logits(const void* x, int x_dtype, int T, int H, int E, const float* R, const float* g,
                          float* logits, cudaStream_t st, int* launches) {
  if (T > 8) return cudaErrorInvalidValue;  // router_logits_sliced
  const unsigned grid = unsigned((E + 1 + 7) / 8);
  if (x_dtype == kF32)
    router_gemv_kernel<float, 8><<<grid, 256, 0, st>>>(static_cast<const float*>(x), T, H, E, R, g, logits);
  else
    router_gemv_kernel<__nv_bfloat16, 8><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), T, H, E, R, g,
                                                                 logits);
  ++*launches;
  return cudaGetLastError();
}

// k rounds of warp arg-max over a lane's PER_LANE logits (lane + 32 i): the larger value first, then the smaller
// expert id; the renormalised weights exp(l_i - l_0) / sum_j exp(l_j - l_0) of the picks, in pick order.
template <int PER_LANE>
__device__ __forceinline__ void select_topk(float (&v)[PER_LANE], int lane, int E, int k, float* __restrict__ w_out,
                                            int32_t* __restrict__ idx_out) {
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
    w_out[lane] = sel_l / sum;
    idx_out[lane] = sel_e;
  }
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
  const float* row = splits == 0 ? logits + size_t(t) * (E + 1) : logits + size_t(t) * E;
  float v[PER_LANE];
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i) v[i] = lane + 32 * i < E ? row[lane + 32 * i] : -INFINITY;
  // partial sums added in order, each pass issuing the loads of all of a lane's logits at once (four passes' loads
  // in flight)
#pragma unroll 4
  for (int s = 1; s < splits; ++s) {
    const float* part = logits + (size_t(s) * T + t) * E;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i)
      if (lane + 32 * i < E) v[i] += part[lane + 32 * i];
  }
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i) {
    const int e = lane + 32 * i;
    if (e < E) {
      if (bias) v[i] += bias[e];
      if (logits_out) logits_out[size_t(t) * E + e] = v[i];
    }
  }
  select_topk<PER_LANE>(v, lane, E, k, topk_w + size_t(t) * k, topk_idx + size_t(t) * k);
  if (shared_s) {
    float sl;
    if (splits == 0) {
      sl = row[E];
    } else {
      // four quarter sums of H / 4, each a lane-strided fma chain and a warp tree, added as ((q0 + q1) + (q2 + q3)):
      // the same bits as topk_split_kernel's four warps
      const int quarters = H % 512 == 0 ? 4 : 1;
      float gq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (q >= quarters) break;
        const int h0 = q * (H / quarters), h1 = (q + 1) * (H / quarters);
        float acc = 0.f;
#pragma unroll 4
        for (int h = h0 + lane * 4; h < h1; h += 128) {
          const float4 w = __ldg(reinterpret_cast<const float4*>(g + h));
          const float4 xv = x_dtype == kF32 ? load4<float>(static_cast<const float*>(x) + size_t(t) * H + h)
                                            : load4<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(x) + size_t(t) * H + h);
          acc = fmaf(w.x, xv.x, acc);
          acc = fmaf(w.y, xv.y, acc);
          acc = fmaf(w.z, xv.z, acc);
          acc = fmaf(w.w, xv.w, acc);
        }
        gq[q] = warp_sum(acc);
      }
      sl = quarters == 4 ? (gq[0] + gq[1]) + (gq[2] + gq[3]) : gq[0];
    }
    if (lane == 0) shared_s[t] = 1.0f / (1.0f + expf(-sl));
  }
}

// Top-k from 1..16 partial logit sums with E <= 256 and H a multiple of 512 (the sliced and tensor-core routers):
// two tokens per CTA, four warps per token. Warp q adds, for experts [64q, 64q + 64), every partial in order with
// all of them loaded at once, and forms a quarter of the shared-gate dot product; one warp per token then selects.
// Per-logit arithmetic and the shared-gate sum ((q0 + q1) + (q2 + q3)) are those of topk_kernel.
constexpr int kFastSplits = 16;

__global__ void __launch_bounds__(256) topk_split_kernel(const float* __restrict__ logits, int splits, int T, int E,
                                                         int k, const float* __restrict__ bias,
                                                         float* __restrict__ topk_w, int32_t* __restrict__ topk_idx,
                                                         float* __restrict__ shared_s, float* __restrict__ logits_out,
                                                         const void* __restrict__ x, int x_dtype,
                                                         const float* __restrict__ g, int H) {
  __shared__ float lg[2][256];
  __shared__ float gq[2][4];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int tl = warp / 4, q = warp % 4;
  const int t = blockIdx.x * 2 + tl;
  if (t < T) {
    float p[2][kFastSplits];
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      const int e = 64 * q + 32 * m + lane;
#pragma unroll
      for (int s = 0; s < kFastSplits; ++s)
        p[m][s] = s < splits && e < E ? logits[(size_t(s) * T + t) * E + e] : 0.f;
    }
    float acc = 0.f;
    if (shared_s) {
      const int h1 = (q + 1) * (H / 4);
#pragma unroll 4
      for (int h = q * (H / 4) + lane * 4; h < h1; h += 128) {
        const float4 w = __ldg(reinterpret_cast<const float4*>(g + h));
        const float4 xv = x_dtype == kF32 ? load4<float>(static_cast<const float*>(x) + size_t(t) * H + h)
                                          : load4<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(x) + size_t(t) * H + h);
        acc = fmaf(w.x, xv.x, acc);
        acc = fmaf(w.y, xv.y, acc);
        acc = fmaf(w.z, xv.z, acc);
        acc = fmaf(w.w, xv.w, acc);
      }
    }
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      const int e = 64 * q + 32 * m + lane;
      float v = p[m][0];
#pragma unroll
      for (int s = 1; s < kFastSplits; ++s)
        if (s < splits) v += p[m][s];
      if (e < E) {
        if (bias) v += bias[e];
        if (logits_out) logits_out[size_t(t) * E + e] = v;
      }
      lg[tl][e] = e < E ? v : -INFINITY;
    }
    if (shared_s) {
      acc = warp_sum(acc);
      if (lane == 0) gq[tl][q] = acc;
    }
  }
  __syncthreads();
  if (t >= T || q != 0) return;
  float v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = lg[tl][lane + 32 * i];
  select_topk<8>(v, lane, E, k, topk_w + size_t(t) * k, topk_idx + size_t(t) * k);
  if (shared_s && lane == 0) {
    const float sl = (gq[tl][0] + gq[tl][1]) + (gq[tl][2] + gq[tl][3]);
    shared_s[t] = 1.0f / (1.0f + expf(-sl));
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

// willow's skip_small_experts (engines/base.py:413-429) on the renormalised weights of T tokens, one thread per
// token: pick j of a token is kept when j == 0 (the largest weight; picks are in descending order) or its weight is
// >= min_w; the kept weights are scaled so that they add up to the picks' former total, the dropped ones become 0.
// The expert ids stay as they are: a dropped pick's expert is then added with weight 0, which leaves every sum
// unchanged.
__global__ void skip_small_kernel(float* __restrict__ topk_w, int T, int k, float min_w) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  float* w = topk_w + size_t(t) * k;
  float total = 0.f, kept = 0.f;
  for (int j = 0; j < k; ++j) {
    total += w[j];
    if (j == 0 || w[j] >= min_w) kept += w[j];
  }
  const float scale = total / kept;
  for (int j = 0; j < k; ++j) w[j] = (j == 0 || w[j] >= min_w) ? w[j] * scale : 0.f;
}

cudaError_t skip_small_experts(float* topk_w, int T, int k, float min_w, cudaStream_t st, int* launches) {
  if (T <= 0 || !(min_w > 0.f)) return cudaSuccess;
  skip_small_kernel<<<unsigned((T + 255) / 256), 256, 0, st>>>(topk_w, T, k, min_w);
  ++*launches;
  return cudaGetLastError();
}

// out[i] = idx[i], or -1 where the pick's weight is 0 (dropped by skip_small_experts), as willow marks them
__global__ void mark_dropped_kernel(const int32_t* __restrict__ idx, const float* __restrict__ w,
                                    int32_t* __restrict__ out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = w[i] == 0.f ? -1 : idx[i];
}

cudaError_t mark_dropped(const int32_t* idx, const float* w, int32_t* out, int n, cudaStream_t st, int* launches) {
  if (n <= 0) return cudaSuccess;
  mark_dropped_kernel<<<unsigned((n + 255) / 256), 256, 0, st>>>(idx, w, out, n);
  ++*launches;
  return cudaGetLastError();
}

cudaError_t pack_router(const float* router_w, const float* shared_gate, int E, int H, float* out, cudaStream_t st) {
  const dim3 grid(unsigned((H + 31) / 32), unsigned((kRouterStride + 31) / 32));
  pack_router_kernel<<<grid, dim3(32, 8), 0, st>>>(router_w, shared_gate, E, H, out);
  return cudaGetLastError();
}

cudaError_t router_topk_split(const float* logits, int splits, int T, int E, int k, const float* bias, float* topk_w,
                              int32_t* topk_idx, float* shared_s, float* logits_out, const void* x, int x_dtype,
                              const float* g, int H, cudaStream_t st, int* launches) {
  // up to 1024 tokens four warps per token (topk_kernel has too few CTAs there); above, one warp per token keeps
  // more selecting warps per SM. Both give the same bits.
  if (splits >= 1 && splits <= kFastSplits && E <= 256 && H % 512 == 0 && k <= 32 && T <= 1024) {
    topk_split_kernel<<<unsigned((T + 1) / 2), 256, 0, st>>>(logits, splits, T, E, k, bias, topk_w, topk_idx, shared_s,
                                                             logits_out, x, x_dtype, g, H);
    ++*launches;
    return cudaGetLastError();
  }
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
