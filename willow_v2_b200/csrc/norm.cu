// Residual add + RMS normalisation between MoE layers (engines/qwen36/model.py:17-22, engines/base.py:27-32 with
// weight 1): x_out = x + y, xn = x_out / sqrt(mean(x_out^2) + eps). One CTA per token row, float32 arithmetic; the
// sum of squares is reduced in a fixed order (per-thread partials, then warp and CTA trees), so a row's result does
// not depend on the batch it is in.
#include "common.cuh"
#include "kernels.cuh"

namespace wmoe {

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 ld4(const __nv_bfloat16* p) {
  const uint2 v = *reinterpret_cast<const uint2*>(p);
  return make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xFFFF0000u), __uint_as_float(v.y << 16),
                     __uint_as_float(v.y & 0xFFFF0000u));
}
__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ void st4(__nv_bfloat16* p, float4 v) {
  const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
  *reinterpret_cast<uint2*>(p) =
      make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
}

// W consecutive values per thread (8 when H % 8 == 0: the partition and summation order of the combine kernels'
// residual epilogue, so that a layer's fused and unfused glue give the same bits; else 4).
template <int W>
__device__ __forceinline__ void load_row(const float* p, float* v) {
#pragma unroll
  for (int j = 0; j < W; j += 4) {
    const float4 a = ld4(p + j);
    v[j] = a.x, v[j + 1] = a.y, v[j + 2] = a.z, v[j + 3] = a.w;
  }
}
template <int W, typename YT>
__device__ __forceinline__ void add_row(const YT* p, float* v) {
#pragma unroll
  for (int j = 0; j < W; j += 4) {
    const float4 a = ld4(p + j);
    v[j] += a.x, v[j + 1] += a.y, v[j + 2] += a.z, v[j + 3] += a.w;
  }
}
template <int W, typename T>
__device__ __forceinline__ void store_row(T* p, const float* v) {
#pragma unroll
  for (int j = 0; j < W; j += 4) st4(p + j, make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
}

template <int W, typename YT, typename NT>
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(const float* x, const YT* __restrict__ y, int H, float eps,
                                                          float* x_out, NT* __restrict__ xn) {  // x_out may be x
  __shared__ float red[32];
  const size_t row = size_t(blockIdx.x) * H;
  float ss = 0.f;
  for (int h = threadIdx.x * W; h < H; h += blockDim.x * W) {
    float v[W];
    load_row<W>(x + row + h, v);
    if (y) add_row<W>(y + row + h, v);
    store_row<W>(x_out + row + h, v);
#pragma unroll
    for (int j = 0; j < W; ++j) ss = fmaf(v[j], v[j], ss);
  }
  const float r = rsqrtf(block_sum(ss, red) / float(H) + eps);
  for (int h = threadIdx.x * W; h < H; h += blockDim.x * W) {
    float v[W];
    load_row<W>(x_out + row + h, v);
#pragma unroll
    for (int j = 0; j < W; ++j) v[j] *= r;
    store_row<W>(xn + row + h, v);
  }
}

template <typename YT>
static void launch_norm(const float* x, const YT* y, int T, int H, float eps, float* x_out, void* xn, int xn_dtype,
                        cudaStream_t st) {
  float* xf = static_cast<float*>(xn);
  __nv_bfloat16* xb = static_cast<__nv_bfloat16*>(xn);
  if (H % 8 == 0) {
    if (xn_dtype == kF32)
      add_rmsnorm_kernel<8, YT, float><<<T, 256, 0, st>>>(x, y, H, eps, x_out, xf);
    else
      add_rmsnorm_kernel<8, YT, __nv_bfloat16><<<T, 256, 0, st>>>(x, y, H, eps, x_out, xb);
  } else if (xn_dtype == kF32) {
    add_rmsnorm_kernel<4, YT, float><<<T, 256, 0, st>>>(x, y, H, eps, x_out, xf);
  } else {
    add_rmsnorm_kernel<4, YT, __nv_bfloat16><<<T, 256, 0, st>>>(x, y, H, eps, x_out, xb);
  }
}

cudaError_t add_rmsnorm(const float* x, const void* y, int y_dtype, int T, int H, float eps, float* x_out, void* xn,
                        int xn_dtype, cudaStream_t st, int* launches) {
  if (y_dtype == kBF16 && y)
    launch_norm(x, static_cast<const __nv_bfloat16*>(y), T, H, eps, x_out, xn, xn_dtype, st);
  else
    launch_norm(x, static_cast<const float*>(y), T, H, eps, x_out, xn, xn_dtype, st);
  ++*launches;
  return cudaGetLastError();
}

}  // namespace wmoe
