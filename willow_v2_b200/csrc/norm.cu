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

template <typename YT, typename NT>
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(const float* x, const YT* __restrict__ y, int H, float eps,
                                                          float* x_out, NT* __restrict__ xn) {  // x_out may be x
  __shared__ float red[8];
  const size_t row = size_t(blockIdx.x) * H;
  const int tid = threadIdx.x;
  float ss = 0.f;
  for (int h = tid * 4; h < H; h += 1024) {
    float4 v = ld4(x + row + h);
    if (y) {
      const float4 a = ld4(y + row + h);
      v.x += a.x, v.y += a.y, v.z += a.z, v.w += a.w;
    }
    st4(x_out + row + h, v);
    ss = fmaf(v.x, v.x, ss);
    ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss);
    ss = fmaf(v.w, v.w, ss);
  }
  ss = warp_sum(ss);
  if (tid % 32 == 0) red[tid / 32] = ss;
  __syncthreads();
  float t = tid < 8 ? red[tid] : 0.f;
  if (tid < 32) t = warp_sum(t);
  if (tid == 0) red[0] = t;
  __syncthreads();
  const float r = rsqrtf(red[0] / float(H) + eps);
  for (int h = tid * 4; h < H; h += 1024) {
    const float4 v = ld4(x_out + row + h);
    st4(xn + row + h, make_float4(v.x * r, v.y * r, v.z * r, v.w * r));
  }
}

template <typename YT>
static void launch_norm(const float* x, const YT* y, int T, int H, float eps, float* x_out, void* xn, int xn_dtype,
                        cudaStream_t st) {
  if (xn_dtype == kF32)
    add_rmsnorm_kernel<YT, float><<<T, 256, 0, st>>>(x, y, H, eps, x_out, static_cast<float*>(xn));
  else
    add_rmsnorm_kernel<YT, __nv_bfloat16><<<T, 256, 0, st>>>(x, y, H, eps, x_out, static_cast<__nv_bfloat16*>(xn));
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
