// Q4_K / Q6_K super-blocks -> f32 (bit-identical to gguf/quants.py:dequantize), bf16 or f16 (RNE of that).
// One thread per 32-value chunk. Products and differences use __fmul_rn/__fsub_rn so nvcc cannot contract them
// into an FMA: the reference rounds d*sc, then scale*q, then the subtraction, each to float32
// (gguf/quants.py:87-92, 104-116; gguf/metal.py:133-168).
#include "common.cuh"
#include "kernels.cuh"

namespace wmoe {

template <typename OutT>
__device__ __forceinline__ OutT cast_out(float v);
template <>
__device__ __forceinline__ float cast_out<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 cast_out<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half cast_out<__half>(float v) { return __float2half_rn(v); }

template <typename OutT>
__global__ void dequant_q4k_kernel(const uint8_t* __restrict__ blocks, size_t nblocks, OutT* __restrict__ out) {
  const size_t chunk = blockIdx.x * size_t(blockDim.x) + threadIdx.x;
  if (chunk >= nblocks * 8) return;
  const size_t n = chunk / 8;
  const int j = int(chunk % 8);
  const uint8_t* b = blocks + n * Q4K_BYTES;
  const float d = f16_to_f32(uint16_t(b[0] | (b[1] << 8)));
  const float dmin = f16_to_f32(uint16_t(b[2] | (b[3] << 8)));
  int sc, mn;
  q4k_scale_min(b + 4, j, sc, mn);
  const float scale = __fmul_rn(d, float(sc));
  const float m = __fmul_rn(dmin, float(mn));
  const uint8_t* qs = b + 16 + 32 * (j / 2);
  const int shift = 4 * (j % 2);
  OutT* o = out + n * QK + 32 * j;
#pragma unroll 8
  for (int l = 0; l < 32; ++l) {
    const int q = (qs[l] >> shift) & 0x0F;
    o[l] = cast_out<OutT>(__fsub_rn(__fmul_rn(scale, float(q)), m));
  }
}

template <typename OutT>
__global__ void dequant_q6k_kernel(const uint8_t* __restrict__ blocks, size_t nblocks, OutT* __restrict__ out) {
  const size_t chunk = blockIdx.x * size_t(blockDim.x) + threadIdx.x;
  if (chunk >= nblocks * 8) return;
  const size_t n = chunk / 8;
  const int c = int(chunk % 8), h = c / 4, s = c % 4;
  const uint8_t* b = blocks + n * Q6K_BYTES;
  const float d = f16_to_f32(uint16_t(b[208] | (b[209] << 8)));
  const float scale0 = __fmul_rn(d, float(int8_t(b[192 + 2 * c])));
  const float scale1 = __fmul_rn(d, float(int8_t(b[193 + 2 * c])));
  const uint8_t* ql = b + 64 * h + 32 * (s % 2);
  const uint8_t* qh = b + 128 + 32 * h;
  const int lshift = 4 * (s / 2), hshift = 2 * s;
  OutT* o = out + n * QK + 32 * c;
#pragma unroll 8
  for (int l = 0; l < 32; ++l) {
    const int q = int(((ql[l] >> lshift) & 0x0F) | (((qh[l] >> hshift) & 3) << 4)) - 32;
    o[l] = cast_out<OutT>(__fmul_rn(l < 16 ? scale0 : scale1, float(q)));
  }
}

template <typename OutT>
static cudaError_t launch_dequant(int type, const uint8_t* blocks, size_t nblocks, OutT* out, cudaStream_t st) {
  const size_t chunks = nblocks * 8;
  const int threads = 256;
  const unsigned grid = unsigned((chunks + threads - 1) / threads);
  if (type == kGgmlQ4K)
    dequant_q4k_kernel<OutT><<<grid, threads, 0, st>>>(blocks, nblocks, out);
  else
    dequant_q6k_kernel<OutT><<<grid, threads, 0, st>>>(blocks, nblocks, out);
  return cudaGetLastError();
}

cudaError_t dequant(int type, const uint8_t* blocks, size_t nblocks, void* out, int out_dtype, cudaStream_t st) {
  if (nblocks == 0) return cudaSuccess;
  switch (out_dtype) {
    case kF32: return launch_dequant(type, blocks, nblocks, static_cast<float*>(out), st);
    case kBF16: return launch_dequant(type, blocks, nblocks, static_cast<__nv_bfloat16*>(out), st);
    default: return launch_dequant(type, blocks, nblocks, static_cast<__half*>(out), st);
  }
}

}  // namespace wmoe
