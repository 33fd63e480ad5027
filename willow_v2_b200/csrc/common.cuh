// Shared definitions for the sm_100a MoE kernels: block layouts, device status codes, small device helpers.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace wmoe {

constexpr int QK = 256;          // values per K-quant super-block
constexpr int Q4K_BYTES = 144;   // d, dmin (fp16), 12 scale bytes, 128 quant bytes
constexpr int Q6K_BYTES = 210;   // ql[128], qh[64], int8 scales[16], d (fp16)
constexpr int XQ_BLOCK = 32;     // activations are quantised to int16 in blocks of 32 values

// Device status causes (written once, first writer wins; read back by wmoe_device_status)
enum DeviceStatus : int {
  kStatusOk = 0,
  kStatusBadExpert = 1,
  kStatusNotResident = 2,
  kStatusBarrierTimeout = 3,
  kStatusBadSegment = 4,
};

__device__ __forceinline__ void set_status(int* status, int cause) {
  if (status) atomicCAS(status, 0, cause);
}

__device__ __forceinline__ float f16_to_f32(uint16_t bits) { return __half2float(__ushort_as_half(bits)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ int warp_sum_int(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// d = c + a.lo16 * b.byte0 + a.hi16 * b.byte1  (signed 16-bit x unsigned 8-bit)
__device__ __forceinline__ int dp2a_lo(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// d = c + a.lo16 * b.byte2 + a.hi16 * b.byte3
__device__ __forceinline__ int dp2a_hi(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp2a.hi.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t ldg_nc_u32(const void* p) {
  uint32_t v;
  asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// 16 bytes starting at a 2-byte aligned global address (Q6_K super-blocks are 210 B, so half of them start
// 2 bytes past a 4-byte boundary): five aligned 32-bit loads and funnel shifts.
__device__ __forceinline__ uint4 ldg_u2_16(const uint8_t* p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  const uint32_t sh = (a & 3u) * 8u;
  uint32_t w0 = ldg_nc_u32(w), w1 = ldg_nc_u32(w + 1), w2 = ldg_nc_u32(w + 2), w3 = ldg_nc_u32(w + 3);
  uint4 r;
  if (sh == 0) {
    r = make_uint4(w0, w1, w2, w3);
  } else {
    uint32_t w4 = ldg_nc_u32(w + 4);
    r.x = __funnelshift_r(w0, w1, sh);
    r.y = __funnelshift_r(w1, w2, sh);
    r.z = __funnelshift_r(w2, w3, sh);
    r.w = __funnelshift_r(w3, w4, sh);
  }
  return r;
}

// The same from shared memory.
__device__ __forceinline__ uint4 lds_u2_16(const uint8_t* p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  const uint32_t sh = (a & 3u) * 8u;
  uint32_t w0 = w[0], w1 = w[1], w2 = w[2], w3 = w[3];
  uint4 r;
  if (sh == 0) {
    r = make_uint4(w0, w1, w2, w3);
  } else {
    uint32_t w4 = w[4];
    r.x = __funnelshift_r(w0, w1, sh);
    r.y = __funnelshift_r(w1, w2, sh);
    r.z = __funnelshift_r(w2, w3, sh);
    r.w = __funnelshift_r(w3, w4, sh);
  }
  return r;
}

// Q4_K 6-bit scale and min of sub-block j (0..7) from the 12 scale bytes s (gguf/quants.py:73-80)
__device__ __forceinline__ void q4k_scale_min(const uint8_t* s, int j, int& sc, int& mn) {
  if (j < 4) {
    sc = s[j] & 63;
    mn = s[j + 4] & 63;
  } else {
    sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 2) & 0x30);
    mn = (s[j + 4] >> 4) | ((s[j] >> 2) & 0x30);
  }
}

// The same from the 12 bytes held as three 32-bit words (little-endian).
__device__ __forceinline__ void q4k_scale_min_w(uint32_t s0, uint32_t s1, uint32_t s2, int j, int& sc, int& mn) {
  auto byte = [&](int i) -> int {
    uint32_t w = i < 4 ? s0 : (i < 8 ? s1 : s2);
    return (w >> (8 * (i & 3))) & 0xFF;
  };
  if (j < 4) {
    sc = byte(j) & 63;
    mn = byte(j + 4) & 63;
  } else {
    sc = (byte(j + 4) & 0x0F) | ((byte(j - 4) >> 2) & 0x30);
    mn = (byte(j + 4) >> 4) | ((byte(j) >> 2) & 0x30);
  }
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }
__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + __expf(-x)); }

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

}  // namespace wmoe
