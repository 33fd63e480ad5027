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
  kStatusRange = 5,  // a value left the range of its fp16 intermediate (h or y of the grouped GEMMs)
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

// Sum of v over the CTA in a fixed order (a tree per warp, then warp 0 over the warp sums), returned to every
// thread. Every thread of the CTA must call it; red is __shared__ float[32], free again on return.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x % 32, wid = threadIdx.x / 32;
  v = warp_sum(v);
  if (lane == 0) red[wid] = v;
  __syncthreads();
  if (wid == 0) {
    float t = lane < int((blockDim.x + 31) / 32) ? red[lane] : 0.f;
    t = warp_sum(t);
    if (lane == 0) red[0] = t;
  }
  __syncthreads();
  const float r = red[0];
  __syncthreads();
  return r;
}

// Eight consecutive floats to a float32 (f32) or bfloat16 row at element offset i (16-byte aligned), bf16 rounded
// to nearest even
__device__ __forceinline__ void store8(void* dst, bool f32, size_t i, const float* v) {
  if (f32) {
    float4* o = reinterpret_cast<float4*>(static_cast<float*>(dst) + i);
    o[0] = make_float4(v[0], v[1], v[2], v[3]);
    o[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    uint32_t b[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const __nv_bfloat162 p = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
      b[j] = *reinterpret_cast<const uint32_t*>(&p);
    }
    *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(dst) + i) = make_uint4(b[0], b[1], b[2], b[3]);
  }
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


// ---- fp16 activation rows of the grouped GEMMs ----
// The GEMM operands and outputs are fp16 rows whose elements are stored in "run-of-8" order: inside every aligned
// run of 8 values, stored position perm8(e) holds element e (order 0, 2, 1, 3, 4, 6, 5, 7), the order in which the
// in-register dequantisation produces weights, so every dot product is unchanged.

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<const __half2*>(&u); }
__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<const uint32_t*>(&h); }

// Stored position of element e within its run of 8 (and back: the map is its own inverse).
__device__ __forceinline__ int perm8(int e) { return (e & ~7) | ((e & 1) << 1) | ((e & 2) >> 1) | (e & 4); }

// 8 consecutive activations as float32 from one 16-byte (bf16) or two 16-byte (f32) loads
__device__ __forceinline__ uint4 pack8_perm(const float (&v)[8]) {
  return make_uint4(pack_h2(v[0], v[2]), pack_h2(v[1], v[3]), pack_h2(v[4], v[6]), pack_h2(v[5], v[7]));
}

__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}


}  // namespace wmoe
