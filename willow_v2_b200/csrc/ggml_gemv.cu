// Typed expert kernels over ggml blocks: every type of willow's Metal path (gguf/metal.py:295: Q5_0, Q8_0, IQ4_NL,
// IQ4_XS, IQ3_XXS, IQ3_S, IQ2_S, Q2_0, Q4_K, Q6_K).
//   ggml_dequant_kernel   blocks -> f32 / bf16 / f16, bit-identical to gguf/quants.py:dequantize
//                         (gguf/metal.py:217-228 dequant_<type>, 357-363 dequantize_gpu)
//   ggml_gemv_kernel      y[pos_i * tokens + t] = W_i x_t for up to 8 tokens and n matrices
//                         (gguf/metal.py:189-215 gemv_<type>, 239-261 gemv_batch_<type>)
//   ggml_combine_kernel   y = sum_i w[perm[i]] * (W_i x_i) in order of i, with engines/base.py:431-443's bf16
//                         rounding at every step, or in float32 (gguf/metal.py:263-291 gemv_combine_<type>)
//
// A CTA owns a tile of consecutive rows of one matrix: those rows are one contiguous byte range, staged into shared
// memory by 16-byte cp.async copies (the unaligned head and tail by 16-bit copies), so HBM sees full coalesced
// sectors whatever the block size. While the copies are in flight the CTA quantises its activations into shared
// memory (int16, a power-of-two scale per 32 values, 15 bits of range). Warps then take the rows from shared memory: a row is spread
// over L lanes (L = the row's 32-value chunks, 8 to 32), each chunk becomes 8 words of int8 weights (ggml_types.cuh
// int_words) and two dp2a instructions cover 4 weights. The dequant kernel uses the float decoders instead, which
// are bit-identical to willow's. The codebooks (generated from gguf-py at build time) are copied to shared memory.
#include <algorithm>
#include <type_traits>

#include "ggml_types.cuh"

#include "ggml_tables.inc"

namespace wmoe {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kCombineThreads = 128;  // combine: 4 warps, so a [2048, 512] matrix spreads over 256 CTAs
constexpr int kGemvTileRows = 16;     // gemv: rows per CTA (8 x 1024 rows -> 512 CTAs, whatever the block size)

__device__ __forceinline__ void cp_async16(void* dst_smem, const void* src) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst_smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

// Copies bytes [src, src + len) (src 2-aligned, len even) to shared memory at dst, where dst is 16-aligned plus
// (src % 16), so the 16-byte-aligned middle of the source lands 16-byte aligned. Returns without waiting; the
// caller waits with cp_async_wait_all() and a barrier.
__device__ __forceinline__ void stage_bytes(uint8_t* dst, const uint8_t* src, size_t len) {
  const uintptr_t s = reinterpret_cast<uintptr_t>(src), e = s + len;
  const uintptr_t a = (s + 15) & ~uintptr_t(15), z = e & ~uintptr_t(15);
  if (a < z) {
    const size_t n16 = (z - a) / 16;
    for (size_t i = threadIdx.x; i < n16; i += blockDim.x)
      cp_async16(dst + (a - s) + 16 * i, reinterpret_cast<const uint8_t*>(a) + 16 * i);
    for (uintptr_t p = s + 2 * threadIdx.x; p < a; p += 2 * blockDim.x)
      *reinterpret_cast<uint16_t*>(dst + (p - s)) = *reinterpret_cast<const uint16_t*>(p);
    for (uintptr_t p = z + 2 * threadIdx.x; p < e; p += 2 * blockDim.x)
      *reinterpret_cast<uint16_t*>(dst + (p - s)) = *reinterpret_cast<const uint16_t*>(p);
  } else {
    for (uintptr_t p = s + 2 * threadIdx.x; p < e; p += 2 * blockDim.x)
      *reinterpret_cast<uint16_t*>(dst + (p - s)) = *reinterpret_cast<const uint16_t*>(p);
  }
}

// The type's codebook into shared memory at tab (16-byte aligned); returns the table view.
template <int T>
__device__ __forceinline__ GgmlTables load_tables(uint8_t* tab) {
  GgmlTables tb{nullptr, nullptr, nullptr};
  if constexpr (T == kGgmlIQ4NL || T == kGgmlIQ4XS) {
    float* lv = reinterpret_cast<float*>(tab);
    if (threadIdx.x < 16) lv[threadIdx.x] = float(kIq4nlLevels[threadIdx.x]);
    tb.levels = lv;
  } else if constexpr (T == kGgmlIQ3XXS || T == kGgmlIQ3S) {
    constexpr int n = T == kGgmlIQ3XXS ? 256 : 512;
    const uint32_t* src = T == kGgmlIQ3XXS ? kIq3xxsGrid : kIq3sGrid;
    uint32_t* g = reinterpret_cast<uint32_t*>(tab);
    for (int i = threadIdx.x; i < n; i += blockDim.x) g[i] = src[i];
    tb.grid32 = g;
  } else if constexpr (T == kGgmlIQ2S) {
    uint2* g = reinterpret_cast<uint2*>(tab);
    for (int i = threadIdx.x; i < 1024; i += blockDim.x)
      g[i] = make_uint2(uint32_t(kIq2sGrid[i]), uint32_t(kIq2sGrid[i] >> 32));
    tb.grid64 = g;
  }
  return tb;
}

// The integer kernels' tables: IQ4 levels as int8 bytes, the grids as for the float decoders.
template <int T>
__device__ __forceinline__ void stage_int_tables(uint8_t* tab) {
  if constexpr (T == kGgmlIQ4NL || T == kGgmlIQ4XS) {
    if (threadIdx.x < 16) tab[threadIdx.x] = uint8_t(kIq4nlLevels[threadIdx.x]);
  } else {
    load_tables<T>(tab);
  }
}

template <int T>
__device__ __forceinline__ IntTables int_tables(const uint8_t* tab) {  // after the barrier that follows staging
  IntTables it{0, 0, 0, 0, nullptr, nullptr};
  if constexpr (T == kGgmlIQ4NL || T == kGgmlIQ4XS) {
    const uint32_t* lv = reinterpret_cast<const uint32_t*>(tab);
    it.lv0 = lv[0];
    it.lv1 = lv[1];
    it.lv2 = lv[2];
    it.lv3 = lv[3];
  } else if constexpr (T == kGgmlIQ3XXS || T == kGgmlIQ3S) {
    it.grid32 = reinterpret_cast<const uint32_t*>(tab);
  } else if constexpr (T == kGgmlIQ2S) {
    it.grid64 = reinterpret_cast<const uint2*>(tab);
  }
  return it;
}

// Activations in shared memory: n rows of k values as int16 with one power-of-two scale per 32 values and the sums
// of the int16 values per 16. A chunk's 64 bytes are stored as 4 quarters of 16 bytes, quarter-major
// ([n][4][chunks] of 16 bytes), so the lanes of a warp, which read consecutive chunks, read consecutive 16-byte
// words (no bank conflicts). Region sizes, each rounded up to 16 bytes.
struct XQ {
  uint4* q;      // [n][4][k / 32]
  float* scale;  // [n, k / 32]
  int* sum16;    // [n, k / 16]
};

__host__ __device__ constexpr size_t align16(size_t v) { return (v + 15) & ~size_t(15); }
__host__ __device__ constexpr size_t xq_bytes(int n, int k) {
  return align16(size_t(n) * k * 2) + align16(size_t(n) * (k / 32) * 4) + align16(size_t(n) * (k / 16) * 4);
}
// the combine's per-matrix addresses and routing weights, and a flag
__host__ __device__ constexpr size_t combine_meta_bytes(int n) { return align16(size_t(n) * 12 + 4); }

__device__ __forceinline__ XQ xq_view(uint8_t* p, int n, int k) {
  XQ v;
  v.q = reinterpret_cast<uint4*>(p);
  v.scale = reinterpret_cast<float*>(p + align16(size_t(n) * k * 2));
  v.sum16 = reinterpret_cast<int*>(p + align16(size_t(n) * k * 2) + align16(size_t(n) * (k / 32) * 4));
  return v;
}

// Quantises x [n, k] (f32 or bf16, global) into xq: 8 lanes per 32-value block, 4 values per lane. The scale of a
// block is 2^(E - 15) for its largest magnitude m = f * 2^E (f in [0.5, 1)), so |q| <= 32767 (the one value that
// rounds to 2^15 is clamped) and every value within 2^7 of m that a bf16 can hold is exact; blocks with m below
// 2^-107 are zero. With int8 weights a chunk's dp2a sum stays below 32 * 32767 * 127 < 2^31.
// willow's expert_gate (engines/base.py:99-102) on one bf16 gate / up pair, as torch computes it on bf16 tensors:
// silu(g) = g / (1 + exp(-g)) in float rounded to bf16, then that times u in float rounded to bf16.
__device__ __forceinline__ float expert_gate_bf16(float g, float u) {
  const float s = __bfloat162float(__float2bfloat16_rn(g / (1.f + expf(-g))));
  return __bfloat162float(__float2bfloat16_rn(s * u));
}

// x_dtype kGated: x is bf16 gate_up rows [n][2k] and row r's input is expert_gate(gate, up) of them
constexpr int kGated = -1;

__device__ __forceinline__ void quantize_x(const void* x, int x_dtype, int n, int k, XQ xq) {
  const int nblk = n * (k / 32);
  const int sub = threadIdx.x % 8, group = threadIdx.x / 8, groups = blockDim.x / 8;
  for (int b0 = 0; b0 < nblk; b0 += groups) {  // the bound is uniform across each warp: shuffles stay converged
    const int b = b0 + group;
    const bool on = b < nblk;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (on) {
      const size_t at = size_t(b) * 32 + 4 * sub;
      if (x_dtype == kF32) {
        const float4 f = *reinterpret_cast<const float4*>(static_cast<const float*>(x) + at);
        v[0] = f.x, v[1] = f.y, v[2] = f.z, v[3] = f.w;
      } else if (x_dtype == kGated) {
        const size_t r = at / size_t(k), j = at % size_t(k);
        const __nv_bfloat16* gp = static_cast<const __nv_bfloat16*>(x) + r * 2 * k + j;
        const uint2 g = *reinterpret_cast<const uint2*>(gp), u = *reinterpret_cast<const uint2*>(gp + k);
        v[0] = expert_gate_bf16(__uint_as_float(g.x << 16), __uint_as_float(u.x << 16));
        v[1] = expert_gate_bf16(__uint_as_float(g.x & 0xFFFF0000u), __uint_as_float(u.x & 0xFFFF0000u));
        v[2] = expert_gate_bf16(__uint_as_float(g.y << 16), __uint_as_float(u.y << 16));
        v[3] = expert_gate_bf16(__uint_as_float(g.y & 0xFFFF0000u), __uint_as_float(u.y & 0xFFFF0000u));
      } else {
        const uint2 h = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(x) + at);
        v[0] = __uint_as_float(h.x << 16), v[1] = __uint_as_float(h.x & 0xFFFF0000u);
        v[2] = __uint_as_float(h.y << 16), v[3] = __uint_as_float(h.y & 0xFFFF0000u);
      }
    }
    float m = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
    const int eb = int(__float_as_uint(m) >> 23);  // biased exponent; m = 1.f * 2^(eb - 127)
    const bool zero = eb < 20;
    const float inv = zero ? 0.f : __uint_as_float(uint32_t(268 - eb) << 23);  // 2^(141 - eb)
    int q[4], sum = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      q[i] = max(-32767, min(32767, __float2int_rn(v[i] * inv)));
      sum += q[i];
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    if (on) {
      const uint2 packed = make_uint2((uint32_t(q[0]) & 0xFFFFu) | (uint32_t(q[1]) << 16),
                                      (uint32_t(q[2]) & 0xFFFFu) | (uint32_t(q[3]) << 16));
      const int chunks = k / 32, r = b / chunks, c = b % chunks;
      reinterpret_cast<uint2*>(xq.q + (size_t(r) * 4 + sub / 2) * chunks + c)[sub % 2] = packed;
      if (sub == 0) xq.scale[b] = zero ? 0.f : __uint_as_float(uint32_t(eb - 14) << 23);  // 2^(eb - 141)
      if (sub % 4 == 0) xq.sum16[2 * b + sub / 4] = sum;
    }
  }
}

// the 32 int16 activations of chunk c of row r, their scale and half sums
__device__ __forceinline__ float chunk_x(const XQ& xq, int k, int r, int c, uint32_t (&xw)[16], int& s0, int& s1) {
  const int chunks = k / 32;
  const uint4* p = xq.q + size_t(r) * 4 * chunks + c;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint4 u = p[i * chunks];
    xw[4 * i] = u.x, xw[4 * i + 1] = u.y, xw[4 * i + 2] = u.z, xw[4 * i + 3] = u.w;
  }
  const int blk = r * (k / 32) + c;
  s0 = xq.sum16[2 * blk];
  s1 = xq.sum16[2 * blk + 1];
  return xq.scale[blk];
}

template <typename OutT>
__device__ __forceinline__ OutT to_out(float v);
template <>
__device__ __forceinline__ float to_out<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 to_out<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half to_out<__half>(float v) { return __float2half_rn(v); }

__device__ __forceinline__ float round_bf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// sum over the L lanes of a row group (L a power of two, groups aligned to L)
template <int L>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = L / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ------------------------------------------------------------------------------------------------ dequant

template <int T, typename OutT>
__global__ void __launch_bounds__(kThreads) ggml_dequant_kernel(const uint8_t* __restrict__ blocks, size_t nblocks,
                                                                OutT* __restrict__ out) {
  __shared__ __align__(16) uint8_t tab[table_bytes(T) > 0 ? table_bytes(T) : 16];
  const GgmlTables tb = load_tables<T>(tab);
  __syncthreads();
  constexpr BlockGeom g = block_geom(T);
  constexpr int per = g.elements / 32;
  const size_t chunk = blockIdx.x * size_t(blockDim.x) + threadIdx.x;
  if (chunk >= nblocks * per) return;
  float v[32];
  decode_chunk<T>(blocks + (chunk / per) * g.bytes, int(chunk % per), tb, v);
  OutT* o = out + chunk * 32;
#pragma unroll
  for (int l = 0; l < 32; ++l) o[l] = to_out<OutT>(v[l]);
}

// ------------------------------------------------------------------------------------------------ gemv

struct GemvArgs {
  const uint8_t* const* weights;  // n device pointers to [rows, k] matrices, or null: the one matrix `single`
  const uint8_t* single;
  const int64_t* positions;       // nullable: output slot of matrix i (default i); checked against n_out
  int n, n_out, rows, k, tokens, tile_rows;
  size_t row_bytes;
  const void* x;  // [tokens, k]
  int x_dtype;
  void* y;        // [n_out * tokens, rows]
  int y_dtype;
  int* status;
};

// L lanes per row, MAXT token accumulators. Shared memory: the type's table, the quantised activations, then the
// staged rows of the tile.
template <int T, int L, int MAXT>
__global__ void __launch_bounds__(kThreads) ggml_gemv_kernel(GemvArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint8_t* tab = smem;
  const XQ xq = xq_view(smem + align16(table_bytes(T)), a.tokens, a.k);
  uint8_t* stage = smem + align16(table_bytes(T)) + xq_bytes(a.tokens, a.k);
  const int i = blockIdx.y, r0 = blockIdx.x * a.tile_rows;
  const int nr = min(a.tile_rows, a.rows - r0);
  const uint8_t* mat = a.weights ? a.weights[i] : a.single;
  const int64_t pos64 = a.positions ? a.positions[i] : i;
  // an output slot out of range or an odd matrix address: flag it and touch nothing (uniform over the CTA)
  if (pos64 < 0 || pos64 >= a.n_out || (reinterpret_cast<uintptr_t>(mat) & 1)) {
    if (threadIdx.x == 0) atomicCAS(a.status, kStatusOk, kStatusBadExpert);
    return;
  }
  const int pos = int(pos64);
  const uint8_t* src = mat + size_t(r0) * a.row_bytes;
  uint8_t* base = stage + (reinterpret_cast<uintptr_t>(src) & 15);
  stage_bytes(base, src, size_t(nr) * a.row_bytes);  // in flight while x is quantised
  stage_int_tables<T>(tab);
  quantize_x(a.x, a.x_dtype, a.tokens, a.k, xq);
  cp_async_wait_all();
  __syncthreads();
  const IntTables it = int_tables<T>(tab);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  constexpr int kRowsPerWarp = 32 / L;
  const int chunks = a.k / 32;
  for (int rr = warp * kRowsPerWarp + lane / L; rr - lane / L < nr; rr += kWarps * kRowsPerWarp) {
    const bool valid = rr < nr;
    const uint8_t* row = base + size_t(valid ? rr : 0) * a.row_bytes;
    float acc[MAXT];
#pragma unroll
    for (int t = 0; t < MAXT; ++t) acc[t] = 0.f;
    if (valid) {
      for (int c = lane % L; c < chunks; c += L) {
        uint32_t w[8];
        ChunkScale cs;
        int_row_words<T>(row, c, it, w, cs);
#pragma unroll
        for (int t = 0; t < MAXT; ++t) {
          if (t < a.tokens) {
            uint32_t xw[16];
            int s0, s1;
            const float xs = chunk_x(xq, a.k, t, c, xw, s0, s1);
            acc[t] += chunk_apply(w, cs, xw, xs, s0, s1);
          }
        }
      }
    }
#pragma unroll
    for (int t = 0; t < MAXT; ++t) {
      if (t >= a.tokens) break;
      const float s = group_sum<L>(acc[t]);
      if (valid && lane % L == 0) {
        const size_t o = (size_t(pos) * a.tokens + t) * a.rows + r0 + rr;
        if (a.y_dtype == kF32)
          static_cast<float*>(a.y)[o] = s;
        else
          static_cast<__nv_bfloat16*>(a.y)[o] = __float2bfloat16_rn(s);
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------ combine

struct CombineArgs {
  const uint8_t* const* weights;  // n device pointers to [rows, k] matrices
  const int64_t* perm;            // [n]: index of matrix i's routing weight in route_w (checked against n_route)
  int n, n_route, rows, k, tile_rows, group;  // group: matrices staged at once
  size_t row_bytes;
  const void* x;        // [n, k]: matrix i's input row (gated: bf16 [n, 2k] gate_up rows, see kGated)
  const void* route_w;  // [n_route]
  int dtype;            // kBF16: bf16 x, weights, y and rounding at each step; kF32: all float32
  int gated;            // x holds gate_up rows and the input is willow's expert_gate of them (kBF16 only)
  void* y;              // [rows]
  int* status;
};

// One CTA (kCombineThreads) per tile of rows_per_pass rows (each group of L lanes owns one row), all matrices of a
// group staged at once, then summed in order. Shared memory: table, the n quantised input rows, the stage.
template <int T, int L>
__global__ void __launch_bounds__(kCombineThreads) ggml_combine_kernel(CombineArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint8_t* tab = smem;
  const XQ xq = xq_view(smem + align16(table_bytes(T)), a.n, a.k);
  // the matrices' addresses, routing weights and a bad-entry flag, read from global memory once, in parallel
  const uint8_t** mats = reinterpret_cast<const uint8_t**>(smem + align16(table_bytes(T)) + xq_bytes(a.n, a.k));
  float* rws = reinterpret_cast<float*>(mats + a.n);
  int* bad = reinterpret_cast<int*>(rws + a.n);
  uint8_t* stage = smem + align16(table_bytes(T)) + xq_bytes(a.n, a.k) + combine_meta_bytes(a.n);
  const int r0 = blockIdx.x * a.tile_rows, nr = min(a.tile_rows, a.rows - r0);
  const size_t tile_bytes = size_t(nr) * a.row_bytes;
  const size_t slot = align16(size_t(a.tile_rows) * a.row_bytes) + 16;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int rr = warp * (32 / L) + lane / L;  // this lane group's row of the tile
  const bool valid = rr < nr;
  const int chunks = a.k / 32;
  if (threadIdx.x == 0) *bad = 0;
  __syncthreads();
  for (int e = threadIdx.x; e < a.n; e += blockDim.x) {
    const int64_t pe = a.perm[e];
    const uint8_t* w = a.weights[e];
    mats[e] = w;
    if (pe < 0 || pe >= a.n_route || (reinterpret_cast<uintptr_t>(w) & 1)) {
      *bad = 1;
      rws[e] = 0.f;
    } else {
      rws[e] = a.dtype == kF32 ? static_cast<const float*>(a.route_w)[pe]
                               : __bfloat162float(static_cast<const __nv_bfloat16*>(a.route_w)[pe]);
    }
  }
  __syncthreads();
  // a routing index out of range or an odd matrix address: flag it and touch nothing (uniform over the CTA)
  if (*bad) {
    if (threadIdx.x == 0) atomicCAS(a.status, kStatusOk, kStatusBadExpert);
    return;
  }
  stage_int_tables<T>(tab);
  float total = 0.f;
  for (int g0 = 0; g0 < a.n; g0 += a.group) {
    const int gn = min(a.group, a.n - g0);
    __syncthreads();  // the previous group's reads of the stage are done
    for (int m = 0; m < gn; ++m) {
      const uint8_t* src = mats[g0 + m] + size_t(r0) * a.row_bytes;
      stage_bytes(stage + m * slot + (reinterpret_cast<uintptr_t>(src) & 15), src, tile_bytes);
    }
    if (g0 == 0) quantize_x(a.x, a.gated ? kGated : a.dtype, a.n, a.k, xq);  // while the first copies fly
    cp_async_wait_all();
    __syncthreads();
    const IntTables it = int_tables<T>(tab);
    for (int m = 0; m < gn; ++m) {
      const int e = g0 + m;
      const float rw = rws[e];
      const uint8_t* src = mats[e] + size_t(r0) * a.row_bytes;
      const uint8_t* row = stage + m * slot + (reinterpret_cast<uintptr_t>(src) & 15) +
                           size_t(valid ? rr : 0) * a.row_bytes;
      float acc = 0.f;
      if (valid) {
        for (int c = lane % L; c < chunks; c += L) {
          uint32_t w[8], xw[16];
          ChunkScale cs;
          int s0, s1;
          int_row_words<T>(row, c, it, w, cs);
          const float xs = chunk_x(xq, a.k, e, c, xw, s0, s1);
          acc += chunk_apply(w, cs, xw, xs, s0, s1);
        }
      }
      const float p = group_sum<L>(acc);
      if (a.dtype == kF32) {
        total = e == 0 ? __fmul_rn(rw, p) : fmaf(rw, p, total);
      } else {
        const float scaled = round_bf16(__fmul_rn(round_bf16(p), rw));
        total = e == 0 ? scaled : round_bf16(__fadd_rn(total, scaled));
      }
    }
  }
  if (valid && lane % L == 0) {
    if (a.dtype == kF32)
      static_cast<float*>(a.y)[r0 + rr] = total;
    else
      static_cast<__nv_bfloat16*>(a.y)[r0 + rr] = __float2bfloat16_rn(total);
  }
}

// ------------------------------------------------------------------------------------------------ launch

template <typename F>
cudaError_t by_type(int type, F&& f) {
  switch (type) {
    case kGgmlQ5_0: return f(std::integral_constant<int, kGgmlQ5_0>{});
    case kGgmlQ8_0: return f(std::integral_constant<int, kGgmlQ8_0>{});
    case kGgmlIQ4NL: return f(std::integral_constant<int, kGgmlIQ4NL>{});
    case kGgmlIQ4XS: return f(std::integral_constant<int, kGgmlIQ4XS>{});
    case kGgmlIQ3XXS: return f(std::integral_constant<int, kGgmlIQ3XXS>{});
    case kGgmlIQ3S: return f(std::integral_constant<int, kGgmlIQ3S>{});
    case kGgmlIQ2S: return f(std::integral_constant<int, kGgmlIQ2S>{});
    case kGgmlQ2_0: return f(std::integral_constant<int, kGgmlQ2_0>{});
    case kGgmlQ4K: return f(std::integral_constant<int, kGgmlQ4K>{});
    case kGgmlQ6K: return f(std::integral_constant<int, kGgmlQ6K>{});
    default: return cudaErrorInvalidValue;
  }
}

// lanes per row: the row's chunk count rounded down to a power of two, between 8 and 32 (rows of fewer than 8
// chunks leave lanes idle)
int lanes_for(int chunks) {
  int l = 8;
  while (l * 2 <= chunks && l < 32) l *= 2;
  return l;
}

template <typename F>
cudaError_t by_lanes(int lanes, F&& f) {
  switch (lanes) {
    case 32: return f(std::integral_constant<int, 32>{});
    case 16: return f(std::integral_constant<int, 16>{});
    default: return f(std::integral_constant<int, 8>{});
  }
}

constexpr size_t kStageBudget = 32 * 1024;  // staged weight bytes per CTA of the gemv kernel
constexpr size_t kMaxSmem = 200 * 1024;

// Raises a kernel's dynamic shared-memory limit to kMaxSmem once per device (the launch's own size decides what it
// gets).
template <auto Kernel>
cudaError_t allow_max_smem() {
  static std::atomic<uint64_t> done{0};
  return once_per_device(done, []() {
    return cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kMaxSmem));
  });
}

}  // namespace

size_t ggml_row_bytes(int type, int k) {
  const BlockGeom g = block_geom(type);
  if (g.elements == 0 || k <= 0 || k % g.elements) return 0;
  return size_t(k / g.elements) * g.bytes;
}

cudaError_t ggml_dequant(int type, const uint8_t* blocks, size_t nblocks, void* out, int out_dtype,
                         cudaStream_t st) {
  if (nblocks == 0) return cudaSuccess;
  return by_type(type, [&](auto tc) -> cudaError_t {
    constexpr int T = decltype(tc)::value;
    const size_t chunks = nblocks * (block_geom(T).elements / 32);
    const unsigned grid = unsigned((chunks + kThreads - 1) / kThreads);
    if (out_dtype == kF32)
      ggml_dequant_kernel<T, float><<<grid, kThreads, 0, st>>>(blocks, nblocks, static_cast<float*>(out));
    else if (out_dtype == kBF16)
      ggml_dequant_kernel<T, __nv_bfloat16><<<grid, kThreads, 0, st>>>(blocks, nblocks,
                                                                        static_cast<__nv_bfloat16*>(out));
    else
      ggml_dequant_kernel<T, __half><<<grid, kThreads, 0, st>>>(blocks, nblocks, static_cast<__half*>(out));
    return cudaGetLastError();
  });
}

// The refusal of a call whose activations and row tile do not fit shared memory: a code no launch or attribute
// call of these launchers returns, so that the C ABI can tell it apart (WMOE_ERR_UNSUPPORTED).
constexpr cudaError_t kSmemRefusal = cudaErrorNotSupported;

cudaError_t ggml_gemv(int type, const uint8_t* const* weights, const uint8_t* single, const int64_t* positions, int n,
                      int n_out, int rows, int k, const void* x, int x_dtype, int tokens, void* y, int y_dtype,
                      int* status, cudaStream_t st) {
  const size_t rb = ggml_row_bytes(type, k);
  if (rb == 0 || k % 32 || tokens < 1 || tokens > 8) return cudaErrorInvalidValue;
  if (n == 0 || rows == 0) return cudaSuccess;
  GemvArgs a{weights, single, positions, n, n_out, rows, k, tokens, 0, rb, x, x_dtype, y, y_dtype, status};
  a.tile_rows = int(std::max<size_t>(1, std::min<size_t>(std::min<size_t>(size_t(rows), kGemvTileRows),
                                                         kStageBudget / rb)));
  const size_t smem = align16(table_bytes(type)) + xq_bytes(tokens, k) + size_t(a.tile_rows) * rb + 16;
  if (smem > kMaxSmem) return kSmemRefusal;
  (void)cudaGetLastError();  // an earlier call's non-sticky error must not read as this launch's
  const dim3 grid(unsigned((rows + a.tile_rows - 1) / a.tile_rows), unsigned(n));
  const int lanes = lanes_for(k / 32);
  return by_type(type, [&](auto tc) -> cudaError_t {
    constexpr int T = decltype(tc)::value;
    return by_lanes(lanes, [&](auto lc) -> cudaError_t {
      constexpr int L = decltype(lc)::value;
      if (tokens == 1) {
        if (cudaError_t e = allow_max_smem<ggml_gemv_kernel<T, L, 1>>()) return e;
        ggml_gemv_kernel<T, L, 1><<<grid, kThreads, smem, st>>>(a);
      } else {
        if (cudaError_t e = allow_max_smem<ggml_gemv_kernel<T, L, 8>>()) return e;
        ggml_gemv_kernel<T, L, 8><<<grid, kThreads, smem, st>>>(a);
      }
      return cudaGetLastError();
    });
  });
}

cudaError_t ggml_combine(int type, const uint8_t* const* weights, const int64_t* perm, int n, int n_route, int rows,
                         int k, const void* x, const void* route_w, int dtype, void* y, int* status,
                         cudaStream_t st, bool gated) {
  const size_t rb = ggml_row_bytes(type, k);
  if (rb == 0 || k % 32 || n < 1 || (gated && dtype != kBF16)) return cudaErrorInvalidValue;
  if (rows == 0) return cudaSuccess;
  const int lanes = lanes_for(k / 32);
  const int rows_per_pass = kCombineThreads / 32 * (32 / lanes);  // one row per lane group: the tile is one pass
  CombineArgs a{weights, perm, n, n_route, rows, k, 0, 0, rb, x, route_w, dtype, gated ? 1 : 0, y, status};
  a.tile_rows = std::min(rows, rows_per_pass);
  const size_t slot = align16(size_t(a.tile_rows) * rb) + 16;
  const size_t tab = align16(table_bytes(type)) + xq_bytes(n, k) + combine_meta_bytes(n);
  if (tab + slot > kMaxSmem) return kSmemRefusal;
  (void)cudaGetLastError();  // an earlier call's non-sticky error must not read as this launch's
  a.group = int(std::min<size_t>(size_t(n), (kMaxSmem - tab) / slot));
  a.group = std::min(a.group, int(std::max<size_t>(1, (96 * 1024) / slot)));  // keep a few CTAs per SM
  const size_t smem = tab + size_t(a.group) * slot;
  const dim3 grid(unsigned((rows + a.tile_rows - 1) / a.tile_rows));
  return by_type(type, [&](auto tc) -> cudaError_t {
    constexpr int T = decltype(tc)::value;
    return by_lanes(lanes, [&](auto lc) -> cudaError_t {
      constexpr int L = decltype(lc)::value;
      if (cudaError_t e = allow_max_smem<ggml_combine_kernel<T, L>>()) return e;
      ggml_combine_kernel<T, L><<<grid, kCombineThreads, smem, st>>>(a);
      return cudaGetLastError();
    });
  });
}

// willow's expert_gate on bf16 [n][2F] gate_up rows (expert_gate_bf16 per element)
__global__ void __launch_bounds__(256) swiglu_bf16_kernel(const __nv_bfloat16* __restrict__ gu, int n, int F,
                                                          __nv_bfloat16* __restrict__ out) {
  const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= size_t(n) * F) return;
  const size_t e = i / size_t(F), j = i % size_t(F);
  out[i] = __float2bfloat16_rn(expert_gate_bf16(__bfloat162float(gu[e * 2 * F + j]),
                                                __bfloat162float(gu[e * 2 * F + F + j])));
}

cudaError_t swiglu_bf16(const void* gate_up, int n, int F, void* out, cudaStream_t st) {
  const size_t total = size_t(n) * F;
  if (total == 0) return cudaSuccess;
  swiglu_bf16_kernel<<<unsigned((total + 255) / 256), 256, 0, st>>>(static_cast<const __nv_bfloat16*>(gate_up), n, F,
                                                                   static_cast<__nv_bfloat16*>(out));
  return cudaGetLastError();
}

}  // namespace wmoe
