// Grouped expert GEMMs for many tokens per expert (prefill), on the 5th-generation tensor cores (tcgen05 + TMEM).
// Replaces willow's dequantize-to-bf16 + matmul path for more than 8 tokens (gguf/metal.py:357-363, 404-407) and
// the per-expert loop of Engine.each_expert (engines/base.py:534-591).
//
// Swap-AB: the expert's weight rows are the MMA's M (128 per tile), its tokens are N (128 per tile), K runs over the
// hidden size (gate_up) or the FFN width (down) in blocks of 64.
//   A  128 x 64 weight tile: 4 warps dequantise it from the raw Q4_K / Q6_K bytes in global memory (one row per
//      thread: 48 or 100 bytes) to fp16 and store it in shared memory in the 128-byte-swizzled K-major layout the
//      MMA reads. Values are the exact float32 dequantisation of willow (gguf/quants.py:87-116) rounded to fp16.
//   B  128 tokens x 64 activations (fp16): one TMA tile load (128-byte swizzle) from the gathered activations.
//   D  128 x 128 float32 accumulator in TMEM (128 columns), 4 tcgen05.mma (K = 16 each) per K block, issued by one
//      thread; tcgen05.commit signals an mbarrier when they have read shared memory and finished.
// gate_up tiles pair 64 gate rows with the 64 matching up rows (rows j and F + j), so the SwiGLU epilogue has both:
// h = silu(gate) * up, stored as fp16 scaled by 1/32 (fp16 has the precision the 2e-3 bound needs - bf16 does
// not - but not the range of raw h). down tiles write y / 32 as fp16; the combine multiplies the 32 back.
// Waits are bounded (1 s of %globaltimer); on a timeout the CTA records the device status, waits (bounded) for its
// outstanding MMAs, frees its TMEM and returns.
#include <cuda.h>

#include "common.cuh"
#include "kernels.cuh"

namespace wmoe {

namespace {

constexpr int kBM = 128, kBN = 128, kBK = 64;
constexpr int kThreads = 128;
constexpr int kTileBytes = kBM * kBK * 2;  // 16 KB per operand tile (fp16)
constexpr unsigned long long kTimeoutNs = 1000000000ull;

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ bool mbar_wait(uint64_t* bar, unsigned parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer() - t0 > kTimeoutNs) return false;
  return true;
}

// 2-D TMA tile load (box 64 fp16 x 128 rows, 128-byte swizzle) completing on an mbarrier; x = column, y = row.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 bytes apart (sm100 version 1).
__device__ __forceinline__ uint64_t smem_desc(const void* p) {
  const uint64_t addr = smem_u32(p);
  return ((addr >> 4) & 0x3FFFull)        // start address
         | (1ull << 16)                   // leading byte offset (unused for swizzled K-major): 16 B
         | (uint64_t(1024 >> 4) << 32)    // stride byte offset: 1024 B between 8-row groups
         | (1ull << 46)                   // descriptor version
         | (2ull << 61);                  // SWIZZLE_128B
}

// Instruction descriptor of kind::f16: fp16 A and B, fp32 accumulator, both K-major, M = 128, N = kBN.
constexpr uint32_t kIdesc = (1u << 4) | (0u << 7) | (0u << 10) | (uint32_t(kBN >> 3) << 17) | (uint32_t(kBM >> 4) << 24);

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 consecutive TMEM columns of this thread's lane (the warp's 32 lanes)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Byte offset of (row, 16-byte chunk c of the row's 128 bytes) in a 128-byte-swizzled K-major tile.
__device__ __forceinline__ int sw128(int row, int c) { return (row >> 3) * 1024 + (row & 7) * 128 + ((c ^ (row & 7)) << 4); }

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// One Q4_K row's K block kb (elements 64 kb .. 64 kb + 63 = sub-blocks 2g, 2g + 1 of super-block kb / 4, g = kb % 4)
// -> 64 fp16 into the row of the swizzled tile.
__device__ __forceinline__ void dequant_q4k_row(const uint8_t* row, int kb, uint8_t* tile, int r) {
  const uint8_t* b = row + (kb / 4) * Q4K_BYTES;
  const int g = kb % 4;
  const uint4 hd = ldg_nc_v4(b);
  const uint4 qa = ldg_nc_v4(b + 16 + 32 * g), qb = ldg_nc_v4(b + 32 + 32 * g);
  const float d = f16_to_f32(uint16_t(hd.x & 0xFFFF)), dmin = f16_to_f32(uint16_t(hd.x >> 16));
  int sc0, mn0, sc1, mn1;
  q4k_scale_min_w(hd.y, hd.z, hd.w, 2 * g, sc0, mn0);
  q4k_scale_min_w(hd.y, hd.z, hd.w, 2 * g + 1, sc1, mn1);
  const float A0 = __fmul_rn(d, float(sc0)), B0 = __fmul_rn(dmin, float(mn0));
  const float A1 = __fmul_rn(d, float(sc1)), B1 = __fmul_rn(dmin, float(mn1));
  const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
  // chunks 0..3: sub-block 2g (low nibbles of bytes 0..31), chunks 4..7: sub-block 2g + 1 (high nibbles)
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const float A = half ? A1 : A0, B = half ? B1 : B0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t o[4];
#pragma unroll
      for (int w = 0; w < 2; ++w) {
        const uint32_t word = qw[2 * c + w] >> (4 * half);
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = __fsub_rn(__fmul_rn(A, float((word >> (8 * i)) & 0xF)), B);
        o[2 * w] = pack_h2(v[0], v[1]);
        o[2 * w + 1] = pack_h2(v[2], v[3]);
      }
      *reinterpret_cast<uint4*>(tile + sw128(r, 4 * half + c)) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// One Q6_K row's K block kb (64 elements of super-block kb / 4: half hh = (kb % 4) / 2, quarters 2q and 2q + 1,
// q = kb % 2) -> 64 fp16. Element e: ql byte hh*64 + e (nibble q), qh byte 128 + hh*32 + e % 32 (bits 4q + 2(e/32)),
// scale index hh*8 + 4q + e / 16.
__device__ __forceinline__ void dequant_q6k_row(const uint8_t* row, int kb, uint8_t* tile, int r) {
  const uint8_t* b = row + (kb / 4) * Q6K_BYTES;
  const int hh = (kb % 4) / 2, q = kb % 2;
  uint32_t ql[16], qh[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint4 v = ldg_u2_16(b + hh * 64 + 16 * i);
    ql[4 * i] = v.x, ql[4 * i + 1] = v.y, ql[4 * i + 2] = v.z, ql[4 * i + 3] = v.w;
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint4 v = ldg_u2_16(b + 128 + hh * 32 + 16 * i);
    qh[4 * i] = v.x, qh[4 * i + 1] = v.y, qh[4 * i + 2] = v.z, qh[4 * i + 3] = v.w;
  }
  const uint4 scw = ldg_u2_16(b + 192);
  const uint32_t sw[4] = {scw.x, scw.y, scw.z, scw.w};
  const float d = f16_to_f32(__ldg(reinterpret_cast<const unsigned short*>(b + 208)));
  float D[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int si = hh * 8 + 4 * q + i;
    D[i] = __fmul_rn(d, float(int8_t((sw[si / 4] >> (8 * (si % 4))) & 0xFF)));
  }
#pragma unroll
  for (int c = 0; c < 8; ++c) {  // chunk c: elements 8c .. 8c + 7
    uint32_t o[4];
#pragma unroll
    for (int w = 0; w < 2; ++w) {
      const int e0 = 8 * c + 4 * w;  // 4 elements e0..e0+3, one ql word and one qh word
      const uint32_t lw = (ql[e0 / 4] >> (4 * q)) & 0x0F0F0F0Fu;
      const uint32_t hw = (qh[(e0 % 32) / 4] >> (4 * q + 2 * (e0 / 32))) & 0x03030303u;
      const uint32_t q6 = lw | (hw << 4);
      float v[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = __fmul_rn(D[e0 / 16], float(int((q6 >> (8 * i)) & 0xFF) - 32));
      o[2 * w] = pack_h2(v[0], v[1]);
      o[2 * w + 1] = pack_h2(v[2], v[3]);
    }
    *reinterpret_cast<uint4*>(tile + sw128(r, c)) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

struct GemmParams {
  ExpertSource src;
  int layer;
  PairMap pm;
  const int2* items;     // (segment u, first token of the tile within the segment)
  const int* n_items;
  int mode;              // 0: gate_up + SwiGLU -> h, 1: down -> y
  int F, H;
  __half* out;           // mode 0: h [P][F]; mode 1: y [P][H]
  int* status;
};

__global__ void __launch_bounds__(kThreads) grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmap_b,
                                                                const __grid_constant__ GemmParams p) {
  extern __shared__ __align__(1024) uint8_t dyn[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn) + 1023) & ~uintptr_t(1023));
  uint8_t* tileA = base;
  uint8_t* tileB = base + kTileBytes;
  __shared__ uint64_t mbar_b, mbar_mma;
  __shared__ uint32_t tmem_base;
  __shared__ int fail;

  const int item = blockIdx.y;
  if (item >= *p.n_items) return;
  const int2 it = p.items[item];
  const int u = it.x, n0 = it.y;
  const int e = p.pm.used[u];
  const int seg0 = p.pm.seg[u], cnt = p.pm.seg[u + 1] - seg0;
  const int n_valid = min(kBN, cnt - n0);
  const int mt = blockIdx.x;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int K = p.mode == 0 ? p.H : p.F;

  // the expert's weights
  const uint8_t* w;
  if (e == p.src.experts) {
    w = p.mode == 0 ? p.src.shared_gate_up : p.src.shared_down;
  } else {
    const int s = p.src.slot_of[size_t(p.layer) * p.src.experts + e];
    if (s < 0) {
      if (tid == 0) set_status(p.status, kStatusNotResident);
      return;
    }
    w = p.src.slab + size_t(s) * p.src.slot_bytes + (p.mode == 0 ? 0 : p.src.gate_up_bytes);
  }
  const size_t row_bytes = p.mode == 0 ? size_t(K / QK) * Q4K_BYTES : size_t(K / QK) * Q6K_BYTES;
  // weight row of this thread's tile row
  int wrow;
  if (p.mode == 0)
    wrow = tid < 64 ? 64 * mt + tid : p.F + 64 * mt + (tid - 64);
  else
    wrow = kBM * mt + tid;
  const uint8_t* my_row = w + size_t(wrow) * row_bytes;

  if (tid == 0) {
    fail = 0;
    mbar_init(&mbar_b, 1);
    mbar_init(&mbar_mma, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(kBN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem_d = tmem_base;

  const int nk = K / kBK;
  int issued = 0;  // MMA groups committed
  for (int kb = 0; kb < nk; ++kb) {
    // B: this tile's tokens x activations kb*64 .. +63
    if (tid == 0) {
      mbar_arrive_expect_tx(&mbar_b, kTileBytes);
      tma_load_2d(tileB, &tmap_b, kb * kBK, seg0 + n0, &mbar_b);
    }
    // A: 128 weight rows, dequantised
    if (p.mode == 0)
      dequant_q4k_row(my_row, kb, tileA, tid);
    else
      dequant_q6k_row(my_row, kb, tileA, tid);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic stores -> visible to the MMA
    __syncthreads();
    if (tid == 0) {
      bool ok = mbar_wait(&mbar_b, unsigned(kb & 1));
      if (ok) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t da = smem_desc(tileA), db = smem_desc(tileB);
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k)  // 32 bytes of K per MMA: +2 in the 16-byte address field
          mma_f16(tmem_d, da + 2 * k, db + 2 * k, (kb | k) != 0 ? 1u : 0u);
        mma_commit(&mbar_mma);
        ++issued;
      } else {
        fail = 1;
        set_status(p.status, kStatusBarrierTimeout);
      }
    }
    __syncthreads();
    if (fail) break;
    // the tiles are rewritten next iteration: wait until the MMAs have consumed them (the decision to stop is
    // taken after a CTA barrier, so every thread leaves the loop together)
    if (!mbar_wait(&mbar_mma, unsigned(kb & 1))) {
      fail = 1;
      set_status(p.status, kStatusBarrierTimeout);
    }
    __syncthreads();
    if (fail) break;
  }
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (!fail) {
    float* xbuf = reinterpret_cast<float*>(base);  // [32 columns][64 rows] up values, reusing the tiles
    if (p.mode == 0) {
      // gate rows in warps 0-1, up rows in warps 2-3; up values pass through shared memory column by column
      for (int c0 = 0; c0 < kBN; c0 += 32) {
        float v[32];
        tmem_ld32(tmem_d + (uint32_t(32 * warp) << 16) + uint32_t(c0), v);
        if (warp >= 2) {
#pragma unroll
          for (int i = 0; i < 32; ++i) xbuf[i * 64 + (tid - 64)] = v[i];
        }
        __syncthreads();
        if (warp < 2) {
          const int j = 64 * mt + tid;  // h index
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int col = c0 + i;
            if (col < n_valid) {
              const float up = xbuf[i * 64 + tid];
              p.out[size_t(seg0 + n0 + col) * p.F + j] = __float2half_rn(silu(v[i]) * up * (1.0f / 32.0f));
            }
          }
        }
        __syncthreads();
      }
    } else {
      const int row = kBM * mt + tid;  // hidden row
      for (int c0 = 0; c0 < kBN; c0 += 32) {
        float v[32];
        tmem_ld32(tmem_d + (uint32_t(32 * warp) << 16) + uint32_t(c0), v);
        for (int i = 0; i < 32; ++i) {
          const int col = c0 + i;
          if (col < n_valid) p.out[size_t(seg0 + n0 + col) * p.H + row] = __float2half_rn(v[i]);
        }
      }
    }
  } else if (issued > 0) {
    // a wait ran out: let the MMAs already committed finish (bounded) before the accumulator is freed
    mbar_wait(&mbar_mma, unsigned((issued - 1) & 1));
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(kBN) : "memory");
}

// Work list: one item per (segment, 128-token tile).
__global__ void tile_list_kernel(PairMap pm, int2* items, int* n_items) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const int n = *pm.n_used;
  int k = 0;
  for (int u = 0; u < n; ++u) {
    const int cnt = pm.seg[u + 1] - pm.seg[u];
    for (int n0 = 0; n0 < cnt; n0 += kBN) items[k++] = make_int2(u, n0);
  }
  *n_items = k;
}

// X_g[p] = fp16(x[token(p)]) for every pair position p (routed pairs, then the shared expert's rows).
template <typename XT>
__global__ void gather_fp16_kernel(PairMap pm, const XT* __restrict__ x, int H, __half* __restrict__ xg) {
  const int p = blockIdx.x;
  const int t = pair_token(pm, p);
  const XT* src = x + size_t(t) * H;
  __half* dst = xg + size_t(p) * H;
  for (int i = threadIdx.x * 4; i < H; i += blockDim.x * 4) {
    const float a = to_f32(src[i]), b = to_f32(src[i + 1]), c = to_f32(src[i + 2]), d = to_f32(src[i + 3]);
    *reinterpret_cast<uint2*>(dst + i) = make_uint2(pack_h2(a, b), pack_h2(c, d));
  }
}

// Combine from the fp16 down outputs (stored / 32): out[t] = sum over picks in ascending expert id of
// w * 32 * y[pick] (engines/base.py:580-586), + s_t * 32 * y[shared row t] (base.py:481-489).
template <int K>
__global__ void __launch_bounds__(256) combine_f16_kernel(PairMap pm, int H, const float* __restrict__ topk_w,
                                                          const float* __restrict__ shared_s,
                                                          const __half* __restrict__ y, void* __restrict__ out,
                                                          int out_dtype) {
  const int t = blockIdx.y;
  int ps[K];
  float ws[K];
#pragma unroll
  for (int s = 0; s < K; ++s) {
    ps[s] = pm.pos[size_t(t) * K + s];
    ws[s] = topk_w[size_t(t) * K + s] * 32.0f;
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
  const float s = shared_s[t] * 32.0f;
  const size_t shared_row = size_t(pm.T) * K + t;
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < H; r += gridDim.x * blockDim.x) {
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < K; ++i) acc = __fadd_rn(acc, __fmul_rn(__half2float(y[size_t(ps[i]) * H + r]), ws[i]));
    acc = __fadd_rn(acc, __fmul_rn(s, __half2float(y[shared_row * H + r])));
    if (out_dtype == kF32)
      static_cast<float*>(out)[size_t(t) * H + r] = acc;
    else
      static_cast<__nv_bfloat16*>(out)[size_t(t) * H + r] = __float2bfloat16_rn(acc);
  }
}

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(f);
  }
  return fn;
}

// fp16 [rows, cols] row-major, tiles of 128 rows x 64 columns with the 128-byte swizzle
cudaError_t make_tmap(CUtensorMap* map, const __half* base, uint64_t rows, uint64_t cols) {
  EncodeFn fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * sizeof(__half)};
  const cuuint32_t box[2] = {uint32_t(kBK), uint32_t(kBN)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// Two tiles, 1024-aligned (the epilogue reuses them), padded so that at most 4 CTAs share an SM: their 4 x 128
// TMEM columns then fit the SM's 512 and tcgen05.alloc never has to wait for another CTA.
constexpr size_t kSmem = 48 * 1024 + 1024;

}  // namespace

size_t prefill_scratch_bytes(int T, int k, int E, int H, int F) {
  const size_t P = size_t(T) * (k + 1);
  const size_t items = P / kBN + size_t(E) + 2;
  return items * sizeof(int2) + 256 + P * H * sizeof(__half) * 2 + P * F * sizeof(__half) + 4 * 256;
}

cudaError_t prefill_experts(const ExpertSource& src, int layer, const PairMap& pm, int H, int F, const void* x,
                            int x_dtype, const float* topk_w, const float* shared_s, void* out, int out_dtype,
                            void* scratch, int* status, cudaStream_t st, int* launches) {
  if (H % kBK || F % kBK || F % 128 || H % 128) return cudaErrorInvalidValue;
  const size_t P = size_t(pm.T) * (pm.k + 1);
  const size_t max_items = P / kBN + size_t(pm.E) + 2;
  char* b = static_cast<char*>(scratch);
  int2* items = reinterpret_cast<int2*>(b);
  b += (max_items * sizeof(int2) + 255) / 256 * 256;
  int* n_items = reinterpret_cast<int*>(b);
  b += 256;
  __half* xg = reinterpret_cast<__half*>(b);
  b += (P * H * sizeof(__half) + 255) / 256 * 256;
  __half* hbuf = reinterpret_cast<__half*>(b);
  b += (P * F * sizeof(__half) + 255) / 256 * 256;
  __half* ybuf = reinterpret_cast<__half*>(b);

  tile_list_kernel<<<1, 32, 0, st>>>(pm, items, n_items);
  if (x_dtype == kF32)
    gather_fp16_kernel<float><<<unsigned(P), 256, 0, st>>>(pm, static_cast<const float*>(x), H, xg);
  else
    gather_fp16_kernel<__nv_bfloat16><<<unsigned(P), 256, 0, st>>>(pm, static_cast<const __nv_bfloat16*>(x), H, xg);
  *launches += 2;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;

  e = cudaFuncSetAttribute(grouped_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmem));
  if (e != cudaSuccess) return e;
  CUtensorMap map_x, map_h;
  if ((e = make_tmap(&map_x, xg, P, uint64_t(H))) != cudaSuccess) return e;
  if ((e = make_tmap(&map_h, hbuf, P, uint64_t(F))) != cudaSuccess) return e;

  GemmParams gp{};
  gp.src = src;
  gp.layer = layer;
  gp.pm = pm;
  gp.items = items;
  gp.n_items = n_items;
  gp.F = F;
  gp.H = H;
  gp.status = status;
  gp.mode = 0;
  gp.out = hbuf;
  grouped_gemm_kernel<<<dim3(unsigned(F / 64), unsigned(max_items)), kThreads, kSmem, st>>>(map_x, gp);
  gp.mode = 1;
  gp.out = ybuf;
  grouped_gemm_kernel<<<dim3(unsigned(H / kBM), unsigned(max_items)), kThreads, kSmem, st>>>(map_h, gp);
  if (pm.k != 8) return cudaErrorInvalidValue;
  combine_f16_kernel<8><<<dim3(unsigned((H + 255) / 256), unsigned(pm.T)), 256, 0, st>>>(pm, H, topk_w, shared_s, ybuf,
                                                                                         out, out_dtype);
  *launches += 3;
  return cudaGetLastError();
}

}  // namespace wmoe
