// Grouped expert GEMMs for many tokens per expert (prefill), on the 5th-generation tensor cores (tcgen05 + TMEM).
// Replaces willow's dequantize-to-bf16 + matmul path for more than 8 tokens (gguf/metal.py:357-363, 404-407) and
// the per-expert loop of Engine.each_expert (engines/base.py:534-591).
//
// Swap-AB: the expert's weight rows are the MMA's M (128 per tile), its tokens are N (a chunk of up to 192 of the
// expert's tokens; the MMA's N is the chunk rounded up to 16), K runs over the hidden size (gate_up, Q4_K) or the
// FFN width (down, Q6_K) in blocks of 64. An item is (chunk, 128-row M tile). The kernel is persistent: one CTA
// per SM walks the items i = blockIdx.x, + gridDim.x, ... with specialised warps:
//   warp 0      TMA: the token tile of each K block (fp16, 128-byte swizzle) into a shared-memory ring
//   warp 1      allocates all 512 TMEM columns: two fp32 accumulators of 192 columns and a 4-stage ring of fp16
//               weight tiles (32 columns each). One lane issues 4 tcgen05.mma (K = 16) per K block with A read
//               from TMEM and B from shared memory; tcgen05.commit frees the stages, and after an item's last K
//               block marks its accumulator full
//   warp 2      the weight bytes into shared memory. Q4_K: one super-block column (144 bytes of 128 rows) per
//               TMA load pair, 3 deep (the expert matrices are a 3-D tensor map over the slab). Q6_K: the item's
//               128 rows, contiguous, by one bulk copy, 2 deep
//   warps 3-6   the epilogue: accumulator -> registers (tcgen05.ld), SwiGLU or scaling, fp16 stores; it works on
//               one accumulator while the MMAs fill the other
//   warps 7-14  dequantise the 128 x 64 weight tile of each K block from the shared-memory bytes into a TMEM
//               stage (tcgen05.st), two groups of 4 warps taking alternate K blocks; thread = tile row = TMEM lane
// Keeping A out of shared memory matters: an M = 128 MMA already reads ~100 bytes per clock of shared memory for
// its operands, close to the port's 128, so writing and re-reading the dequantised tile there would bound the
// kernel by shared-memory bandwidth.
// Dequantisation is packed fp16 arithmetic: codes are moved into the low mantissa bits of 1024.0 (low nibbles,
// 6-bit codes) or 64.0 (high nibbles, spacing 1/16) by byte permutes and masks, the magic is subtracted exactly,
// and one fused multiply-add applies the sub-block's d*sc and -dmin*mn rounded to fp16 (measured error on an
// expert FFN: 5.2e-4 relative L2 against the float32 reference; bound 2e-3). The codes of a 32-bit word come out
// as elements (0, 2, 1, 3) of its 4, so the activations are stored with the same order inside every run of 8
// (gather and SwiGLU epilogue), which leaves every dot product unchanged.
// gate_up tiles pair 64 gate rows with the 64 matching up rows (rows j and F + j): the epilogue forms
// h = silu(gate) * up, stored as fp16 h / kHScale (fp16 keeps the precision the 2e-3 bound needs, bf16 does not);
// down tiles write y / kYScale as fp16 and the combine multiplies kYScale back. The powers of two place fp16's
// window at |h| <= 1.7e7 and |y| <= 2.7e8 (BASELINE's synthetic experts reach |y| ~ 2e6 a few layers deep), with
// an absolute floor below 1e-4; a value outside the window sets the device status instead of passing on an inf.
// Every wait is bounded (1 s of %globaltimer) and any timeout stops every role: the CTA records the device status,
// waits (bounded) for its copies and MMAs in flight, frees its TMEM and returns.
#include <cuda.h>

#include "common.cuh"
#include "kernels.cuh"
#include "sm100.cuh"

namespace wmoe {

namespace {

using namespace sm100;

constexpr int kBM = 128, kBN = 192, kBK = 64, kBoxRows = 64;
constexpr int kAStages = 4;                           // weight tiles in TMEM
constexpr int kAccCols = kBN;                         // accumulator b at columns [b * kBN, (b + 1) * kBN)
constexpr int kACol0 = 2 * kAccCols;                  // weight stage s at columns kACol0 + 32 s
constexpr int kTmemCols = 512;
static_assert(kACol0 + 32 * kAStages <= kTmemCols, "TMEM columns");
constexpr int kMaxBStages = 6;
constexpr int kWarps = 15, kThreads = kWarps * 32;
constexpr float kHScale = 256.f, kYScale = 4096.f;  // h and y are stored as fp16 h / kHScale, y / kYScale
constexpr int kTileB = kBN * kBK * 2;                 // 24 KB fp16 tokens
constexpr int kQ4Row = 144;                           // one Q4_K super-block of a row
constexpr int kQ4Unit = kBM * kQ4Row;                 // 18,432 B: one super-block column of the tile
constexpr int kQ6Unit = kBM * 2 * Q6K_BYTES;          // 53,760 B: 128 down rows of F = 512
constexpr int kQ4DRow = 2 * Q4K_BYTES;                // a Q4_K down row of F = 512
constexpr int kQ4DUnit = kBM * kQ4DRow;               // 36,864 B: 128 Q4_K down rows
constexpr int kXbufBytes = 32 * 64 * 4;               // gate/up exchange of 32 columns (fp32)
constexpr int kOutBytes = 32 * kBM * 2;                // one 32-column chunk of the output, token-major fp16

// MODE 0: gate_up (Q4_K) + SwiGLU; 1: down with Q6_K rows; 2: down with Q4_K rows
template <int MODE>
struct Layout {
  static constexpr int bstages = MODE == 0 ? 6 : 4;      // token tile ring
  static constexpr int depth = MODE == 1 ? 2 : 3;        // weight byte ring
  static constexpr int unit = MODE == 0 ? kQ4Unit : (MODE == 1 ? kQ6Unit : kQ4DUnit);
  static constexpr int raw = bstages * kTileB;           // weight ring offset (1024-aligned)
  static constexpr int xbuf = raw + depth * unit;        // gate_up only
  static constexpr int obuf = xbuf + (MODE == 0 ? kXbufBytes : 0);
  static constexpr int bytes = obuf + kOutBytes + 1024;  // + alignment slack
};
static_assert(Layout<0>::bytes <= 232448 && Layout<1>::bytes <= 232448 && Layout<2>::bytes <= 232448, "shared memory");
static_assert(Layout<2>::bstages <= kMaxBStages && Layout<2>::depth <= 3 && kQ4DUnit % 1024 == 0, "Q4_K down ring");
static_assert(Layout<0>::bstages <= kMaxBStages && Layout<1>::bstages <= kMaxBStages, "barrier arrays");
static_assert(kTileB % 1024 == 0 && kQ4Unit % 1024 == 0, "TMA destinations stay 1024-aligned");




// Q4_K K block (sub-blocks 2g and 2g + 1 of one super-block) of one tile row, from the row's 144 bytes in shared
// memory, into the thread's TMEM lane at taddr: 32 columns of fp16 pairs, stored position p in column p / 2. Low
// nibbles of quant bytes 32g .. 32g + 31 are elements 0-31, high nibbles elements 32-63 (gguf/quants.py:82-98).
__device__ __forceinline__ void dequant_q4k_block(const uint8_t* row, int g, uint32_t taddr) {
  const uint4 hd = *reinterpret_cast<const uint4*>(row);
  const float d = f16_to_f32(uint16_t(hd.x & 0xFFFF)), dmin = f16_to_f32(uint16_t(hd.x >> 16));
  int sc0, mn0, sc1, mn1;
  q4k_scale_min_w(hd.y, hd.z, hd.w, 2 * g, sc0, mn0);
  q4k_scale_min_w(hd.y, hd.z, hd.w, 2 * g + 1, sc1, mn1);
  const __half2 A0 = __float2half2_rn(d * float(sc0)), A1 = __float2half2_rn(d * float(sc1));
  const __half2 B0 = __float2half2_rn(-dmin * float(mn0)), B1 = __float2half2_rn(-dmin * float(mn1));
  const uint4 qa = *reinterpret_cast<const uint4*>(row + 16 + 32 * g);
  const uint4 qb = *reinterpret_cast<const uint4*>(row + 32 + 32 * g);
  const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
  const __half2 k1024 = u2h(0x64006400u), k64 = u2h(0x54005400u);
  uint32_t o[16];
#pragma unroll
  for (int half = 0; half < 2; ++half) {  // low nibbles (elements 0-31), then high nibbles (32-63)
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const uint32_t pe = __byte_perm(qw[w], 0, 0x4240), po = __byte_perm(qw[w], 0, 0x4341);  // bytes (0,2), (1,3)
      if (half == 0) {
        o[2 * w] = h2u(__hfma2(__hsub2(u2h((pe & 0x000F000Fu) | 0x64006400u), k1024), A0, B0));
        o[2 * w + 1] = h2u(__hfma2(__hsub2(u2h((po & 0x000F000Fu) | 0x64006400u), k1024), A0, B0));
      } else {
        o[2 * w] = h2u(__hfma2(__hsub2(u2h((pe & 0x00F000F0u) | 0x54005400u), k64), A1, B1));
        o[2 * w + 1] = h2u(__hfma2(__hsub2(u2h((po & 0x00F000F0u) | 0x54005400u), k64), A1, B1));
      }
    }
    tmem_st16(taddr + uint32_t(16 * half), o);
  }
}

// Q6_K K block kb of one tile row (64 elements of super-block kb / 4: half hh = (kb % 4) / 2, quarters 2q and
// 2q + 1, q = kb % 2) from the row's bytes in shared memory (gguf/quants.py:120-140) into the thread's TMEM lane.
// Element e: ql byte hh*64 + e (nibble q), qh byte 128 + hh*32 + e % 32 (bits 4q + 2 (e / 32)), scale index
// hh*8 + 4q + e / 16.
__device__ __forceinline__ void dequant_q6k_block(const uint8_t* row, int kb, uint32_t taddr) {
  const uint8_t* b = row + (kb / 4) * Q6K_BYTES;
  const int hh = (kb % 4) / 2, q = kb % 2;
  uint32_t qh[8];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint4 v = lds_u2_16(b + 128 + hh * 32 + 16 * i);
    qh[4 * i] = v.x, qh[4 * i + 1] = v.y, qh[4 * i + 2] = v.z, qh[4 * i + 3] = v.w;
  }
  const uint4 scw = lds_u2_16(b + 192);
  const uint32_t sw[4] = {scw.x, scw.y, scw.z, scw.w};
  const float d = f16_to_f32(*reinterpret_cast<const uint16_t*>(b + 208));
  __half2 D[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int si = hh * 8 + 4 * q + i;
    D[i] = __float2half2_rn(d * float(int8_t((sw[si / 4] >> (8 * (si % 4))) & 0xFF)));
  }
  const __half2 k1056 = u2h(0x64206420u);  // 1024 + 32
#pragma unroll
  for (int half = 0; half < 2; ++half) {  // elements 32 half .. 32 half + 31
    uint32_t ql[8];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint4 v = lds_u2_16(b + hh * 64 + 32 * half + 16 * i);
      ql[4 * i] = v.x, ql[4 * i + 1] = v.y, ql[4 * i + 2] = v.z, ql[4 * i + 3] = v.w;
    }
    uint32_t o[16];
#pragma unroll
    for (int w = 0; w < 8; ++w) {  // elements 4w .. 4w + 3 of the half
      const uint32_t code = ((ql[w] >> (4 * q)) & 0x0F0F0F0Fu) |
                            (((qh[w] >> (4 * q + 2 * half)) & 0x03030303u) << 4);  // q6, 0..63
      const uint32_t pe = __byte_perm(code, 0x64646464u, 0x4240), po = __byte_perm(code, 0x64646464u, 0x4341);
      const __half2 dd = D[2 * half + w / 4];
      o[2 * w] = h2u(__hmul2(__hsub2(u2h(pe), k1056), dd));
      o[2 * w + 1] = h2u(__hmul2(__hsub2(u2h(po), k1056), dd));
    }
    tmem_st16(taddr + uint32_t(16 * half), o);
  }
}

struct GemmParams {
  ExpertSource src;
  int layer;
  PairMap pm;
  const int2* chunks;    // (segment u, first token of the chunk within the segment)
  const int* n_chunks;
  int n_mtiles;
  int F, H;
  __half* out;           // gate_up: h [P][F] (columns in run-of-8 order); down: y [P][H]
  const int32_t* out_rows;  // down: y row of pair position p < n_routed is out_rows[p] (null: p)
  int n_routed;
  int* status;
};

struct Item {
  int u, seg0, n0, ncols, mt;
};

__device__ __forceinline__ Item get_item(const GemmParams& p, int i) {
  Item t;
  const int2 c = p.chunks[i / p.n_mtiles];
  t.mt = i % p.n_mtiles;
  t.u = c.x;
  t.n0 = c.y;
  t.seg0 = p.pm.seg[t.u];
  t.ncols = min(kBN, p.pm.seg[t.u + 1] - t.seg0 - t.n0);
  return t;
}

// slot of the item's expert in the slab, kSharedSlot for the shared expert, -1 if not resident
constexpr int kSharedSlot = -2;
__device__ __forceinline__ int item_slot(const GemmParams& p, int u) {
  const int e = p.pm.used[u];
  if (e == p.src.experts) return kSharedSlot;
  return p.src.slot_of[size_t(p.layer) * p.src.experts + e];
}

struct Bars {
  uint64_t full_a[kAStages], empty_a[kAStages];
  uint64_t full_b[kMaxBStages], empty_b[kMaxBStages];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t raw_full[3], raw_empty[3];
  uint64_t done;
  uint32_t tmem;
  int fail;
};

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmap_b, const __grid_constant__ CUtensorMap tmap_w,
                        const __grid_constant__ CUtensorMap tmap_ws, const __grid_constant__ GemmParams p) {
  using L = Layout<MODE>;
  constexpr int BS = L::bstages;
  extern __shared__ __align__(1024) uint8_t dyn[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn) + 1023) & ~uintptr_t(1023));
  uint8_t* raw = base + L::raw;
  __shared__ Bars bars;

  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int total = *p.n_chunks * p.n_mtiles;
  const int K = MODE == 0 ? p.H : p.F, nk = K / kBK;
  const int units = MODE == 0 ? K / QK : 1;  // weight units per item

  if (tid == 0) {
    bars.fail = 0;
    for (int s = 0; s < kAStages; ++s) {
      mbar_init(&bars.full_a[s], 4);  // the 4 warps of one dequant group
      mbar_init(&bars.empty_a[s], 1);
    }
    for (int s = 0; s < BS; ++s) {
      mbar_init(&bars.full_b[s], 1);
      mbar_init(&bars.empty_b[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars.acc_full[b], 1);
      mbar_init(&bars.acc_empty[b], 4);  // the 4 epilogue warps
    }
    for (int s = 0; s < L::depth; ++s) {
      mbar_init(&bars.raw_full[s], 1);
      mbar_init(&bars.raw_empty[s], 8);  // all 8 dequant warps
    }
    mbar_init(&bars.done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&bars.tmem)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem_base = bars.tmem;
  volatile int* fail = &bars.fail;
  int issued_b = 0, issued_w = 0;  // copies the two producer lanes issued (for the drain after a failure)

  if (warp == 0) {
    // ---------------- token tiles: 1-3 boxes of 64 rows per K block
    if (lane == 0) {
      int it = 0;
      for (int i = blockIdx.x; i < total; i += gridDim.x, ++it) {
        const Item t = get_item(p, i);
        const int nbox = (t.ncols + kBoxRows - 1) / kBoxRows;
        for (int kb = 0; kb < nk; ++kb) {
          const int kbg = it * nk + kb, s = kbg % BS;
          if (kbg >= BS && !mbar_wait(&bars.empty_b[s], unsigned((kbg / BS - 1) & 1), fail)) goto out;
          mbar_arrive_expect_tx(&bars.full_b[s], unsigned(nbox * kBoxRows * kBK * 2));
          uint8_t* dst = base + s * kTileB;
          for (int bx = 0; bx < nbox; ++bx)
            tma_load_2d(dst + bx * kBoxRows * 128, &tmap_b, kb * kBK, t.seg0 + t.n0 + bx * kBoxRows, &bars.full_b[s]);
          issued_b = kbg + 1;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: A from the TMEM ring, B from the shared-memory ring
    if (lane == 0) {
      int it = 0;
      for (int i = blockIdx.x; i < total; i += gridDim.x, ++it) {
        const Item t = get_item(p, i);
        const int buf = it & 1;
        if (it >= 2 && !mbar_wait(&bars.acc_empty[buf], unsigned((it / 2 - 1) & 1), fail)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t idesc = idesc_f16(kBM, (t.ncols + 15) & ~15, false);
        const uint32_t d = tmem_base + uint32_t(buf * kAccCols);
        bool ok = true;
        for (int kb = 0; kb < nk && ok; ++kb) {
          const int kbg = it * nk + kb, sa = kbg % kAStages, sb = kbg % BS;
          ok = mbar_wait(&bars.full_a[sa], unsigned((kbg / kAStages) & 1), fail) &&
               mbar_wait(&bars.full_b[sb], unsigned((kbg / BS) & 1), fail);
          if (!ok) break;
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t ta = tmem_base + uint32_t(kACol0 + 32 * sa);
          const uint64_t db = smem_desc(base + sb * kTileB);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)  // K = 16 per MMA: 8 TMEM columns of A, +32 bytes (+2) of B
            mma_f16_ts(d, ta + uint32_t(8 * k), db + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
          mma_commit(&bars.empty_a[sa]);
          mma_commit(&bars.empty_b[sb]);
        }
        if (!ok) break;
        mma_commit(&bars.acc_full[buf]);
      }
      mma_commit(&bars.done);  // arrives once every MMA issued above has completed
    }
  } else if (warp == 2) {
    // ---------------- weight bytes
    if (lane == 0) {
      int it = 0;
      for (int i = blockIdx.x; i < total; i += gridDim.x, ++it) {
        const Item t = get_item(p, i);
        const int slot = item_slot(p, t.u);
        if (slot == -1 || slot >= p.src.n_slots) {
          set_status(p.status, kStatusNotResident);
          *fail = 1;
          break;
        }
        for (int un = 0; un < units; ++un) {
          const int ru = it * units + un, rs = ru % L::depth;
          if (ru >= L::depth && !mbar_wait(&bars.raw_empty[rs], unsigned((ru / L::depth - 1) & 1), fail)) goto out;
          uint8_t* dst = raw + rs * L::unit;
          mbar_arrive_expect_tx(&bars.raw_full[rs], unsigned(L::unit));
          if (MODE == 0) {  // gate rows 64 mt .., up rows F + 64 mt .., super-block un
            const CUtensorMap* m = slot == kSharedSlot ? &tmap_ws : &tmap_w;
            const int z = slot == kSharedSlot ? 0 : slot;
            tma_load_3d(dst, m, un * kQ4Row, 64 * t.mt, z, &bars.raw_full[rs]);
            tma_load_3d(dst + 64 * kQ4Row, m, un * kQ4Row, p.F + 64 * t.mt, z, &bars.raw_full[rs]);
          } else {
            const uint8_t* w = slot == kSharedSlot
                                   ? p.src.shared_down
                                   : p.src.slab + size_t(slot) * p.src.slot_bytes + p.src.gate_up_bytes;
            bulk_g2s(dst, w + size_t(L::unit) * t.mt, unsigned(L::unit), &bars.raw_full[rs]);
          }
          issued_w = ru + 1;
        }
      }
    }
  } else if (warp <= 6) {
    // ---------------- epilogue (warps 3-6 cover the four TMEM lane quadrants). Per 32-column chunk: accumulator
    // -> registers (thread = row), SwiGLU or scaling, fp16 into a token-major chunk in shared memory, then 16-byte
    // stores of whole token rows.
    const int quad = warp % 4, trow = 32 * quad + lane, e = tid - 96;
    float* xbuf = reinterpret_cast<float*>(base + L::xbuf);     // [32 columns][64 rows] up values
    __half* obuf = reinterpret_cast<__half*>(base + L::obuf);   // [32 columns][rows of the tile] fp16
    constexpr int orows = MODE == 0 ? 64 : kBM;                 // output rows per tile
    const int ld = MODE == 0 ? p.F : p.H;
    int it = 0;
    for (int i = blockIdx.x; i < total; i += gridDim.x, ++it) {
      const Item t = get_item(p, i);
      const int buf = it & 1;
      const bool ready = mbar_wait(&bars.acc_full[buf], unsigned((it / 2) & 1), fail) && !*fail;
      unsigned all_ready;  // one decision for the four epilogue warps (they meet at named barrier 1)
      asm volatile(
          "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, 1, 128, p;\n selp.u32 %0, 1, 0, q;\n}\n"
          : "=r"(all_ready)
          : "r"(unsigned(ready))
          : "memory");
      if (!all_ready) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t taddr = tmem_base + uint32_t(buf * kAccCols) + (uint32_t(32 * quad) << 16);
      const int prow0 = t.seg0 + t.n0;  // pair position of the chunk's first token
      __half* gout = p.out + orows * t.mt;
      for (int c0 = 0; c0 < t.ncols; c0 += 32) {
        float v[32];
        tmem_ld32(taddr + uint32_t(c0), v);
        const int nv = min(32, t.ncols - c0);  // columns past the chunk's tokens hold padding or stale values
        if (MODE == 0) {
          // gate rows are quadrants 0-1, up rows quadrants 2-3; h index 64 mt + trow, stored in run-of-8 order
          if (quad >= 2) {
#pragma unroll
            for (int c = 0; c < 32; ++c) xbuf[c * 64 + (trow - 64)] = v[c];
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (quad < 2) {
            const int j = perm8(trow);
            float vmax = 0.f;
#pragma unroll
            for (int c = 0; c < 32; ++c) {
              const float g = v[c];
              const float hv = __fdividef(g, 1.0f + __expf(-g)) * xbuf[c * 64 + trow] * (1.0f / kHScale);
              if (c < nv) vmax = fmaxf(vmax, fabsf(hv));
              obuf[c * 64 + j] = __float2half_rn(hv);
            }
            if (!(vmax <= 65504.f)) set_status(p.status, kStatusRange);
          }
        } else {
          // the accumulator holds y / kHScale
          float vmax = 0.f;
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const float yv = v[c] * (kHScale / kYScale);
            if (c < nv) vmax = fmaxf(vmax, fabsf(yv));
            obuf[c * kBM + trow] = __float2half_rn(yv);
          }
          if (!(vmax <= 65504.f)) set_status(p.status, kStatusRange);
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const int n = nv;
        // output row of column c0 + lane (remapped rows of the down launch fetched once per chunk)
        int lane_row = prow0 + c0 + lane;
        if (MODE != 0 && p.out_rows && lane < n && lane_row < p.n_routed) lane_row = p.out_rows[lane_row];
        constexpr int pieces = 32 * orows / 8;  // 16-byte pieces of the chunk
#pragma unroll
        for (int q = e; q < pieces; q += 128) {
          const int c = q / (orows / 8), g = q % (orows / 8);
          const int row = __shfl_sync(0xffffffffu, lane_row, c);
          if (c < n)
            *reinterpret_cast<uint4*>(gout + size_t(row) * ld + 8 * g) =
                *reinterpret_cast<const uint4*>(obuf + c * orows + 8 * g);
        }
        if (MODE != 0) asm volatile("bar.sync 1, 128;" ::: "memory");  // obuf is rewritten by the next chunk
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars.acc_empty[buf]);
    }
  } else {
    // ---------------- dequantisation: group j takes the K blocks kb with kb % 2 == j; thread = tile row = TMEM
    // lane 32 (warp % 4) + lane (a warp reaches only its own lane quadrant)
    const int dw = warp - 7, j = dw / 4, r = 32 * (warp % 4) + lane;
    const uint32_t tlane = tmem_base + (uint32_t(32 * (warp % 4)) << 16);
    int it = 0;
    for (int i = blockIdx.x; i < total; i += gridDim.x, ++it) {
      for (int un = 0; un < units; ++un) {
        const int ru = it * units + un, rs = ru % L::depth;
        if (!mbar_wait_warp(&bars.raw_full[rs], unsigned((ru / L::depth) & 1), fail)) goto out;
        const uint8_t* wrow = raw + rs * L::unit + r * (MODE == 0 ? kQ4Row : (MODE == 1 ? 2 * Q6K_BYTES : kQ4DRow));
        const int kb0 = MODE == 0 ? 4 * un : 0, kb1 = MODE == 0 ? 4 * un + 4 : nk;
        for (int kb = kb0 + j; kb < kb1; kb += 2) {
          const int kbg = it * nk + kb, s = kbg % kAStages;
          if (kbg >= kAStages &&
              !mbar_wait_warp(&bars.empty_a[s], unsigned((kbg / kAStages - 1) & 1), fail))
            goto out;
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t ta = tlane + uint32_t(kACol0 + 32 * s);
          if (MODE == 0)
            dequant_q4k_block(wrow, kb % 4, ta);
          else if (MODE == 1)
            dequant_q6k_block(wrow, kb, ta);
          else  // K block kb: nibble group kb % 4 of super-block kb / 4
            dequant_q4k_block(wrow + (kb / 4) * Q4K_BYTES, kb % 4, ta);
          asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
          asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars.full_a[s]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars.raw_empty[rs]);
      }
    }
  }
out:
  __syncwarp();
  if (tid == 0 && *fail) set_status(p.status, kStatusBarrierTimeout);
  {
    // every MMA this CTA issued has completed, and after a failure every copy in flight gets a bounded wait,
    // before the CTA frees its shared memory and TMEM
    volatile int never = 0;
    if (warp == 1) mbar_wait(&bars.done, 0, &never);
    if (*fail && lane == 0) {
      if (warp == 0)
        for (int kbg = max(0, issued_b - BS); kbg < issued_b; ++kbg)
          mbar_wait(&bars.full_b[kbg % BS], unsigned((kbg / BS) & 1), &never);
      if (warp == 2)
        for (int ru = max(0, issued_w - L::depth); ru < issued_w; ++ru)
          mbar_wait(&bars.raw_full[ru % L::depth], unsigned((ru / L::depth) & 1), &never);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols) : "memory");
}

// Chunk list: one entry per (segment, up to kBN tokens), segments in order.
__global__ void __launch_bounds__(512) chunk_list_kernel(PairMap pm, int2* chunks, int* n_chunks) {
  __shared__ int warp_sum[16];
  const int n = *pm.n_used, u = threadIdx.x, lane = u % 32, wid = u / 32;
  const int cnt = u < n ? (pm.seg[u + 1] - pm.seg[u] + kBN - 1) / kBN : 0;
  int incl = cnt;  // inclusive scan within the warp, then across the 16 warp totals
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += v;
  }
  if (lane == 31) warp_sum[wid] = incl;
  __syncthreads();
  int before = 0, total = 0;
  for (int i = 0; i < 16; ++i) {
    before += i < wid ? warp_sum[i] : 0;
    total += warp_sum[i];
  }
  const int off = before + incl - cnt;
  for (int c = 0; c < cnt; ++c) chunks[off + c] = make_int2(u, c * kBN);
  if (u == 0) *n_chunks = total;
}

// X_g[p] = fp16(x[token(p)]) for every pair position p (routed pairs, then the shared expert's rows), columns in
// run-of-8 order.
template <typename XT>
__global__ void __launch_bounds__(256) gather_fp16_kernel(PairMap pm, const XT* __restrict__ x, int H,
                                                          __half* __restrict__ xg) {
  const int p = blockIdx.x;
  const int t = pair_token(pm, p);
  const XT* src = x + size_t(t) * H;
  __half* dst = xg + size_t(p) * H;
  for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
    float v[8];
    load8(src + i, v);
    *reinterpret_cast<uint4*>(dst + i) = pack8_perm(v);
  }
}

// Combine from the fp16 down outputs (stored / kYScale): out[t] = sum over the token's picks in ascending expert id
// of w * kYScale * y_routed[rows[t][j]] (engines/base.py:580-586), + s_t * kYScale * y_shared[t] (base.py:481-489).
// One CTA per token, 8 consecutive outputs per thread from 16-byte loads of each row. The token rows (x) are
// converted to fp16 unscaled: callers pass normalised hidden states (|x| far below 65504). With the residual
// epilogue (an.h set) the CTA adds its row to h[t] and, when an.xn is set, writes the next layer's normalised input
// from the updated row it holds: the separate residual + RMSNorm pass over the activations goes away. EPI selects
// the epilogue at compile time (a run-time branch cost the plain combine 8%).
template <int K, bool EPI>
__global__ void __launch_bounds__(256) combine_rows_kernel(int H, const int32_t* __restrict__ topk_idx,
                                                           const float* __restrict__ topk_w,
                                                           const int32_t* __restrict__ rows,
                                                           const float* __restrict__ shared_s,
                                                           const __half* __restrict__ y_routed,
                                                           const __half* __restrict__ y_shared,
                                                           void* __restrict__ out, int out_dtype, AddNorm an) {
  __shared__ float red[32];
  const int t = blockIdx.x;
  int ex[K], ps[K];
  float ws[K];
#pragma unroll
  for (int s = 0; s < K; ++s) {
    ex[s] = topk_idx[size_t(t) * K + s];
    ps[s] = rows[size_t(t) * K + s];
    ws[s] = topk_w[size_t(t) * K + s] * kYScale;
  }
#pragma unroll
  for (int i = 1; i < K; ++i)
#pragma unroll
    for (int j = i; j > 0; --j)
      if (ex[j] < ex[j - 1]) {
        const int te = ex[j];
        ex[j] = ex[j - 1];
        ex[j - 1] = te;
        const int tp = ps[j];
        ps[j] = ps[j - 1];
        ps[j - 1] = tp;
        const float tw = ws[j];
        ws[j] = ws[j - 1];
        ws[j - 1] = tw;
      }
  const float s = shared_s[t] * kYScale;
  float ss = 0.f;  // squares of the updated residual row (epilogue)
  for (int r = threadIdx.x * 8; r < H; r += blockDim.x * 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < K + 1; ++i) {
      const __half* src = i < K ? y_routed + size_t(ps[i]) * H : y_shared + size_t(t) * H;
      const float wi = i < K ? ws[i] : s;
      const uint4 u = *reinterpret_cast<const uint4*>(src + r);
      const uint32_t hw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hw[j]));
        acc[2 * j] = __fadd_rn(acc[2 * j], __fmul_rn(f.x, wi));
        acc[2 * j + 1] = __fadd_rn(acc[2 * j + 1], __fmul_rn(f.y, wi));
      }
    }
    if constexpr (EPI) {  // h[t] += out[t] (x + moe(...), engines/qwen36/model.py:22)
      float4* hp = reinterpret_cast<float4*>(an.h + size_t(t) * H + r);
      const float4 a = hp[0], b = hp[1];
      const float v[8] = {__fadd_rn(a.x, acc[0]), __fadd_rn(a.y, acc[1]), __fadd_rn(a.z, acc[2]),
                          __fadd_rn(a.w, acc[3]), __fadd_rn(b.x, acc[4]), __fadd_rn(b.y, acc[5]),
                          __fadd_rn(b.z, acc[6]), __fadd_rn(b.w, acc[7])};
      hp[0] = make_float4(v[0], v[1], v[2], v[3]);
      hp[1] = make_float4(v[4], v[5], v[6], v[7]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(v[j], v[j], ss);
    } else {
      store8(out, out_dtype == kF32, size_t(t) * H + r, acc);
    }
  }
  if (EPI && an.xn) {  // uniform over the CTA: xn[t] = h[t] / sqrt(mean(h[t]^2) + eps) (engines/base.py:27-32)
    const float rs = rsqrtf(block_sum(ss, red) / float(H) + an.eps);
    for (int r = threadIdx.x * 8; r < H; r += blockDim.x * 8) {
      const float4* hp = reinterpret_cast<const float4*>(an.h + size_t(t) * H + r);
      const float4 a = hp[0], b = hp[1];
      const float v[8] = {a.x * rs, a.y * rs, a.z * rs, a.w * rs, b.x * rs, b.y * rs, b.z * rs, b.w * rs};
      store8(an.xn, an.xn_dtype == kF32, size_t(t) * H + r, v);
    }
  }
}

// fp16 [rows, cols] row-major, boxes of 128 rows x 64 columns with the 128-byte swizzle
cudaError_t make_tmap_f16(CUtensorMap* map, const __half* ptr, uint64_t rows, uint64_t cols) {
  EncodeFn fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * sizeof(__half)};
  const cuuint32_t box[2] = {uint32_t(kBK), uint32_t(kBoxRows)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// Q4_K matrices as bytes [slots][rows][row_bytes] (slot stride slot_bytes), boxes of one super-block (144 bytes)
// of 64 rows, no swizzle.
cudaError_t make_tmap_q4k(CUtensorMap* map, const uint8_t* ptr, uint64_t row_bytes, uint64_t rows, uint64_t slots,
                          uint64_t slot_bytes) {
  EncodeFn fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  const cuuint64_t dims[3] = {row_bytes, rows, slots};
  const cuuint64_t strides[2] = {row_bytes, slot_bytes};
  const cuuint32_t box[3] = {uint32_t(kQ4Row), 64, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace

size_t prefill_gemm_scratch_bytes(size_t P, int E, int H, int F) {
  const size_t chunks = P / kBN + size_t(E) + 2;
  return (chunks * sizeof(int2) + 255) / 256 * 256 + 256 + (P * F * sizeof(__half) + 255) / 256 * 256;
}

size_t prefill_scratch_bytes(int T, int k, int E, int H, int F) {
  const size_t P = size_t(T) * (k + 1);
  return prefill_gemm_scratch_bytes(P, E, H, F) + 2 * ((P * H * sizeof(__half) + 255) / 256 * 256);
}

cudaError_t check_weight_alignment(const ExpertSource& src) {
  // weight rows are copied by TMA and bulk copies: the matrices must start on 16-byte boundaries
  if (reinterpret_cast<uintptr_t>(src.shared_down) % 16 || reinterpret_cast<uintptr_t>(src.shared_gate_up) % 16 ||
      reinterpret_cast<uintptr_t>(src.slab) % 16 || src.slot_bytes % 16 || src.gate_up_bytes % 16)
    return cudaErrorInvalidValue;
  return cudaSuccess;
}

cudaError_t prefill_gemms(const ExpertSource& src, int layer, const PairMap& pm, size_t P, int H, int F,
                          const __half* xg, __half* y, const int32_t* out_rows, int n_routed, void* scratch,
                          int num_sms, int* status, const cudaEvent_t* marks, cudaStream_t st, int* launches) {
  if (H % QK || F != 2 * QK || H % kBM || pm.E + 1 > 512 || num_sms <= 0) return cudaErrorInvalidValue;
  cudaError_t e = check_weight_alignment(src);
  if (e != cudaSuccess) return e;
  const size_t max_chunks = P / kBN + size_t(pm.E) + 2;
  char* b = static_cast<char*>(scratch);
  int2* chunks = reinterpret_cast<int2*>(b);
  b += (max_chunks * sizeof(int2) + 255) / 256 * 256;
  int* n_chunks = reinterpret_cast<int*>(b);
  b += 256;
  __half* hbuf = reinterpret_cast<__half*>(b);

  chunk_list_kernel<<<1, 512, 0, st>>>(pm, chunks, n_chunks);
  ++*launches;
  static std::atomic<uint64_t> attr_done{0};  // the kernels' shared memory limit, once per device
  e = once_per_device(attr_done, []() -> cudaError_t {
    cudaError_t r;
    if ((r = cudaFuncSetAttribute(grouped_gemm_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  Layout<0>::bytes)) != cudaSuccess)
      return r;
    if ((r = cudaFuncSetAttribute(grouped_gemm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  Layout<1>::bytes)) != cudaSuccess)
      return r;
    return cudaFuncSetAttribute(grouped_gemm_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                Layout<2>::bytes);
  });
  if (e != cudaSuccess) return e;
  const uint64_t q4_row = uint64_t(H / QK) * Q4K_BYTES;
  CUtensorMap map_x, map_h, map_w, map_ws;
  if ((e = make_tmap_f16(&map_x, xg, P, uint64_t(H))) != cudaSuccess) return e;
  if ((e = make_tmap_f16(&map_h, hbuf, P, uint64_t(F))) != cudaSuccess) return e;
  if ((e = make_tmap_q4k(&map_w, src.slab, q4_row, uint64_t(2 * F), uint64_t(src.n_slots), src.slot_bytes)) !=
      cudaSuccess)
    return e;
  if ((e = make_tmap_q4k(&map_ws, src.shared_gate_up, q4_row, uint64_t(2 * F), 1, q4_row * 2 * F)) != cudaSuccess)
    return e;

  GemmParams gp{};
  gp.src = src;
  gp.layer = layer;
  gp.pm = pm;
  gp.chunks = chunks;
  gp.n_chunks = n_chunks;
  gp.F = F;
  gp.H = H;
  gp.status = status;
  gp.n_mtiles = F / 64;
  gp.out = hbuf;
  grouped_gemm_kernel<0><<<unsigned(num_sms), kThreads, Layout<0>::bytes, st>>>(map_x, map_w, map_ws, gp);
  if (marks) cudaEventRecord(marks[0], st);
  gp.n_mtiles = H / kBM;
  gp.out = y;
  gp.out_rows = out_rows;
  gp.n_routed = n_routed;
  if (src.down_type == kGgmlQ4K)
    grouped_gemm_kernel<2><<<unsigned(num_sms), kThreads, Layout<2>::bytes, st>>>(map_h, map_w, map_ws, gp);
  else
    grouped_gemm_kernel<1><<<unsigned(num_sms), kThreads, Layout<1>::bytes, st>>>(map_h, map_w, map_ws, gp);
  if (marks) cudaEventRecord(marks[1], st);
  *launches += 2;
  return cudaGetLastError();
}

cudaError_t combine_rows(int T, int k, int H, const int32_t* topk_idx, const float* topk_w, const int32_t* rows,
                         const float* shared_s, const __half* y_routed, const __half* y_shared, void* out,
                         int out_dtype, const AddNorm& an, cudaStream_t st, int* launches) {
  if (k != 8 || H % 8) return cudaErrorInvalidValue;
  if (an.h ? (reinterpret_cast<uintptr_t>(an.h) % 16 || reinterpret_cast<uintptr_t>(an.xn) % 16)
           : reinterpret_cast<uintptr_t>(out) % 16)
    return cudaErrorInvalidValue;
  if (T > 0) {
    if (an.h)
      combine_rows_kernel<8, true><<<unsigned(T), 256, 0, st>>>(H, topk_idx, topk_w, rows, shared_s, y_routed,
                                                                y_shared, out, out_dtype, an);
    else
      combine_rows_kernel<8, false><<<unsigned(T), 256, 0, st>>>(H, topk_idx, topk_w, rows, shared_s, y_routed,
                                                                 y_shared, out, out_dtype, an);
    ++*launches;
  }
  return cudaGetLastError();
}

cudaError_t prefill_experts(const ExpertSource& src, int layer, const PairMap& pm, const int32_t* topk_idx, int H,
                            int F, const void* x, int x_dtype, const float* topk_w, const float* shared_s, void* out,
                            int out_dtype, const AddNorm& an, void* scratch, int num_sms, int* status,
                            const cudaEvent_t* marks, cudaStream_t st, int* launches) {
  if (pm.k != 8) return cudaErrorInvalidValue;
  // activations are read and written 16 bytes at a time (out, or the epilogue's rows, checked by combine_rows)
  if (reinterpret_cast<uintptr_t>(x) % 16) return cudaErrorInvalidValue;
  const size_t P = size_t(pm.T) * (pm.k + 1);
  char* b = static_cast<char*>(scratch);
  __half* xg = reinterpret_cast<__half*>(b);
  b += (P * H * sizeof(__half) + 255) / 256 * 256;
  __half* ybuf = reinterpret_cast<__half*>(b);
  b += (P * H * sizeof(__half) + 255) / 256 * 256;
  if (x_dtype == kF32)
    gather_fp16_kernel<float><<<unsigned(P), 256, 0, st>>>(pm, static_cast<const float*>(x), H, xg);
  else
    gather_fp16_kernel<__nv_bfloat16><<<unsigned(P), 256, 0, st>>>(pm, static_cast<const __nv_bfloat16*>(x), H, xg);
  ++*launches;
  if (marks) cudaEventRecord(marks[0], st);
  cudaError_t e = prefill_gemms(src, layer, pm, P, H, F, xg, ybuf, nullptr, 0, b, num_sms, status,
                                marks ? marks + 1 : nullptr, st, launches);
  if (e != cudaSuccess) return e;
  e = combine_rows(pm.T, pm.k, H, topk_idx, topk_w, pm.pos, shared_s, ybuf, ybuf + size_t(pm.T) * pm.k * H, out,
                   out_dtype, an, st, launches);
  if (marks) cudaEventRecord(marks[3], st);
  return e;
}

}  // namespace wmoe
