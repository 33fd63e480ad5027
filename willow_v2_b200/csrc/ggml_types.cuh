// The ggml block formats of the typed expert kernels (gguf/metal.py:295 TYPES): per type, the block geometry and a
// decoder of one 32-value chunk to float32 that is bit-identical to willow's dequantizers (gguf/quants.py:27-195).
// Every product and sum the reference rounds separately is written with __fmul_rn / __fadd_rn / __fsub_rn so nvcc
// cannot contract it into an FMA. Sign flips (IQ types) are exact and applied after the rounded product.
//
// Block bytes are read as aligned 16-bit words: every block size and field offset is even, so a 2-byte-aligned
// matrix keeps every read aligned. The IQ codebooks live in shared memory (GgmlTables), filled once per CTA.
#pragma once

#include "common.cuh"
#include "kernels.cuh"

namespace wmoe {

// ggml type ids (GGUF tensor infos, gguf/reader.py:14-48); Q4_K = 12 and Q6_K = 14 are in kernels.cuh
constexpr int kGgmlQ5_0 = 6, kGgmlQ8_0 = 8, kGgmlIQ3XXS = 18, kGgmlIQ4NL = 20, kGgmlIQ3S = 21, kGgmlIQ2S = 22,
              kGgmlIQ4XS = 23, kGgmlQ2_0 = 42;

struct BlockGeom {
  int elements, bytes;
};

// elements and bytes of one block; {0, 0} for a type the typed kernels do not run
__host__ __device__ constexpr BlockGeom block_geom(int type) {
  return type == kGgmlQ5_0    ? BlockGeom{32, 22}
         : type == kGgmlQ8_0  ? BlockGeom{32, 34}
         : type == kGgmlIQ4NL ? BlockGeom{32, 18}
         : type == kGgmlIQ4XS ? BlockGeom{256, 136}
         : type == kGgmlIQ3XXS ? BlockGeom{256, 98}
         : type == kGgmlIQ3S  ? BlockGeom{256, 110}
         : type == kGgmlIQ2S  ? BlockGeom{256, 82}
         : type == kGgmlQ2_0  ? BlockGeom{64, 18}
         : type == kGgmlQ4K   ? BlockGeom{256, 144}
         : type == kGgmlQ6K   ? BlockGeom{256, 210}
                              : BlockGeom{0, 0};
}

// codebook bytes a type needs in shared memory
__host__ __device__ constexpr int table_bytes(int type) {
  return type == kGgmlIQ2S ? 1024 * 8 : type == kGgmlIQ3S ? 512 * 4 : type == kGgmlIQ3XXS ? 256 * 4
         : (type == kGgmlIQ4NL || type == kGgmlIQ4XS) ? 16 * 4 : 0;
}

struct GgmlTables {
  const float* levels;       // IQ4_NL / IQ4_XS: the 16 levels
  const uint32_t* grid32;    // IQ3_XXS [256] / IQ3_S [512]: 4 values per entry, one per byte
  const uint2* grid64;       // IQ2_S [1024]: 8 values per entry
};

__device__ __forceinline__ uint32_t rd16(const uint8_t* p, int i) {
  return *reinterpret_cast<const uint16_t*>(p + i);
}
__device__ __forceinline__ uint32_t rd32(const uint8_t* p, int i) { return rd16(p, i) | (rd16(p, i + 2) << 16); }
__device__ __forceinline__ float half_at(const uint8_t* p, int i) { return f16_to_f32(uint16_t(rd16(p, i))); }
__device__ __forceinline__ float signed_by(float v, uint32_t bit) { return bit ? -v : v; }

// ggml's ksigns_iq2xs byte for a 7-bit index: the 7 bits plus an eighth that makes the parity even
__device__ __forceinline__ uint32_t ksigns(uint32_t i) { return i | ((__popc(i) & 1u) << 7); }

// Decodes values 32*c .. 32*c+31 of the block at blk (c < elements / 32) into v.
template <int T>
__device__ __forceinline__ void decode_chunk(const uint8_t* blk, int c, const GgmlTables& tb, float (&v)[32]);

template <>  // gguf/quants.py:35-38
__device__ __forceinline__ void decode_chunk<kGgmlQ5_0>(const uint8_t* b, int, const GgmlTables&, float (&v)[32]) {
  const float d = half_at(b, 0);
  const uint32_t qh = rd32(b, 2);
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    const uint32_t two = rd16(b, 6 + 2 * w);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int j = 2 * w + h;
      const uint32_t q = (two >> (8 * h)) & 0xFF;
      v[j] = __fmul_rn(d, float(int((q & 0xF) | (((qh >> j) & 1) << 4)) - 16));
      v[j + 16] = __fmul_rn(d, float(int((q >> 4) | (((qh >> (j + 16)) & 1) << 4)) - 16));
    }
  }
}

template <>  // gguf/quants.py:45-47
__device__ __forceinline__ void decode_chunk<kGgmlQ8_0>(const uint8_t* b, int, const GgmlTables&, float (&v)[32]) {
  const float d = half_at(b, 0);
#pragma unroll
  for (int w = 0; w < 16; ++w) {
    const uint32_t two = rd16(b, 2 + 2 * w);
    v[2 * w] = __fmul_rn(d, float(int8_t(two & 0xFF)));
    v[2 * w + 1] = __fmul_rn(d, float(int8_t(two >> 8)));
  }
}

template <>  // gguf/quants.py:122-124
__device__ __forceinline__ void decode_chunk<kGgmlIQ4NL>(const uint8_t* b, int, const GgmlTables& tb,
                                                        float (&v)[32]) {
  const float d = half_at(b, 0);
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    const uint32_t two = rd16(b, 2 + 2 * w);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t q = (two >> (8 * h)) & 0xFF;
      v[2 * w + h] = __fmul_rn(d, tb.levels[q & 0xF]);
      v[2 * w + h + 16] = __fmul_rn(d, tb.levels[q >> 4]);
    }
  }
}

template <>  // gguf/quants.py:126-136: sub-block c of 32, scale (low | high << 4) - 32
__device__ __forceinline__ void decode_chunk<kGgmlIQ4XS>(const uint8_t* b, int c, const GgmlTables& tb,
                                                        float (&v)[32]) {
  const float d = half_at(b, 0);
  const uint32_t high = (rd16(b, 2) >> (2 * c)) & 3;
  const uint32_t low = (rd16(b, 4 + 2 * (c / 4)) >> (4 * (c % 4))) & 0xF;  // scales_l[c / 2], nibble c % 2
  const float dl = __fmul_rn(d, float(int(low | (high << 4)) - 32));
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    const uint32_t two = rd16(b, 8 + 16 * c + 2 * w);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t q = (two >> (8 * h)) & 0xFF;
      v[2 * w + h] = __fmul_rn(dl, tb.levels[q & 0xF]);
      v[2 * w + h + 16] = __fmul_rn(dl, tb.levels[q >> 4]);
    }
  }
}

template <>  // gguf/quants.py:154-165: 8 grid indices of 4 values, then a u32 of 4-bit scale + 4 x 7-bit signs
__device__ __forceinline__ void decode_chunk<kGgmlIQ3XXS>(const uint8_t* b, int c, const GgmlTables& tb,
                                                         float (&v)[32]) {
  const float d = half_at(b, 0);
  const uint32_t aux = rd32(b, 66 + 4 * c);
  const float db = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, float(aux >> 28))), 0.5f);
#pragma unroll
  for (int l = 0; l < 4; ++l) {
    const uint32_t two = rd16(b, 2 + 8 * c + 2 * l);  // grid indices 2l, 2l + 1 of the chunk
    const uint32_t s = ksigns((aux >> (7 * l)) & 0x7F);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t g = tb.grid32[(two >> (8 * h)) & 0xFF];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int j = 4 * h + i;  // value j of the 8-value sign group l
        v[8 * l + j] = signed_by(__fmul_rn(db, float((g >> (8 * i)) & 0xFF)), (s >> j) & 1);
      }
    }
  }
}

template <>  // gguf/quants.py:167-177: 4 grid entries of 8 values (10-bit indices), explicit signs, 2 scales
__device__ __forceinline__ void decode_chunk<kGgmlIQ2S>(const uint8_t* b, int c, const GgmlTables& tb,
                                                       float (&v)[32]) {
  const float d = half_at(b, 0);
  const uint32_t qs = rd32(b, 2 + 4 * c);       // low index bytes of entries 4c .. 4c+3
  const uint32_t sg = rd32(b, 34 + 4 * c);      // their sign bytes
  const uint32_t qh = (rd16(b, 66 + 2 * (c / 2)) >> (8 * (c % 2))) & 0xFF;
  const uint32_t sc = (rd16(b, 74 + 2 * (c / 2)) >> (8 * (c % 2))) & 0xFF;
  float db[2];
#pragma unroll
  for (int h = 0; h < 2; ++h)
    db[h] = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, float((sc >> (4 * h)) & 0xF))), 0.25f);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const uint32_t idx = ((qs >> (8 * e)) & 0xFF) | (((qh >> (2 * e)) & 3) << 8);
    const uint2 g = tb.grid64[idx];
    const uint32_t s = (sg >> (8 * e)) & 0xFF;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t gv = ((j < 4 ? g.x : g.y) >> (8 * (j % 4))) & 0xFF;
      v[8 * e + j] = signed_by(__fmul_rn(db[e / 2], float(gv)), (s >> j) & 1);
    }
  }
}

template <>  // gguf/quants.py:179-189: 8 grid entries of 4 values (9-bit indices), explicit signs, one scale
__device__ __forceinline__ void decode_chunk<kGgmlIQ3S>(const uint8_t* b, int c, const GgmlTables& tb,
                                                       float (&v)[32]) {
  const float d = half_at(b, 0);
  const uint32_t qh = (rd16(b, 66 + 2 * (c / 2)) >> (8 * (c % 2))) & 0xFF;
  const uint32_t sg = rd32(b, 74 + 4 * c);      // 32 sign bits, one per value
  const uint32_t sc = (rd16(b, 106 + 2 * (c / 4)) >> (4 * (c % 4))) & 0xF;  // byte c / 2, nibble c % 2
  const float db = __fmul_rn(d, float(1 + 2 * int(sc)));
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const uint32_t two = rd16(b, 2 + 8 * c + 2 * w);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int e = 2 * w + h;
      const uint32_t g = tb.grid32[((two >> (8 * h)) & 0xFF) | (((qh >> e) & 1) << 8)];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int j = 4 * e + i;
        v[j] = signed_by(__fmul_rn(db, float((g >> (8 * i)) & 0xFF)), (sg >> j) & 1);
      }
    }
  }
}

template <>  // gguf/quants.py:191-195: blocks of 64, value j = bits 2 (j % 4) of byte j / 4, 0..3 -> -1..+2
__device__ __forceinline__ void decode_chunk<kGgmlQ2_0>(const uint8_t* b, int c, const GgmlTables&, float (&v)[32]) {
  const float d = half_at(b, 0);
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const uint32_t two = rd16(b, 2 + 8 * c + 2 * w);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[8 * w + i] = __fmul_rn(d, float(int((two >> (2 * i)) & 3) - 1));
  }
}

template <>  // gguf/quants.py:73-92: sub-block c = (d * sc) * q - (dmin * mn)
__device__ __forceinline__ void decode_chunk<kGgmlQ4K>(const uint8_t* b, int c, const GgmlTables&, float (&v)[32]) {
  const float d = half_at(b, 0), dmin = half_at(b, 2);
  uint8_t s12[12];
#pragma unroll
  for (int w = 0; w < 6; ++w) {
    const uint32_t two = rd16(b, 4 + 2 * w);
    s12[2 * w] = uint8_t(two);
    s12[2 * w + 1] = uint8_t(two >> 8);
  }
  int sc, mn;
  q4k_scale_min(s12, c, sc, mn);
  const float scale = __fmul_rn(d, float(sc)), m = __fmul_rn(dmin, float(mn));
  const int shift = 4 * (c % 2);
#pragma unroll
  for (int w = 0; w < 16; ++w) {
    const uint32_t two = rd16(b, 16 + 32 * (c / 2) + 2 * w);
    v[2 * w] = __fsub_rn(__fmul_rn(scale, float((two >> shift) & 0xF)), m);
    v[2 * w + 1] = __fsub_rn(__fmul_rn(scale, float((two >> (8 + shift)) & 0xF)), m);
  }
}

template <>  // gguf/quants.py:104-116: (d * sc_i8) * (q6 - 32), one scale per 16 values
__device__ __forceinline__ void decode_chunk<kGgmlQ6K>(const uint8_t* b, int c, const GgmlTables&, float (&v)[32]) {
  const float d = half_at(b, 208);
  const uint32_t sc2 = rd16(b, 192 + 2 * c);
  const float s0 = __fmul_rn(d, float(int8_t(sc2 & 0xFF))), s1 = __fmul_rn(d, float(int8_t(sc2 >> 8)));
  const int h = c / 4, s = c % 4, lshift = 4 * (s / 2), hshift = 2 * s;
#pragma unroll
  for (int w = 0; w < 16; ++w) {
    const uint32_t lo = rd16(b, 64 * h + 32 * (s % 2) + 2 * w), hi = rd16(b, 128 + 32 * h + 2 * w);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int l = 2 * w + i;
      const int q = int(((lo >> (8 * i + lshift)) & 0xF) | (((hi >> (8 * i + hshift)) & 3) << 4)) - 32;
      v[l] = __fmul_rn(l < 16 ? s0 : s1, float(q));
    }
  }
}

// ------------------------------------------------------------------------------------------------ integer form
// The typed GEMV kernels take a chunk as 8 words of 4 signed int8 weights (word i = values 4i .. 4i+3) and its
// scales: chunk . x = xs * (s0 * acc0 + s1 * acc1 - m0 * xsum0 - m1 * xsum1), where x ~ xs * xq (int16, one
// power-of-two scale per 32 values), acc0 / acc1 = the integer dot products of words 0-3 / 4-7 with xq, and
// xsum0 / xsum1 = the sums of xq over values 0-15 / 16-31 (offsets and mins: Q5_0 q - 16, Q2_0 q - 1, Q6_K q - 32,
// Q4_K's dmin * mn). Products of small integers are exact, so the only differences from the float path are the
// rounding of x to int16 (exact for bf16 values within 2^7 of their block's maximum) and the summation order.

struct ChunkScale {
  float s0, s1, m0, m1;
};

struct IntTables {
  uint32_t lv0, lv1, lv2, lv3;  // IQ4_NL / IQ4_XS: the 16 int8 levels, 4 per word
  const uint32_t* grid32;       // IQ3_XXS / IQ3_S
  const uint2* grid64;          // IQ2_S
};

__device__ __forceinline__ int dp2a_lo_s(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp2a.lo.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp2a_hi_s(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp2a.hi.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// bit i of a 4-bit value -> byte i of the result (0 or 1)
__device__ __forceinline__ uint32_t spread4(uint32_t b) { return (b * 0x00204081u) & 0x01010101u; }

// bytes of g (each 1..127) negated where the matching bit of the 4-bit s is set: (g ^ 0xFF) + 1 per byte, which
// carries into no neighbour because no byte is 0
__device__ __forceinline__ uint32_t with_signs(uint32_t g, uint32_t s) {
  const uint32_t one = spread4(s);
  return (g ^ (one * 0xFFu)) + one;
}

// the IQ4 level of each of 4 nibbles (one per byte of nb) as int8 bytes, by byte permutes of the 16-level table
__device__ __forceinline__ uint32_t iq4_levels(uint32_t nb, const IntTables& it) {
  const uint32_t t = nb | (nb >> 4);
  const uint32_t sel = __byte_perm(t, 0, 0x4420);  // n0 | n1 << 4 | n2 << 8 | n3 << 12
  const uint32_t lo = __byte_perm(it.lv0, it.lv1, sel & 0x7777), hi = __byte_perm(it.lv2, it.lv3, sel & 0x7777);
  const uint32_t m = spread4((nb >> 3) & 1 | (nb >> 10) & 2 | (nb >> 17) & 4 | (nb >> 24) & 8) * 0xFFu;
  return (lo & ~m) | (hi & m);
}

template <int T>
__device__ __forceinline__ void int_words(const uint8_t* b, int c, const IntTables& it, uint32_t (&w)[8],
                                          ChunkScale& cs);

template <>
__device__ __forceinline__ void int_words<kGgmlQ5_0>(const uint8_t* b, int, const IntTables&, uint32_t (&w)[8],
                                                     ChunkScale& cs) {
  const float d = half_at(b, 0);
  const uint32_t qh = rd32(b, 2);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t q = rd32(b, 6 + 4 * i);
    w[i] = (q & 0x0F0F0F0Fu) | (spread4((qh >> (4 * i)) & 0xF) << 4);
    w[i + 4] = ((q >> 4) & 0x0F0F0F0Fu) | (spread4((qh >> (16 + 4 * i)) & 0xF) << 4);
  }
  cs = {d, d, 16.f * d, 16.f * d};
}

template <>
__device__ __forceinline__ void int_words<kGgmlQ8_0>(const uint8_t* b, int, const IntTables&, uint32_t (&w)[8],
                                                     ChunkScale& cs) {
  const float d = half_at(b, 0);
#pragma unroll
  for (int i = 0; i < 8; ++i) w[i] = rd32(b, 2 + 4 * i);
  cs = {d, d, 0.f, 0.f};
}

template <>
__device__ __forceinline__ void int_words<kGgmlIQ4NL>(const uint8_t* b, int, const IntTables& it, uint32_t (&w)[8],
                                                      ChunkScale& cs) {
  const float d = half_at(b, 0);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t q = rd32(b, 2 + 4 * i);
    w[i] = iq4_levels(q & 0x0F0F0F0Fu, it);
    w[i + 4] = iq4_levels((q >> 4) & 0x0F0F0F0Fu, it);
  }
  cs = {d, d, 0.f, 0.f};
}

template <>
__device__ __forceinline__ void int_words<kGgmlIQ4XS>(const uint8_t* b, int c, const IntTables& it, uint32_t (&w)[8],
                                                      ChunkScale& cs) {
  const float d = half_at(b, 0);
  const uint32_t high = (rd16(b, 2) >> (2 * c)) & 3;
  const uint32_t low = (rd16(b, 4 + 2 * (c / 4)) >> (4 * (c % 4))) & 0xF;
  const float dl = __fmul_rn(d, float(int(low | (high << 4)) - 32));
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t q = rd32(b, 8 + 16 * c + 4 * i);
    w[i] = iq4_levels(q & 0x0F0F0F0Fu, it);
    w[i + 4] = iq4_levels((q >> 4) & 0x0F0F0F0Fu, it);
  }
  cs = {dl, dl, 0.f, 0.f};
}

template <>
__device__ __forceinline__ void int_words<kGgmlIQ3XXS>(const uint8_t* b, int c, const IntTables& it,
                                                       uint32_t (&w)[8], ChunkScale& cs) {
  const float d = half_at(b, 0);
  const uint32_t aux = rd32(b, 66 + 4 * c);
  const float db = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, float(aux >> 28))), 0.5f);
#pragma unroll
  for (int l = 0; l < 4; ++l) {
    const uint32_t two = rd16(b, 2 + 8 * c + 2 * l);
    const uint32_t s = ksigns((aux >> (7 * l)) & 0x7F);
    w[2 * l] = with_signs(it.grid32[two & 0xFF], s & 0xF);
    w[2 * l + 1] = with_signs(it.grid32[two >> 8], s >> 4);
  }
  cs = {db, db, 0.f, 0.f};
}

template <>
__device__ __forceinline__ void int_words<kGgmlIQ2S>(const uint8_t* b, int c, const IntTables& it, uint32_t (&w)[8],
                                                     ChunkScale& cs) {
  const float d = half_at(b, 0);
  const uint32_t qs = rd32(b, 2 + 4 * c), sg = rd32(b, 34 + 4 * c);
  const uint32_t qh = (rd16(b, 66 + 2 * (c / 2)) >> (8 * (c % 2))) & 0xFF;
  const uint32_t sc = (rd16(b, 74 + 2 * (c / 2)) >> (8 * (c % 2))) & 0xFF;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const uint2 g = it.grid64[((qs >> (8 * e)) & 0xFF) | (((qh >> (2 * e)) & 3) << 8)];
    const uint32_t s = (sg >> (8 * e)) & 0xFF;
    w[2 * e] = with_signs(g.x, s & 0xF);
    w[2 * e + 1] = with_signs(g.y, s >> 4);
  }
  const float db0 = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, float(sc & 0xF))), 0.25f);
  const float db1 = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, float(sc >> 4))), 0.25f);
  cs = {db0, db1, 0.f, 0.f};
}

template <>
__device__ __forceinline__ void int_words<kGgmlIQ3S>(const uint8_t* b, int c, const IntTables& it, uint32_t (&w)[8],
                                                     ChunkScale& cs) {
  const float d = half_at(b, 0);
  const uint32_t qh = (rd16(b, 66 + 2 * (c / 2)) >> (8 * (c % 2))) & 0xFF;
  const uint32_t sg = rd32(b, 74 + 4 * c);
  const uint32_t sc = (rd16(b, 106 + 2 * (c / 4)) >> (4 * (c % 4))) & 0xF;
  const float db = __fmul_rn(d, float(1 + 2 * int(sc)));
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t two = rd16(b, 2 + 8 * c + 2 * i);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int e = 2 * i + h;
      const uint32_t g = it.grid32[((two >> (8 * h)) & 0xFF) | (((qh >> e) & 1) << 8)];
      w[e] = with_signs(g, (sg >> (4 * e)) & 0xF);
    }
  }
  cs = {db, db, 0.f, 0.f};
}

template <>
__device__ __forceinline__ void int_words<kGgmlQ2_0>(const uint8_t* b, int c, const IntTables&, uint32_t (&w)[8],
                                                     ChunkScale& cs) {
  const float d = half_at(b, 0);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t q = rd32(b, 2 + 8 * c + 4 * h);  // values 16h .. 16h+15, 2 bits each
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const uint32_t y = (q >> (8 * m)) & 0xFF;   // values 4m .. 4m+3 of this half
      w[4 * h + m] = (y & 3) | ((y & 0xC) << 6) | ((y & 0x30) << 12) | ((y & 0xC0) << 18);
    }
  }
  cs = {d, d, d, d};
}

template <>
__device__ __forceinline__ void int_words<kGgmlQ4K>(const uint8_t* b, int c, const IntTables&, uint32_t (&w)[8],
                                                    ChunkScale& cs) {
  const float d = half_at(b, 0), dmin = half_at(b, 2);
  uint8_t s12[12];
#pragma unroll
  for (int i = 0; i < 6; ++i) {
    const uint32_t two = rd16(b, 4 + 2 * i);
    s12[2 * i] = uint8_t(two);
    s12[2 * i + 1] = uint8_t(two >> 8);
  }
  int sc, mn;
  q4k_scale_min(s12, c, sc, mn);
  const float scale = __fmul_rn(d, float(sc)), m = __fmul_rn(dmin, float(mn));
  const int shift = 4 * (c % 2);
#pragma unroll
  for (int i = 0; i < 8; ++i) w[i] = (rd32(b, 16 + 32 * (c / 2) + 4 * i) >> shift) & 0x0F0F0F0Fu;
  cs = {scale, scale, m, m};
}

template <>
__device__ __forceinline__ void int_words<kGgmlQ6K>(const uint8_t* b, int c, const IntTables&, uint32_t (&w)[8],
                                                    ChunkScale& cs) {
  const float d = half_at(b, 208);
  const uint32_t sc2 = rd16(b, 192 + 2 * c);
  const float s0 = __fmul_rn(d, float(int8_t(sc2 & 0xFF))), s1 = __fmul_rn(d, float(int8_t(sc2 >> 8)));
  const int h = c / 4, s = c % 4, lshift = 4 * (s / 2), hshift = 2 * s;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t lo = rd32(b, 64 * h + 32 * (s % 2) + 4 * i), hi = rd32(b, 128 + 32 * h + 4 * i);
    w[i] = ((lo >> lshift) & 0x0F0F0F0Fu) | (((hi >> hshift) & 0x03030303u) << 4);
  }
  cs = {s0, s1, 32.f * s0, 32.f * s1};
}

template <int T>
__device__ __forceinline__ void int_row_words(const uint8_t* row, int c, const IntTables& it, uint32_t (&w)[8],
                                              ChunkScale& cs) {
  constexpr BlockGeom g = block_geom(T);
  constexpr int per = g.elements / 32;
  int_words<T>(row + (c / per) * g.bytes, c % per, it, w, cs);
}

// chunk . x for one token: xw = the chunk's 32 int16 activations as 16 words, xs their scale, xsum0 / xsum1 the
// sums of values 0-15 / 16-31
__device__ __forceinline__ float chunk_apply(const uint32_t (&w)[8], const ChunkScale& cs, const uint32_t (&xw)[16],
                                             float xs, int xsum0, int xsum1) {
  int a0 = 0, a1 = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    a0 = dp2a_lo_s(xw[2 * i], w[i], a0);
    a0 = dp2a_hi_s(xw[2 * i + 1], w[i], a0);
    a1 = dp2a_lo_s(xw[8 + 2 * i], w[4 + i], a1);
    a1 = dp2a_hi_s(xw[8 + 2 * i + 1], w[4 + i], a1);
  }
  const float t = cs.s0 * float(a0) + cs.s1 * float(a1) - cs.m0 * float(xsum0) - cs.m1 * float(xsum1);
  return xs * t;
}

// Value chunk c of a row (32 values each) for any block size: block c / (elements / 32), chunk within it.
template <int T>
__device__ __forceinline__ void decode_row_chunk(const uint8_t* row, int c, const GgmlTables& tb, float (&v)[32]) {
  constexpr BlockGeom g = block_geom(T);
  constexpr int per = g.elements / 32;
  decode_chunk<T>(row + (c / per) * g.bytes, c % per, tb, v);
}

}  // namespace wmoe
