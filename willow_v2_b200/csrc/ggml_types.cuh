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

// Value chunk c of a row (32 values each) for any block size: block c / (elements / 32), chunk within it.
template <int T>
__device__ __forceinline__ void decode_row_chunk(const uint8_t* row, int c, const GgmlTables& tb, float (&v)[32]) {
  constexpr BlockGeom g = block_geom(T);
  constexpr int per = g.elements / 32;
  decode_chunk<T>(row + (c / per) * g.bytes, c % per, tb, v);
}

}  // namespace wmoe
