"""CPU oracle for the ggml expert types beyond Q4_K/Q6_K: a numpy restatement of willow's dequantizers and of the
arithmetic of its Metal GEMV kernels.

TEST INFRASTRUCTURE ONLY. Only tests/ and bench.py's CPU-baseline leg may import this module, and only as the
checker or the timed CPU baseline. The product path (willow_v2_b200) never calls it.

Parity pins: tests/test_ggml_types.py checks every dequantizer here, bit for bit, against golden vectors that
tests/golden/make_golden_types.py produced by running willow's own gguf/quants.py:dequantize (and, for the types it
has, llama.cpp's gguf-py 0.19.0) on the same blocks.

What each function restates (paths within the willow-v2 project):
  dequant_q5_0     gguf/quants.py:35-38    d * (q5 - 16); low nibbles are values 0..15, high nibbles 16..31
  dequant_q8_0     gguf/quants.py:45-47    d * int8
  dequant_iq4_nl   gguf/quants.py:122-124  d * level[nibble]
  dequant_iq4_xs   gguf/quants.py:126-136  (d * (6-bit scale - 32)) * level[nibble], 8 sub-blocks of 32
  dequant_iq3_xxs  gguf/quants.py:154-165  ((d * (0.5 + s4)) * 0.5) * grid * sign (ksigns parity bytes)
  dequant_iq2_s    gguf/quants.py:167-177  ((d * (0.5 + s4)) * 0.25) * grid * sign, 10-bit grid indices
  dequant_iq3_s    gguf/quants.py:179-189  (d * (1 + 2 * s4)) * grid * sign, 9-bit grid indices
  dequant_q2_0     gguf/quants.py:191-195  d * (q2 - 1), blocks of 64
  gemv / gemv_combine_bf16   gguf/metal.py:189-291 (y = W x summed in float32; the combine's bf16 rounding of
                   engines/base.py:431-443 combine_decode_experts)

The IQ codebooks (ggml's iq2s_grid, iq3xxs_grid, iq3s_grid) and IQ4_NL's 16 levels are format tables. They are
read from the installed gguf-py package (llama.cpp's own Python reader), not written out here.
"""
import functools

import numpy as np

from .moe_oracle import QK_K, dequant_q4_k, dequant_q6_k

# (elements per block, bytes per block), the ggml block layouts (gguf/reader.py:14-48)
BLOCKS = {"Q5_0": (32, 22), "Q8_0": (32, 34), "IQ4_NL": (32, 18), "IQ4_XS": (256, 136), "IQ3_XXS": (256, 98),
          "IQ3_S": (256, 110), "IQ2_S": (256, 82), "Q2_0": (64, 18), "Q4_K": (256, 144), "Q6_K": (256, 210)}
TYPES = tuple(BLOCKS)


def _f16(raw: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(raw).view(np.float16).astype(np.float32)


def _nibbles(qs: np.ndarray) -> np.ndarray:
    """[n, 16] bytes -> [n, 32]: low nibbles are values 0..15, high nibbles 16..31 (gguf/quants.py:19-21)."""
    return np.concatenate((qs & 0x0F, qs >> 4), axis=-1)


def _bits(raw: np.ndarray) -> np.ndarray:
    """[n, m] bytes -> [n, 8m] of 0/1, bit i of byte j at position 8j + i."""
    return ((raw[:, :, None] >> np.arange(8, dtype=np.uint8)) & 1).reshape(raw.shape[0], -1)


@functools.cache
def tables():
    """(iq4nl levels [16] f32, iq3xxs grid [256, 4], iq3s grid [512, 4], iq2s grid [1024, 8]) as float32."""
    from gguf import quants
    grids = []
    for cls in (quants.IQ3_XXS, quants.IQ3_S, quants.IQ2_S):
        cls.init_grid()
        grids.append(np.asarray(cls.grid, dtype=np.float32).reshape(cls.grid_shape))
    levels = np.asarray(quants.IQ4_NL.kvalues, dtype=np.float32)
    return (levels, *grids)


def _signs(k: np.ndarray) -> np.ndarray:
    """7-bit ksigns indices -> [.., 8] of +1/-1: the byte i | parity(i) << 7, one sign per bit (ggml ksigns_iq2xs,
    gguf/quants.py:145-148)."""
    k = k.astype(np.int64)
    par = np.zeros_like(k)
    for b in range(7):
        par ^= (k >> b) & 1
    byte = k | (par << 7)
    return (1 - 2 * ((byte[..., None] >> np.arange(8)) & 1)).astype(np.float32)


def dequant_q5_0(b):
    d = _f16(b[:, :2])
    qh = _bits(b[:, 2:6])
    q = _nibbles(b[:, 6:]) | (qh << 4)
    return d * (q.astype(np.float32) - 16)


def dequant_q8_0(b):
    return _f16(b[:, :2]) * np.ascontiguousarray(b[:, 2:]).view(np.int8).astype(np.float32)


def dequant_iq4_nl(b):
    levels = tables()[0]
    return _f16(b[:, :2]) * levels[_nibbles(b[:, 2:])]


def dequant_iq4_xs(b):
    n = b.shape[0]
    levels = tables()[0]
    d = _f16(b[:, :2])
    scales_h = b[:, 2].astype(np.int32) | (b[:, 3].astype(np.int32) << 8)
    high = (scales_h[:, None] >> np.arange(0, 16, 2)) & 3
    low = ((b[:, 4:8, None] >> np.array([0, 4], dtype=np.uint8)) & 0x0F).reshape(n, 8).astype(np.int32)
    dl = d * ((low | (high << 4)) - 32).astype(np.float32)
    q = _nibbles(b[:, 8:].reshape(n * 8, 16)).reshape(n, 8, 32)
    return (dl[:, :, None] * levels[q]).reshape(n, QK_K)


def dequant_iq3_xxs(b):
    n = b.shape[0]
    grid = tables()[1]
    d = _f16(b[:, :2])
    g = grid[b[:, 2:66]].reshape(n, 8, 32)
    aux = np.ascontiguousarray(b[:, 66:98]).view("<u4").astype(np.int64)          # [n, 8]
    db = (d * (np.float32(0.5) + (aux >> 28).astype(np.float32))) * np.float32(0.5)
    sign = _signs((aux[:, :, None] >> np.array([0, 7, 14, 21])) & 0x7F).reshape(n, 8, 32)
    return (db[:, :, None] * g * sign).reshape(n, QK_K)


def dequant_iq2_s(b):
    n = b.shape[0]
    grid = tables()[3]
    d = _f16(b[:, :2])
    qh = ((b[:, 66:74, None] >> np.array([0, 2, 4, 6], dtype=np.uint8)) & 3).reshape(n, 32).astype(np.int64)
    g = grid[b[:, 2:34].astype(np.int64) | (qh << 8)].reshape(n, 16, 16)
    sign = (1 - 2 * _bits(b[:, 34:66]).astype(np.float32)).reshape(n, 16, 16)
    sc = ((b[:, 74:82, None] >> np.array([0, 4], dtype=np.uint8)) & 0x0F).reshape(n, 16).astype(np.float32)
    db = (d * (np.float32(0.5) + sc)) * np.float32(0.25)
    return (db[:, :, None] * g * sign).reshape(n, QK_K)


def dequant_iq3_s(b):
    n = b.shape[0]
    grid = tables()[2]
    d = _f16(b[:, :2])
    qh = _bits(b[:, 66:74]).astype(np.int64)
    g = grid[b[:, 2:66].astype(np.int64) | (qh << 8)].reshape(n, 8, 32)
    sign = (1 - 2 * _bits(b[:, 74:106]).astype(np.float32)).reshape(n, 8, 32)
    sc = ((b[:, 106:110, None] >> np.array([0, 4], dtype=np.uint8)) & 0x0F).reshape(n, 8).astype(np.float32)
    db = d * (1 + 2 * sc)
    return (db[:, :, None] * g * sign).reshape(n, QK_K)


def dequant_q2_0(b):
    q = (b[:, 2:, None] >> np.array([0, 2, 4, 6], dtype=np.uint8)) & 3
    return _f16(b[:, :2]) * (q.reshape(b.shape[0], -1).astype(np.float32) - 1)


DEQUANTIZERS = {"Q5_0": dequant_q5_0, "Q8_0": dequant_q8_0, "IQ4_NL": dequant_iq4_nl, "IQ4_XS": dequant_iq4_xs,
                "IQ3_XXS": dequant_iq3_xxs, "IQ3_S": dequant_iq3_s, "IQ2_S": dequant_iq2_s, "Q2_0": dequant_q2_0,
                "Q4_K": dequant_q4_k, "Q6_K": dequant_q6_k}


def row_bytes(type_name: str, k: int) -> int:
    elements, size = BLOCKS[type_name]
    assert k % elements == 0, (type_name, k)
    return k // elements * size


def dequantize(raw: np.ndarray, type_name: str, shape: tuple) -> np.ndarray:
    """Raw bytes of one tensor -> float32 of shape (gguf/quants.py:207-227)."""
    elements, size = BLOCKS[type_name]
    blocks = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1, size)
    assert blocks.shape[0] * elements == int(np.prod(shape)), (type_name, shape, blocks.shape)
    return DEQUANTIZERS[type_name](blocks).astype(np.float32).reshape(shape)


def bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> the nearest bfloat16 (ties to even), returned as float32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16 << 16
    return u.astype(np.uint32).view(np.float32)


def gemv(raw: np.ndarray, type_name: str, shape: tuple, x: np.ndarray) -> np.ndarray:
    """y [tokens, rows] = x [tokens, k] W^T in float32 (gguf/metal.py:189-215, 311-318)."""
    return x.astype(np.float32) @ dequantize(raw, type_name, shape).T


def gemv_combine_bf16(weights: list, type_name: str, shape: tuple, x: np.ndarray, route_w: np.ndarray,
                      perm: list) -> np.ndarray:
    """sum over i of route_w[perm[i]] * (W_i x[i]) with engines/base.py:431-443's bf16 rounding: p = bf16(W_i x_i),
    bf16(p * w), then a bf16 running total (gguf/metal.py:263-291, 345-355). x bf16-valued [n, k]."""
    total = None
    for i, raw in enumerate(weights):
        p = bf16(dequantize(raw, type_name, shape) @ x[i].astype(np.float32))
        scaled = bf16(p * np.float32(route_w[perm[i]]))
        total = scaled if total is None else bf16(total + scaled)
    return total
