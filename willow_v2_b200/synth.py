"""Seeded synthetic inputs for the qwen35moe MoE block, with the value distributions of the benchmark configs.

Expert weights are GGUF super-blocks whose bytes come from a counter-based hash (splitmix64 over a key derived
from (seed, layer, expert, tensor) and the word index), so the same bytes can be produced on the host (this
module, numpy) and on the GPU (``csrc/synth.cuh``, used by ``wmoe_store_fill_synthetic``) without moving the
~21 GB of a 40-layer store. Both sides use only integer arithmetic plus two correctly rounded float64 operations
and a round-to-nearest-even float64 -> fp16 conversion, so they agree bit for bit.

Block contents (ggml layouts, gguf/reader.py:14-48 for the sizes):
  Q4_K (144 B): bytes 0-1 d, 2-3 dmin = fp16(U[1e-3, 4e-3]); bytes 4-143 (12 scale bytes, 128 quant bytes)
                uniform random.
  Q6_K (210 B): bytes 0-191 (ql, qh) uniform random; bytes 192-207 int8 scales uniform in [-32, 31];
                bytes 208-209 d = fp16(U[1e-3, 4e-3]).
An expert is stored as one blob, gate_up (Q4_K, [2F, H], gate rows then up rows, as gguf/compiler.py:69-88
fuses them) followed by down (Q6_K, [H, F]); the shared expert uses the same layout at expert index E.

The small fp32 tensors (router, shared-expert gate vector, hidden states, Zipf bias) come from numpy's PCG64
generator and are uploaded; they are a few MB per layer.
"""
import numpy as np

# qwen35moe (Qwen3.6-35B-A3B) MoE shapes
HIDDEN = 2048
FFN = 512
EXPERTS = 256
TOP_K = 8
QK_K = 256
Q4K_BYTES = 144
Q6K_BYTES = 210
GATE_UP_BYTES = 2 * FFN * HIDDEN // QK_K * Q4K_BYTES    # 1,179,648
DOWN_BYTES = HIDDEN * FFN // QK_K * Q6K_BYTES            # 860,160
EXPERT_BYTES = GATE_UP_BYTES + DOWN_BYTES                 # 2,039,808

TENSOR_GATE_UP = 0
TENSOR_DOWN = 1
WORDS_PER_BLOCK = 32  # hash words reserved per super-block (Q4_K uses 20, Q6_K 27)

_GAMMA = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)
_D_STEP = 3e-3 / 16777216.0  # U[1e-3, 4e-3] from a 24-bit integer


def _finalize(z: np.ndarray) -> np.ndarray:
    z = (z ^ (z >> np.uint64(30))) * _M1
    z = (z ^ (z >> np.uint64(27))) * _M2
    return z ^ (z >> np.uint64(31))


def _mix(z: int) -> int:
    """splitmix64 step on one value: finalize(z + gamma)."""
    with np.errstate(over="ignore"):
        return int(_finalize(np.array([z], dtype=np.uint64) + _GAMMA)[0])


def tensor_key(seed: int, layer: int, expert: int, tensor: int) -> int:
    m = (1 << 64) - 1
    k = _mix(seed & m)
    k = _mix((k + layer) & m)
    return _mix((k + 2 * expert + tensor) & m)


def _words(key: int, nblocks: int, nwords: int, first_block: int = 0) -> np.ndarray:
    """[nblocks, nwords] uint64: word k of block b is finalize(key + (b * 32 + k + 1) * gamma)."""
    idx = (np.arange(first_block, first_block + nblocks, dtype=np.uint64)[:, None] * np.uint64(WORDS_PER_BLOCK)
           + np.arange(nwords, dtype=np.uint64)[None, :] + np.uint64(1))
    with np.errstate(over="ignore"):
        return _finalize(np.uint64(key) + idx * _GAMMA)


def _fp16_scale(words: np.ndarray) -> np.ndarray:
    """uint64 words -> fp16 bit patterns of 1e-3 + 3e-3 * (top 24 bits / 2^24), rounded to nearest even."""
    u = (words >> np.uint64(40)).astype(np.float64)
    v = u * _D_STEP + 1e-3  # one multiply, one add, each correctly rounded (no fused multiply-add in numpy)
    return v.astype(np.float16).view(np.uint16)


def q4k_blocks(key: int, nblocks: int, first_block: int = 0) -> np.ndarray:
    w = _words(key, nblocks, 20, first_block)
    out = np.ascontiguousarray(w[:, :18]).view(np.uint8).reshape(nblocks, Q4K_BYTES).copy()
    out[:, 0:2] = _fp16_scale(w[:, 18])[:, None].view(np.uint8)
    out[:, 2:4] = _fp16_scale(w[:, 19])[:, None].view(np.uint8)
    return out


def q6k_blocks(key: int, nblocks: int, first_block: int = 0) -> np.ndarray:
    w = _words(key, nblocks, 27, first_block)
    out = np.empty((nblocks, Q6K_BYTES), dtype=np.uint8)
    out[:, 0:192] = np.ascontiguousarray(w[:, :24]).view(np.uint8).reshape(nblocks, 192)
    sc = np.ascontiguousarray(w[:, 24:26]).view(np.uint8).reshape(nblocks, 16)
    out[:, 192:208] = ((sc & 63).astype(np.int16) - 32).astype(np.int8).view(np.uint8)
    out[:, 208:210] = _fp16_scale(w[:, 26])[:, None].view(np.uint8)
    return out


def expert_gate_up(seed: int, layer: int, expert: int, rows=None) -> np.ndarray:
    """Q4_K bytes of an expert's fused [gate | up] weight, [2F rows, H]: uint8 [rows, 1152].
    rows: an optional (start, stop) row range."""
    r0, r1 = rows or (0, 2 * FFN)
    per_row = HIDDEN // QK_K
    b = q4k_blocks(tensor_key(seed, layer, expert, TENSOR_GATE_UP), (r1 - r0) * per_row, r0 * per_row)
    return b.reshape(r1 - r0, per_row * Q4K_BYTES)


def expert_down(seed: int, layer: int, expert: int, rows=None) -> np.ndarray:
    """Q6_K bytes of an expert's down weight, [H rows, F]: uint8 [rows, 420]."""
    r0, r1 = rows or (0, HIDDEN)
    per_row = FFN // QK_K
    b = q6k_blocks(tensor_key(seed, layer, expert, TENSOR_DOWN), (r1 - r0) * per_row, r0 * per_row)
    return b.reshape(r1 - r0, per_row * Q6K_BYTES)


def expert_blob(seed: int, layer: int, expert: int) -> np.ndarray:
    """The expert's bytes as the store holds them: gate_up then down, uint8 [EXPERT_BYTES]."""
    return np.concatenate((expert_gate_up(seed, layer, expert).reshape(-1),
                           expert_down(seed, layer, expert).reshape(-1)))


def _rng(*key) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(list(key)))


def router_weight(seed: int, layer: int) -> np.ndarray:
    """fp32 [E, H] drawn N(0, 0.02)."""
    return _rng(seed, layer, 1).standard_normal((EXPERTS, HIDDEN), dtype=np.float32) * np.float32(0.02)


def shared_gate_weight(seed: int, layer: int) -> np.ndarray:
    """fp32 [H]: the shared expert's sigmoid gate vector, drawn N(0, 0.02)."""
    return _rng(seed, layer, 2).standard_normal(HIDDEN, dtype=np.float32) * np.float32(0.02)


def hidden(seed: int, tokens: int, step: int = 0) -> np.ndarray:
    """fp32 [tokens, H] drawn N(0, 1). step picks an independent draw (one per benchmark step)."""
    return _rng(seed, step, 3, tokens).standard_normal((tokens, HIDDEN), dtype=np.float32)


def zipf_bias(seed: int, s: float = 1.1) -> np.ndarray:
    """fp32 [E]: -s * ln(rank_e), rank = 1 + a seeded permutation of 0..E-1, added to the router logits to skew
    routing towards a few experts (a Zipf(s) popularity law)."""
    rank = 1 + _rng(seed, 4).permutation(EXPERTS)
    return (-s * np.log(rank.astype(np.float64))).astype(np.float32)
