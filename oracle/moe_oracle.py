"""CPU oracle for the qwen35moe MoE block: a numpy restatement of willow's own CPU path.

TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import this
module, and only as the checker or the timed CPU baseline. The product path (willow_v2_b200) never calls it.

Parity pins: tests/test_oracle.py checks every function here against golden vectors that
tests/golden/make_golden.py produced by running willow itself (gguf/quants.py, engines/base.py imported from
the reference checkout) and llama.cpp's gguf-py 0.19.0, on the same seeded synthetic blocks.

What each function restates (paths within the willow-v2 project):
  dequant_q4_k   gguf/quants.py:73-92   (_k_scale_min, _q4_k_parts, dequant_q4_k)
  dequant_q6_k   gguf/quants.py:104-116 (_q6_k_parts, dequant_q6_k)
  route          engines/base.py:91-97  (route; norm_topk_prob=True per engines/qwen36/model.py:41)
  expert_gate    engines/base.py:99-102
  shared_expert  engines/base.py:104-107 (shared_expert_gate.weight [1, H], engines/qwen36/loader.py:127-128)
  moe            engines/base.py:445-490 with each_expert's sum, base.py:534-591 (experts added in ascending id
                 order with index_add_, then the shared expert)
  skip_small_experts  engines/base.py:413-429 (min_expert_weight; dropped picks become -1)
  rms_norm       engines/base.py:27-32 (zero-centred, weight 0 -> scale 1) and the residual wiring of
                 engines/qwen36/model.py:17-22
"""
import numpy as np

QK_K = 256


def _f16(raw: np.ndarray) -> np.ndarray:
    """[n, 2] bytes -> [n, 1] float32 (gguf/quants.py:12-14)."""
    return np.ascontiguousarray(raw).view(np.float16).astype(np.float32)


def _k_scale_min(scales: np.ndarray):
    """Q4_K: 12 bytes -> 8 six-bit scales and 8 six-bit mins (gguf/quants.py:73-80)."""
    n = scales.shape[0]
    s = scales.reshape(n, 3, 4)
    d, m, m_d = s[:, 0], s[:, 1], s[:, 2]
    sc = np.concatenate((d & 0x3F, (m_d & 0x0F) | ((d >> 2) & 0x30)), axis=-1)
    mn = np.concatenate((m & 0x3F, (m_d >> 4) | ((m >> 2) & 0x30)), axis=-1)
    return sc.astype(np.float32), mn.astype(np.float32)


def dequant_q4_k(b: np.ndarray) -> np.ndarray:
    """uint8 [n, 144] -> float32 [n, 256] (gguf/quants.py:82-92). Sub-block j = (d * sc_j) * q - (dmin * mn_j),
    each product and the difference rounded to float32 separately; nibble group g holds sub-block 2g in its low
    nibbles and 2g + 1 in its high nibbles."""
    n = b.shape[0]
    d, dmin = _f16(b[:, 0:2]), _f16(b[:, 2:4])
    sc, mn = _k_scale_min(b[:, 4:16])
    scale, mins = d * sc, dmin * mn
    q = ((b[:, 16:].reshape(n, 4, 1, 32) >> np.array([0, 4], dtype=np.uint8).reshape(1, 1, 2, 1)) & 0x0F)
    q = q.reshape(n, 8, 32).astype(np.float32)
    return (scale[..., None] * q - mins[..., None]).reshape(n, QK_K)


def dequant_q6_k(b: np.ndarray) -> np.ndarray:
    """uint8 [n, 210] -> float32 [n, 256] (gguf/quants.py:104-116). Value = (d * sc_i8) * (q6 - 32) with one scale
    per 16 values; half h uses ql[64h:64h+64] (low nibbles, then high) and qh[32h:32h+32] (2-bit fields)."""
    n = b.shape[0]
    ql, qh = b[:, :128], b[:, 128:192]
    scales = _f16(b[:, 208:210]) * np.ascontiguousarray(b[:, 192:208]).view(np.int8).astype(np.float32)
    ql = ((ql.reshape(n, 2, 1, 64) >> np.array([0, 4], dtype=np.uint8).reshape(1, 1, 2, 1)) & 0x0F).reshape(n, 8, 32)
    qh = ((qh.reshape(n, 2, 1, 32) >> np.array([0, 2, 4, 6], dtype=np.uint8).reshape(1, 1, 4, 1)) & 3).reshape(n, 8, 32)
    q = (ql | (qh << 4)).astype(np.int8) - np.int8(32)
    return (scales[..., None] * q.reshape(n, 16, 16).astype(np.float32)).reshape(n, QK_K)


def dequantize(raw: np.ndarray, type_name: str, shape: tuple) -> np.ndarray:
    """Raw bytes of one tensor -> float32 of shape (gguf/quants.py:207-227, Q4_K and Q6_K only)."""
    fn, block = {"Q4_K": (dequant_q4_k, 144), "Q6_K": (dequant_q6_k, 210)}[type_name]
    blocks = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1, block)
    assert blocks.shape[0] * QK_K == int(np.prod(shape)), (type_name, shape, raw.shape)
    return fn(blocks).reshape(shape)


def softmax(x: np.ndarray) -> np.ndarray:
    e = np.exp(x - x.max(axis=-1, keepdims=True))
    return e / e.sum(axis=-1, keepdims=True)


def route(logits: np.ndarray, top_k: int = 8, normalize: bool = True):
    """engines/base.py:91-97: float32 softmax over the experts, top_k largest (descending), divided by their sum.
    -> (weights [T, top_k] float32, selected [T, top_k] int64)."""
    p = softmax(logits.astype(np.float32))
    sel = np.argsort(-p, axis=-1, kind="stable")[:, :top_k]
    w = np.take_along_axis(p, sel, axis=-1)
    if normalize:
        w = w / w.sum(axis=-1, keepdims=True)
    return w.astype(np.float32), sel.astype(np.int64)


def silu(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):  # exp(-x) -> inf for very negative x gives the right limit, -0
        return x / (np.float32(1) + np.exp(-x))


def expert_gate(gate_up: np.ndarray) -> np.ndarray:
    """engines/base.py:99-102: silu(gate) * up on the fused [gate | up] output."""
    gate, up = np.split(gate_up, 2, axis=-1)
    return silu(gate) * up


def sigmoid(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        return np.float32(1) / (np.float32(1) + np.exp(-x))


def shared_expert(x, gate_w, up_w, down_w, shared_gate_w):
    """engines/base.py:104-107: down(silu(x G^T) * (x U^T)) scaled by sigmoid(x . g)."""
    h = (silu(x @ gate_w.T) * (x @ up_w.T)) @ down_w.T
    return sigmoid(x @ shared_gate_w.reshape(1, -1).T) * h


def skip_small_experts(w: np.ndarray, sel: np.ndarray, min_weight: float):
    """engines/base.py:413-429: keeps each token's top pick (column 0, the largest) and the picks whose weight is
    >= min_weight, scales the kept weights back up to the former total; dropped picks get selected -1."""
    keep = w >= min_weight
    keep[:, 0] = True
    kept = w * keep
    kept = kept * (w.sum(axis=-1, keepdims=True) / kept.sum(axis=-1, keepdims=True))
    return kept.astype(np.float32), np.where(keep, sel, -1)


def moe(x, router_w, expert_weights, shared, shared_gate_w, router_bias=None, top_k=8, min_expert_weight=0.0):
    """One MoE block, engines/base.py:445-490 on the CPU path (each_expert, base.py:534-591).
    x: float32 [T, H]. expert_weights(e) -> (gate_up float32 [2F, H], down float32 [H, F]).
    shared: (gate_up float32 [2F, H], down float32 [H, F]) of the shared expert.
    min_expert_weight > 0: skip_small_experts first (base.py:463-464).
    Returns (out [T, H] float32, routing weights [T, k], selected [T, k])."""
    x = x.astype(np.float32)
    logits = x @ router_w.T
    if router_bias is not None:
        logits = logits + router_bias
    w, sel = route(logits, top_k)
    if min_expert_weight:
        w, sel = skip_small_experts(w, sel, min_expert_weight)
    out = np.zeros_like(x)
    for e in np.unique(sel[sel >= 0]):  # ascending expert id, as each_expert sums them (base.py:580-586)
        tok, slot = np.nonzero(sel == e)
        gu, dn = expert_weights(int(e))
        h = expert_gate(x[tok] @ gu.T) @ dn.T
        np.add.at(out, tok, h * w[tok, slot, None])
    sgu, sdn = shared
    f = sgu.shape[0] // 2
    out = out + shared_expert(x, sgu[:f], sgu[f:], sdn, shared_gate_w)
    return out, w, sel


def rms_norm(x: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """engines/base.py:27-32 with zero_centered=True and a zero weight (scale 1)."""
    x32 = x.astype(np.float32)
    return x32 * (np.float32(1) / np.sqrt((x32 * x32).mean(-1, keepdims=True) + np.float32(eps)))


def moe_stack(h, layers, eps: float = 1e-6):
    """Decode through stacked MoE blocks with the residual wiring of engines/qwen36/model.py:17-22 (the token
    mixer left out): h <- h + moe(rms_norm(h)). layers: list of dicts with the keyword arguments of moe()."""
    for p in layers:
        h = h + moe(rms_norm(h, eps), **p)[0]
    return h
