"""The CPU oracle against the golden vectors willow itself produced (tests/golden/make_golden.py)."""
import hashlib
import json
import os

import numpy as np

from oracle import moe_oracle as ora
from willow_v2_b200 import synth

HERE = os.path.dirname(os.path.abspath(__file__))
SEED = 0


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def test_dequant_q4k_bit_exact(golden):
    g = golden["dequant"]
    np.testing.assert_array_equal(bits(ora.dequant_q4_k(g["q4"])), bits(g["q4_out"]))


def test_dequant_q6k_bit_exact(golden):
    g = golden["dequant"]
    np.testing.assert_array_equal(bits(ora.dequant_q6_k(g["q6"])), bits(g["q6_out"]))


def test_route_matches_reference(golden):
    g = golden["route"]
    w, sel = ora.route(g["logits"], 8)
    ties = 0
    for t in range(g["logits"].shape[0]):
        if not np.array_equal(np.sort(sel[t]), np.sort(g["selected"][t])):
            # allowed only where the 8th and 9th largest logits are within 1e-5
            s = np.sort(g["logits"][t])[::-1]
            assert s[7] - s[8] < 1e-5, t
            ties += 1
            continue
        order_o, order_r = np.argsort(sel[t]), np.argsort(g["selected"][t])
        np.testing.assert_allclose(w[t][order_o], g["weights"][t][order_r], rtol=2e-6, atol=1e-7)
    assert ties <= 2


def rel_l2(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / np.linalg.norm(b.astype(np.float64)))


def expert_weights(layer):
    def f(e):
        return (ora.dequantize(synth.expert_gate_up(SEED, layer, e), "Q4_K", (1024, 2048)),
                ora.dequantize(synth.expert_down(SEED, layer, e), "Q6_K", (2048, 512)))
    return f


def layer_params(layer, bias=None):
    return dict(router_w=synth.router_weight(SEED, layer), expert_weights=expert_weights(layer),
                shared=expert_weights(layer)(256), shared_gate_w=synth.shared_gate_weight(SEED, layer),
                router_bias=bias)


def test_moe_matches_reference(golden):
    g = golden["moe"]
    for name, bias in (("t1", None), ("t4", None), ("t16z", synth.zipf_bias(SEED))):
        out, w, sel = ora.moe(g[name + "_x"], **layer_params(0, bias))
        np.testing.assert_array_equal(sel, g[name + "_sel"])
        np.testing.assert_allclose(w, g[name + "_w"], rtol=2e-6)
        assert rel_l2(out, g[name + "_out"]) < 1e-5, name


def test_stack_matches_reference(golden):
    g = golden["moe"]
    out = ora.moe_stack(g["stack_in"], [layer_params(l) for l in range(3)])
    assert rel_l2(out, g["stack_out"]) < 1e-5


def test_synthetic_bytes_pinned():
    with open(os.path.join(HERE, "golden", "meta.json")) as f:
        meta = json.load(f)
    for key in list(meta["expert_sha256"])[:3] + ["0_256"]:
        layer, e = map(int, key.split("_"))
        blob = synth.expert_blob(SEED, layer, e)
        assert hashlib.sha256(blob.tobytes()).hexdigest() == meta["expert_sha256"][key], key


def test_synthetic_distributions():
    q4 = synth.q4k_blocks(synth.tensor_key(3, 1, 2, 0), 4096)
    d = q4[:, 0:4].copy().view(np.float16).astype(np.float32)
    assert d.min() >= 1e-3 - 1e-6 and d.max() <= 4e-3 + 2e-6
    q6 = synth.q6k_blocks(synth.tensor_key(3, 1, 2, 1), 4096)
    sc = q6[:, 192:208].copy().view(np.int8)
    assert sc.min() == -32 and sc.max() == 31
    d6 = q6[:, 208:210].copy().view(np.float16).astype(np.float32)
    assert d6.min() >= 1e-3 - 1e-6 and d6.max() <= 4e-3 + 2e-6
    # partial-row generation is a slice of the whole tensor
    full = synth.expert_down(3, 1, 2)
    np.testing.assert_array_equal(synth.expert_down(3, 1, 2, rows=(100, 140)), full[100:140])


def test_skip_small_experts_matches_reference():
    """ora.skip_small_experts against willow's Engine.skip_small_experts (engines/base.py:413-429) on 256 routings
    and four thresholds (tests/golden/make_golden_skip.py): the same picks dropped, the kept weights rescaled."""
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "skip.npz"))
    dropped = 0
    for m in (0.05, 0.1, 0.125, 0.2):
        w, sel = ora.skip_small_experts(g["w"], g["sel"], m)
        np.testing.assert_array_equal(sel, g[f"sel_{m}"])
        np.testing.assert_allclose(w, g[f"w_{m}"], rtol=1e-6, atol=0)
        dropped += int((sel < 0).sum())
    assert dropped > 0

