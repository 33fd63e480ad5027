"""Generates the golden fixtures in this directory by running willow's own code (and llama.cpp's gguf-py as a
second opinion) on seeded synthetic inputs. Run it where a willow-v2 checkout is available:

    python tests/golden/make_golden.py --reference <path to the willow-v2 checkout>

It writes:
  dequant.npz  Q4_K and Q6_K blocks (synthetic ones from willow_v2_b200.synth plus hand-made edge blocks) with
               the float32 values gguf/quants.py:dequantize returns for them; gguf-py's dequantize is checked to
               give the same bits.
  route.npz    router logits (random, Zipf-biased and near-tie rows) with engines/base.py:route's outputs.
  moe.npz      MoE blocks (config-0 shapes: T=1, T=4, and T=16 with a Zipf bias) and a 3-layer stack, computed
               by the reference's dequantize/route/expert_gate/shared_expert with the data flow of
               Engine.moe/each_expert (engines/base.py:445-490, 534-591), in float32 on the CPU.
  meta.json    versions, seeds, and SHA-256 digests of the synthetic expert bytes used (pins the generator).
"""
import argparse
import hashlib
import json
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
from willow_v2_b200 import synth  # noqa: E402

SEED = 0


def edge_q4k() -> np.ndarray:
    """Hand-made Q4_K blocks: zero bytes, all-ones bytes, the largest/smallest fp16 scales, subnormal and negative
    scales, every 6-bit scale/min at its maximum."""
    rng = np.random.default_rng(7)
    blocks = []
    for d, dmin, fill in [(0.0, 0.0, 0x00), (1.0, 1.0, 0xFF), (65504.0, 65504.0, 0xFF), (6e-8, 6e-8, 0x5A),
                          (-2e-3, 3e-3, None), (2e-3, -3e-3, None), (1.0, 0.0, 0x3F), (5.96e-8, 1e-4, None)]:
        b = rng.integers(0, 256, 144, dtype=np.uint8) if fill is None else np.full(144, fill, dtype=np.uint8)
        b[0:2] = np.array([d], dtype=np.float16).view(np.uint8)
        b[2:4] = np.array([dmin], dtype=np.float16).view(np.uint8)
        blocks.append(b)
    return np.stack(blocks)


def edge_q6k() -> np.ndarray:
    rng = np.random.default_rng(8)
    blocks = []
    for d, fill, sc in [(0.0, 0x00, 0), (1.0, 0xFF, 127), (65504.0, 0xFF, -128), (6e-8, 0x00, -1), (-3e-3, None, None),
                        (1.0, 0x55, 31), (1.0, 0xAA, -32), (5.96e-8, None, None)]:
        b = rng.integers(0, 256, 210, dtype=np.uint8) if fill is None else np.full(210, fill, dtype=np.uint8)
        if sc is not None:
            b[192:208] = np.array([sc] * 16, dtype=np.int8).view(np.uint8)
        b[208:210] = np.array([d], dtype=np.float16).view(np.uint8)
        blocks.append(b)
    return np.stack(blocks)


def gguf_py_dequant(q4: np.ndarray, q6: np.ndarray):
    """Runs llama.cpp's gguf-py in a separate interpreter (willow's own package is also named gguf)."""
    code = ("import sys, numpy as np, gguf\n"
            "from gguf.quants import dequantize\n"
            "from gguf.constants import GGMLQuantizationType as T\n"
            "a = np.load(sys.argv[1])\n"
            "np.savez(sys.argv[2], q4=dequantize(a['q4'], T.Q4_K).astype(np.float32),\n"
            "         q6=dequantize(a['q6'], T.Q6_K).astype(np.float32), version=np.array(gguf.__version__ if hasattr(gguf, '__version__') else ''))\n")
    src, dst = os.path.join("/tmp", "wmoe_gguf_in.npz"), os.path.join("/tmp", "wmoe_gguf_out.npz")
    np.savez(src, q4=q4, q6=q6)
    env = dict(os.environ, PYTHONPATH="")
    subprocess.run([sys.executable, "-c", code, src, dst], check=True, cwd="/tmp", env=env)
    out = np.load(dst)
    return out["q4"].reshape(q4.shape[0], 256), out["q6"].reshape(q6.shape[0], 256)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the willow-v2 checkout")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import torch
    import torch.nn.functional as F
    from gguf import quants
    from engines import base

    meta = {"seed": SEED, "torch": torch.__version__, "numpy": np.__version__, "expert_sha256": {}}

    # ---- dequant KATs
    q4 = np.concatenate((synth.q4k_blocks(synth.tensor_key(SEED, 0, 0, 0), 120), edge_q4k()))
    q6 = np.concatenate((synth.q6k_blocks(synth.tensor_key(SEED, 0, 0, 1), 120), edge_q6k()))
    ref_q4 = quants.dequantize(torch.from_numpy(q4.reshape(-1).copy()), "Q4_K", (q4.shape[0], 256), torch.float32).numpy()
    ref_q6 = quants.dequantize(torch.from_numpy(q6.reshape(-1).copy()), "Q6_K", (q6.shape[0], 256), torch.float32).numpy()
    g4, g6 = gguf_py_dequant(q4, q6)
    same = lambda a, b: bool(np.array_equal(a.view(np.uint32), b.view(np.uint32)))
    meta["gguf_py_bit_identical"] = {"Q4_K": same(ref_q4, g4), "Q6_K": same(ref_q6, g6)}
    np.savez_compressed(os.path.join(HERE, "dequant.npz"), q4=q4, q4_out=ref_q4, q6=q6, q6_out=ref_q6)

    # ---- route KATs
    rng = np.random.default_rng(11)
    logits = rng.standard_normal((64, 256), dtype=np.float32) * np.float32(0.9)
    logits[:8] += synth.zipf_bias(SEED)
    logits[60, 5] = logits[60, 7]                              # an exact tie
    logits[61, 9] = np.nextafter(logits[61, 3], np.float32(np.inf))  # one ulp apart
    logits[62, :] = 0.0                                        # all equal
    rw, rsel = base.route(torch.from_numpy(logits), 8, True)
    np.savez_compressed(os.path.join(HERE, "route.npz"), logits=logits, weights=rw.numpy(), selected=rsel.numpy())

    # ---- MoE blocks through the reference's functions and Engine.moe's data flow
    def expert_f32(layer, e):
        gu = synth.expert_gate_up(SEED, layer, e)
        dn = synth.expert_down(SEED, layer, e)
        meta["expert_sha256"][f"{layer}_{e}"] = hashlib.sha256(gu.tobytes() + dn.tobytes()).hexdigest()
        return (quants.dequantize(torch.from_numpy(gu.reshape(-1).copy()), "Q4_K", (1024, 2048), torch.float32),
                quants.dequantize(torch.from_numpy(dn.reshape(-1).copy()), "Q6_K", (2048, 512), torch.float32))

    def ref_moe(x, layer, bias=None):
        router = torch.from_numpy(synth.router_weight(SEED, layer))
        gate_vec = torch.from_numpy(synth.shared_gate_weight(SEED, layer)).reshape(1, -1)
        logits = F.linear(x, router)
        if bias is not None:
            logits = logits + torch.from_numpy(bias)
        w, sel = base.route(logits, 8, True)
        out = torch.zeros_like(x)
        for e in sel.unique().tolist():  # each_expert: every token of an expert, summed in ascending id
            tok, slot = (sel == e).nonzero(as_tuple=True)
            gu, dn = expert_f32(layer, e)
            gate, up = F.linear(x[tok], gu).chunk(2, dim=-1)
            h = F.linear(F.silu(gate) * up, dn)
            out.index_add_(0, tok, h * w[tok, slot, None])
        sgu, sdn = expert_f32(layer, 256)
        out = out + base.shared_expert(x, sgu[:512], sgu[512:], sdn, gate_vec)
        return out, w, sel

    cases = {}
    for name, tokens, bias in (("t1", 1, None), ("t4", 4, None), ("t16z", 16, synth.zipf_bias(SEED))):
        x = torch.from_numpy(synth.hidden(SEED, tokens))
        out, w, sel = ref_moe(x, 0, bias)
        cases[name + "_x"], cases[name + "_out"] = x.numpy(), out.numpy()
        cases[name + "_w"], cases[name + "_sel"] = w.numpy(), sel.numpy()

    # 3-layer decode stack: h <- h + moe(rms_norm(h)) (engines/qwen36/model.py:17-22, zero-centred norm, weight 0)
    h = torch.from_numpy(synth.hidden(SEED, 1, step=5))
    cases["stack_in"] = h.numpy().copy()
    for layer in range(3):
        xn = base.rms_norm(h, torch.zeros(2048), 1e-6, True)
        h = h + ref_moe(xn, layer)[0]
    cases["stack_out"] = h.numpy()
    np.savez_compressed(os.path.join(HERE, "moe.npz"), **cases)

    with open(os.path.join(HERE, "meta.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    print(json.dumps({k: v for k, v in meta.items() if k != "expert_sha256"}, indent=1))


if __name__ == "__main__":
    main()
