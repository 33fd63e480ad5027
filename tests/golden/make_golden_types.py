"""Generates tests/golden/ggml_types.npz: blocks of every ggml type the typed expert kernels run (the types of
willow's Metal kernels, gguf/metal.py:295) with the float32 values willow's own gguf/quants.py:dequantize returns
for them. Run it where a willow-v2 checkout is available:

    python tests/golden/make_golden_types.py --reference <path to the willow-v2 checkout>

Per type T the file holds blocks_T (uint8 [n, block bytes]: seeded random blocks with fp16 scales drawn from
U[1e-3, 4e-3], then hand-made edge blocks: zero bytes, 0xFF bytes, the largest, a subnormal and a negative scale)
and values_T (float32 [n, block elements]). llama.cpp's gguf-py is run on the same blocks in a separate interpreter
(willow's package is also named gguf) and must give the same bits for every type it has (all but Q2_0).
"""
import argparse
import json
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# (elements, bytes, byte offset of the fp16 scale d) per block (gguf/reader.py:14-48)
TYPES = {"Q5_0": (32, 22, 0), "Q8_0": (32, 34, 0), "IQ4_NL": (32, 18, 0), "IQ4_XS": (256, 136, 0),
         "IQ3_XXS": (256, 98, 0), "IQ3_S": (256, 110, 0), "IQ2_S": (256, 82, 0), "Q2_0": (64, 18, 0),
         "Q4_K": (256, 144, 0), "Q6_K": (256, 210, 208)}
N_RANDOM = 48


def blocks_for(name: str, seed: int) -> np.ndarray:
    _, size, d_at = TYPES[name]
    rng = np.random.default_rng(seed)
    b = rng.integers(0, 256, (N_RANDOM, size), dtype=np.uint8)
    d = rng.uniform(1e-3, 4e-3, N_RANDOM).astype(np.float16)
    b[:, d_at:d_at + 2] = d.view(np.uint8).reshape(-1, 2)
    if name == "Q4_K":  # dmin beside d
        b[:, 2:4] = rng.uniform(1e-3, 4e-3, N_RANDOM).astype(np.float16).view(np.uint8).reshape(-1, 2)
    edges = []
    for d_val, fill in [(0.0, 0x00), (1.0, 0xFF), (65504.0, None), (6e-8, None), (-2.5e-3, None), (1.0, 0x00)]:
        e = rng.integers(0, 256, size, dtype=np.uint8) if fill is None else np.full(size, fill, dtype=np.uint8)
        e[d_at:d_at + 2] = np.array([d_val], dtype=np.float16).view(np.uint8)
        if name == "Q4_K":
            e[2:4] = np.array([d_val / 2], dtype=np.float16).view(np.uint8)
        edges.append(e)
    return np.concatenate([b, np.stack(edges)])


def gguf_py_values(blocks: dict) -> dict:
    code = ("import sys, numpy as np\n"
            "from gguf.quants import dequantize\n"
            "from gguf.constants import GGMLQuantizationType as T\n"
            "a = np.load(sys.argv[1])\n"
            "out = {k: dequantize(a[k].reshape(-1), getattr(T, k)).astype(np.float32) for k in a.files\n"
            "       if hasattr(T, k)}\n"
            "np.savez(sys.argv[2], **out)\n")
    src, dst = "/tmp/wmoe_types_in.npz", "/tmp/wmoe_types_out.npz"
    np.savez(src, **blocks)
    subprocess.run([sys.executable, "-c", code, src, dst], check=True, cwd="/tmp", env=dict(os.environ, PYTHONPATH=""))
    out = np.load(dst)
    return {k: out[k] for k in out.files}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the willow-v2 checkout")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import torch
    from gguf import quants  # willow's gguf package (gguf/quants.py)

    blocks = {name: blocks_for(name, 100 + i) for i, name in enumerate(TYPES)}
    arrays, versions = {}, {"torch": torch.__version__}
    for name, b in blocks.items():
        elements = TYPES[name][0]
        v = quants.dequantize(torch.from_numpy(b.reshape(-1).copy()), name, (b.shape[0], elements), torch.float32)
        arrays["blocks_" + name] = b
        arrays["values_" + name] = v.numpy()
    second = gguf_py_values(blocks)
    for name, v in second.items():
        ours = arrays["values_" + name].reshape(-1)
        same = np.array_equal(ours.view(np.uint32), v.reshape(-1).view(np.uint32))
        both_nan = np.isnan(ours) & np.isnan(v.reshape(-1))
        assert same or np.array_equal(ours[~both_nan], v.reshape(-1)[~both_nan]), name
    versions["gguf_py_checked"] = sorted(second)
    np.savez_compressed(os.path.join(HERE, "ggml_types.npz"), **arrays)
    with open(os.path.join(HERE, "ggml_types.json"), "w") as f:
        json.dump({"types": list(TYPES), "random_blocks": N_RANDOM, "edge_blocks": 6, "versions": versions}, f,
                  indent=1)
    print("wrote ggml_types.npz:", {k: v.shape for k, v in arrays.items() if k.startswith("blocks_")})


if __name__ == "__main__":
    main()
