"""Generates skip.npz by running willow's own Engine.skip_small_experts (engines/base.py:413-429, the
--min-expert-weight option) on routings that engines/base.py:route produced from seeded random logits. Run it
where a willow-v2 checkout is available:

    python tests/golden/make_golden_skip.py --reference <path to the willow-v2 checkout>

skip.npz holds, per threshold m in MIN_WEIGHTS: the routing weights w [T, 8] and selection sel [T, 8] (the
inputs), and willow's outputs w_<m> (kept weights, rescaled) and sel_<m> (-1 where dropped).
"""
import argparse
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
MIN_WEIGHTS = (0.05, 0.1, 0.125, 0.2)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import torch
    from engines import base

    rng = np.random.default_rng(11)
    T = 256
    logits = rng.normal(0.0, 1.0, (T, 256)).astype(np.float32)
    logits[: T // 4] *= 4.0  # peaked routings: several picks below each threshold
    w, sel = base.route(torch.from_numpy(logits), 8, True)
    out = {"w": w.numpy(), "sel": sel.numpy().astype(np.int64)}
    for m in MIN_WEIGHTS:
        # the method reads only these attributes of the engine
        eng = types.SimpleNamespace(min_expert_weight=m, ops=types.SimpleNamespace(decoding=False), keep_alive=[],
                                    guess_weights=None)
        kw, ks, _ = base.Engine.skip_small_experts(eng, w.clone(), sel.clone(), None)
        out[f"w_{m}"] = kw.numpy()
        out[f"sel_{m}"] = ks.numpy().astype(np.int64)
    np.savez_compressed(os.path.join(HERE, "skip.npz"), **out)
    print("wrote skip.npz", {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
