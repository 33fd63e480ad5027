"""Phase breakdown of the persistent decode kernel (the role of willow's per-section Engine.tick timings,
engines/base.py:384-390). Runs one decode token through a synthetic stack with tracing on and prints, per trace
point, the time from the start of the layer (median and max over CTAs, mean over the middle layers).

    python -m willow_v2_b200.trace [--layers 8] [--seed 0]
"""
import argparse
import ctypes

import numpy as np
import torch

from . import moe, synth
from .lib import lib

POINTS = ["layer start", "x + router sums read", "top-k done (warp 0)", "gate_up copies issued (warp 0)",
          "x quantised, routing published", "gate_up chunk 0 landed", "gate_up chunk 0 computed",
          "gate_up chunk 1 landed", "gate_up done", "h published (S2 arrive)", "down rows landed",
          "down codes unpacked", "after S2", "h copied in", "down dot products", "combine + router sums"]


def synthetic_stack(layers: int, seed: int = 0, ctx=None):
    store = moe.ExpertStore(layers, ctx=ctx)
    store.fill_synthetic(seed)
    lws = [moe.LayerWeights(router_w=torch.from_numpy(synth.router_weight(seed, l)).cuda(),
                            shared_gate=torch.from_numpy(synth.shared_gate_weight(seed, l)).cuda(),
                            shared_gate_up=torch.from_numpy(synth.expert_gate_up(seed, l, 256).reshape(-1)).cuda(),
                            shared_down=torch.from_numpy(synth.expert_down(seed, l, 256).reshape(-1)).cuda())
           for l in range(layers)]
    return store, lws


def trace(layers: int = 8, seed: int = 0):
    ctx = moe.default_context()
    store, lws = synthetic_stack(layers, seed, ctx)
    h = torch.from_numpy(synth.hidden(seed, 1)).cuda()
    for _ in range(3):
        moe.decode_stack(store, lws, h)
    nc = lib.wmoe_decode_ctas(ctx.handle)
    P = len(POINTS)
    buf = torch.zeros(layers * P * nc, dtype=torch.int64, device="cuda")
    lib.wmoe_set_trace(ctx.handle, ctypes.c_void_p(buf.data_ptr()), buf.numel())
    try:
        moe.decode_stack(store, lws, h)
        torch.cuda.synchronize()
    finally:
        lib.wmoe_set_trace(ctx.handle, None, 0)
    ctx.check_device()
    t = buf.cpu().numpy().reshape(layers, P, nc).astype(np.float64)
    mid = range(1, layers - 1) if layers > 2 else range(layers)
    rows = np.array([[(np.median(t[l, q] - t[l, 0].min()), np.max(t[l, q] - t[l, 0].min())) for q in range(P)]
                     for l in mid])
    period = [t[l + 1, 0].min() - t[l, 0].min() for l in range(layers - 1)][1:] or [float("nan")]
    return nc, rows.mean(axis=0) / 1e3, float(np.mean(period)) / 1e3


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args()
    nc, rows, period = trace(a.layers, a.seed)
    print(f"{nc} CTAs; microseconds from the earliest CTA's layer start (median / max over CTAs)")
    for name, (med, mx) in zip(POINTS, rows):
        print(f"  {name:34s} {med:7.3f} {mx:7.3f}")
    print(f"  layer period {period:.3f} us")


if __name__ == "__main__":
    main()
