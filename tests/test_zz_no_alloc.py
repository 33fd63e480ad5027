"""wmoe_decode_stack_noalloc: the decode stack for callers that cannot allocate device memory (a caller inside a
CUDA graph capture, an engine whose memory belongs to a pool allocator, a decode loop that must never grow a
buffer). Its scratch is a fixed static device array, so its results must equal those of the allocating entry
point, wmoe_decode_stack, call after call. This file is collected last so that a failure here cannot hide the
others; it also passes on its own in a fresh process."""
import ctypes

import numpy as np
import pytest

from willow_v2_b200 import synth

pytestmark = pytest.mark.gpu
SEED = 0
LAYERS = 2


def test_noalloc_decode_stack_matches_allocating_entry_point():
    import torch
    from willow_v2_b200 import lib as L
    from willow_v2_b200 import moe
    torch.cuda.set_device(0)
    ctx = moe.Context(0)
    store = moe.ExpertStore(LAYERS, ctx=ctx)
    store.fill_synthetic(SEED)
    layers = [moe.LayerWeights(router_w=torch.from_numpy(synth.router_weight(SEED, l)).cuda(),
                               shared_gate=torch.from_numpy(synth.shared_gate_weight(SEED, l)).cuda(),
                               shared_gate_up=torch.from_numpy(synth.expert_gate_up(SEED, l, 256).reshape(-1)).cuda(),
                               shared_down=torch.from_numpy(synth.expert_down(SEED, l, 256).reshape(-1)).cuda())
              for l in range(LAYERS)]
    for lw in layers:
        lw.router_packed = moe.pack_router(lw.router_w, lw.shared_gate, ctx)
    arr = (L.LayerWeights * LAYERS)(*[lw.as_struct() for lw in layers])
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    for call in range(2):  # two calls in a row: the static scratch keeps the previous call's contents
        h = torch.from_numpy(synth.hidden(SEED, 1, step=40 + call)).cuda().reshape(-1)
        want, want_sel = moe.decode_stack(store, layers, h, 1e-6, return_routing=True)
        got = torch.empty_like(h)
        sel = torch.empty(LAYERS, 8, dtype=torch.int32, device="cuda")
        L.check(ctx.handle, L.lib.wmoe_decode_stack_noalloc(ctx.handle, store.handle, 0, LAYERS,
                                                           ctypes.cast(arr, ctypes.c_void_p), ctypes.c_float(1e-6),
                                                           ctypes.c_void_p(h.data_ptr()),
                                                           ctypes.c_void_p(got.data_ptr()),
                                                           ctypes.c_void_p(sel.data_ptr()), stream))
        torch.cuda.synchronize()
        ctx.check_device()
        assert torch.equal(sel, want_sel), call
        a, b = got.cpu().numpy().astype(np.float64), want.cpu().numpy().astype(np.float64)
        err = np.linalg.norm(a - b) / np.linalg.norm(b)
        assert err < 1e-6, (call, err)  # the same kernel on the same inputs: equal up to float64 sum order
    store.close()
    ctx.close()
