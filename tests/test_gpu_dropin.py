"""The drop-in boundary: willow's Engine.moe(x, layer, residual) (engines/base.py:445-490) served by the CudaMoE
mixin on a minimal engine object that holds its weights under willow's names (engines/qwen36/loader.py:37-41), the
way MoEEngine.forward calls it (engines/qwen36/model.py:22). Checked against the golden outputs willow produced
(tests/golden/moe.npz) and the oracle: the decode kernel (1 token), the dequant-GEMV kernels (4 tokens) and the
grouped GEMMs (16 and 64 tokens); a bf16 router as willow's loader keeps it; min_expert_weight
(engines/base.py:413-429); and the residual-driven next-layer prefetch (base.py:392-406, 473-474) on a capped
store."""
import numpy as np
import pytest

from oracle import moe_oracle as ora
from willow_v2_b200 import synth

pytestmark = pytest.mark.gpu
SEED = 0
LAYERS = 3
PREFIX = "model.language_model."
PATH_TOL = {1: 1e-4, 4: 1e-4, 16: 1e-3, 64: 1e-3}


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def willow_weights(dtype, bias=None):
    """A willow-style weights dict: the dequantised router and shared-expert gate (dtype), the shared expert's GGUF
    bytes under the .qweight names the mixin reads when the engine keeps them."""
    import torch
    w = {}
    for layer in range(LAYERS):
        p = f"{PREFIX}layers.{layer}.mlp"
        w[p + ".gate.weight"] = torch.from_numpy(synth.router_weight(SEED, layer)).to(dtype).cuda()
        w[p + ".shared_expert_gate.weight"] = torch.from_numpy(
            synth.shared_gate_weight(SEED, layer)).reshape(1, -1).to(dtype).cuda()
        w[p + ".shared_expert.gate_up_proj.qweight"] = torch.from_numpy(
            synth.expert_gate_up(SEED, layer, 256).reshape(-1)).cuda()
        w[p + ".shared_expert.down_proj.qweight"] = torch.from_numpy(
            synth.expert_down(SEED, layer, 256).reshape(-1)).cuda()
        if bias is not None:
            w[p + ".gate.bias"] = torch.from_numpy(bias).cuda()
    return w


def make_engine(store, weights, min_expert_weight=0.0, prefetch_top_k=8):
    import torch
    from willow_v2_b200.moe import CudaMoE

    class MinimalEngine:
        """The attributes of willow's Engine that Engine.moe reads."""
        prefix = PREFIX
        num_layers = LAYERS

        def __init__(self):
            self.weights, self.experts = weights, store
            self.min_expert_weight, self.prefetch_top_k = min_expert_weight, prefetch_top_k

        def w(self, name):
            return self.weights[name]

        def router_guess_input(self, residual, layer):  # engines/qwen36/model.py:30-31 with a unit norm weight
            x = residual.float()
            return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)

    class Engine(CudaMoE, MinimalEngine):
        pass

    return Engine()


@pytest.fixture(scope="module")
def model():
    import torch
    from willow_v2_b200 import moe
    torch.cuda.set_device(0)
    ctx = moe.Context(0)
    store = moe.ExpertStore(LAYERS, ctx=ctx)
    store.fill_synthetic(SEED)
    torch.cuda.synchronize()
    return ctx, store


def oracle_layer(layer, bf16_router=False, bias=None):
    def experts(e):
        return (ora.dequantize(synth.expert_gate_up(SEED, layer, e), "Q4_K", (1024, 2048)),
                ora.dequantize(synth.expert_down(SEED, layer, e), "Q6_K", (2048, 512)))
    r = synth.router_weight(SEED, layer)
    g = synth.shared_gate_weight(SEED, layer)
    if bf16_router:  # the values a bf16 copy holds
        import torch
        r = torch.from_numpy(r).to(torch.bfloat16).float().numpy()
        g = torch.from_numpy(g).to(torch.bfloat16).float().numpy()
    return dict(router_w=r, expert_weights=experts, shared=experts(256), shared_gate_w=g, router_bias=bias)


@pytest.mark.parametrize("case", ["t1", "t4", "t16z"])
def test_engine_moe_matches_golden(golden, model, case):
    """engine.moe(x, 0) with willow's f32 weights against the output willow's own code produced."""
    import torch
    ctx, store = model
    g = golden["moe"]
    bias = synth.zipf_bias(SEED) if case.endswith("z") else None
    engine = make_engine(store, willow_weights(torch.float32, bias))
    x = torch.from_numpy(g[case + "_x"]).cuda()
    out = engine.moe(x, 0)
    torch.cuda.synchronize()
    ctx.check_device()
    assert out.shape == x.shape and out.dtype == x.dtype
    err = rel_l2(out.cpu().numpy(), g[case + "_out"])
    assert err < 2e-3 and err < PATH_TOL[x.shape[0]], err


def test_engine_moe_bf16_router(model):
    """willow's loader keeps the router and the shared-expert gate in bf16 (engines/qwen36/loader.py:51-54): the
    mixin widens them to f32 exactly, so the result is the oracle's with the bf16 values."""
    import torch
    ctx, store = model
    engine = make_engine(store, willow_weights(torch.bfloat16))
    x = synth.hidden(SEED, 4, step=31)
    out = engine.moe(torch.from_numpy(x).cuda(), 1).cpu().numpy()
    ref = ora.moe(x, **oracle_layer(1, bf16_router=True))[0]
    assert rel_l2(out, ref) < 1e-4


@pytest.mark.parametrize("T", [1, 4, 64])
def test_engine_min_expert_weight(model, T):
    """min_expert_weight 0.1: the picks willow's skip_small_experts drops (every token keeps its top one) are left
    out and the kept weights rescaled, on the decode kernel (1 token), the GEMV kernels (4) and the GEMMs (64);
    the routing the library reports marks the dropped picks -1."""
    import torch
    from willow_v2_b200 import moe
    ctx, store = model
    engine = make_engine(store, willow_weights(torch.float32), min_expert_weight=0.1)
    x = synth.hidden(SEED, T, step=40 + T)
    xt = torch.from_numpy(x).cuda()
    out = engine.moe(xt, 2).cpu().numpy()
    ref, rw, rsel = ora.moe(x, **oracle_layer(2), min_expert_weight=0.1)
    assert (rsel < 0).any(), "the threshold drops no pick on these tokens"
    assert rel_l2(out, ref) < PATH_TOL[T]
    # the routing as the library reports it
    ctx.set_min_expert_weight(0.1)
    try:
        _, w, sel = moe.moe_forward(store, 2, xt, engine.moe_layer_weights(2), return_routing=True)
    finally:
        ctx.set_min_expert_weight(0.0)
    sel, w = sel.cpu().numpy(), w.cpu().numpy()
    np.testing.assert_array_equal(np.sort(sel, axis=1), np.sort(rsel, axis=1))
    np.testing.assert_allclose(np.sort(w, axis=1), np.sort(rw, axis=1), rtol=1e-5, atol=1e-7)
    ctx.check_device()


def test_engine_residual_prefetches_next_layer(model):
    """Decode through the engine's layers on a capped store, residual given as MoEEngine.forward gives it: each
    call guesses the next layer's experts from the residual (the engine's router_guess_input) and starts copying
    them; outputs stay bit-identical to the resident store, and later calls use prefetched copies."""
    import torch
    from willow_v2_b200 import moe
    ctx, store = model
    blob = (store.blob_bytes + 255) // 256 * 256
    capped = moe.ExpertStore(LAYERS, cap_bytes=120 * blob, ctx=ctx)
    capped.fill_synthetic(SEED)
    weights = willow_weights(torch.float32)
    resident, guessing = make_engine(store, weights), make_engine(capped, weights)
    prev = ctx.set_decode_kernel(False)  # both stores on the GEMV kernels (a capped store never takes the decode one)
    try:
        run_tokens(ctx, store, resident, guessing)
    finally:
        ctx.set_decode_kernel(prev)
    st = capped.stats()
    assert st["prefetched"] > 0 and st["prefetch_used"] > 0, st
    ctx.check_device()
    capped.close()


def run_tokens(ctx, store, resident, guessing):
    import torch
    for step in range(4):
        h_a = h_b = torch.from_numpy(synth.hidden(SEED, 1, step=60 + step)).cuda()
        for layer in range(LAYERS):
            xa = ora_free_rms(h_a)
            a = resident.moe(xa, layer, residual=h_a)
            b = guessing.moe(xa.clone(), layer, residual=h_b)
            torch.cuda.synchronize()
            assert torch.equal(a, b), (step, layer)
            h_a = h_b = h_a + a


def ora_free_rms(h):
    """rms_norm with a unit weight on the GPU (the engine's own norm before its MoE block)."""
    x = h.float()
    return x * x.pow(2).mean(-1, keepdim=True).add(1e-6).rsqrt()
