"""Parity on the exact configurations bench.py times ([2], [3]), against the float32
oracle, through the C ABI:

  configs[1]  one token through the 40-layer stack (rms_norm + residual between layers, engines/qwen36/model.py:
              17-22): every block against the oracle on the GPU's input, and the oracle's own 40-layer stack
  configs[2]  the whole 64-token f32 block with the Zipf routing bias (sliced router, dispatch, grouped GEMMs)
  configs[3]  4096 bf16 tokens through the tensor-core router and the grouped GEMMs; every token routed to two
              chosen experts plus the first 64 tokens (>= 256 tokens) compared with the oracle

Bounds: MoE block outputs within 2e-3 relative L2 (BASELINE.json's bound for fp32 reference vs fp32-accumulated
outputs), with the tighter bound each path measures asserted as well; top-8 picks identical except where the
oracle's float64 logits of the 8th and 9th expert lie within 1e-5."""
import functools

import numpy as np
import pytest

from oracle import moe_oracle as ora
from willow_v2_b200 import synth

pytestmark = pytest.mark.gpu
SEED = 0
TOL = 2e-3
TIE = 1e-5


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@functools.lru_cache(maxsize=None)
def _expert(layer, e):
    return (ora.dequantize(synth.expert_gate_up(SEED, layer, e), "Q4_K", (1024, 2048)),
            ora.dequantize(synth.expert_down(SEED, layer, e), "Q6_K", (2048, 512)))


def oracle_args(layer, bias=None):
    return dict(router_w=synth.router_weight(SEED, layer), expert_weights=lambda e: _expert(layer, e),
                shared=_expert(layer, 256), shared_gate_w=synth.shared_gate_weight(SEED, layer), router_bias=bias)


def near_tie(x, layer, bias=None):
    """Per token: whether the oracle's float64 logits of the 8th and 9th expert lie within TIE."""
    lg = np.asarray(x, np.float64) @ synth.router_weight(SEED, layer).T.astype(np.float64)
    if bias is not None:
        lg = lg + bias
    s = -np.sort(-lg, axis=-1)
    return (s[:, 7] - s[:, 8]) < TIE


def layer_weights(layer, bias=None):
    import torch
    from willow_v2_b200 import moe
    return moe.LayerWeights(
        router_w=torch.from_numpy(synth.router_weight(SEED, layer)).cuda(),
        shared_gate=torch.from_numpy(synth.shared_gate_weight(SEED, layer)).cuda(),
        shared_gate_up=torch.from_numpy(synth.expert_gate_up(SEED, layer, 256).reshape(-1)).cuda(),
        shared_down=torch.from_numpy(synth.expert_down(SEED, layer, 256).reshape(-1)).cuda(),
        router_bias=None if bias is None else torch.from_numpy(bias).cuda())


@pytest.fixture(scope="module")
def ctx():
    import torch
    from willow_v2_b200 import moe
    torch.cuda.set_device(0)
    return moe.Context(0)


def test_decode40_stack_matches_oracle(ctx):
    """the persistent decode kernel over all 40 layers (20.9 GB of experts resident).
    * Every block against the oracle on the GPU's own input to that layer (the 2e-3 bound is a per-block bound):
      the block output h_{l+1} - h_l and the picks.
    * The oracle's free-running 40-layer stack picks the same experts in every layer. Its final state drifts from
      the GPU's by ~4e-3 relative L2: each block's ~5e-5 compounds through 40 residual layers of this synthetic
      model (outputs grow to |h| ~ 3e5), so that drift is bounded loosely (1e-2), not by the per-block bound.
    * 40 one-layer launches chained give the 40-layer launch's output bit for bit."""
    import torch
    from willow_v2_b200 import moe
    layers = 40
    store = moe.ExpertStore(layers, ctx=ctx)
    store.fill_synthetic(SEED)
    lws = [layer_weights(l) for l in range(layers)]
    h0 = synth.hidden(SEED, 1, step=0)
    out, sel = moe.decode_stack(store, lws, torch.from_numpy(h0).cuda(), 1e-6, return_routing=True)
    hs = [torch.from_numpy(h0).cuda().reshape(-1)]
    for l in range(layers):
        hs.append(moe.decode_stack(store, [lws[l]], hs[-1], 1e-6, layer_begin=l))
    torch.cuda.synchronize()
    ctx.check_device()
    assert torch.equal(hs[-1], out.reshape(-1))
    sel = sel.cpu().numpy()
    hs = [h.cpu().numpy().reshape(1, -1) for h in hs]
    h = h0.astype(np.float32)
    worst = 0.0
    for l in range(layers):
        # the block on the GPU's input
        xg = ora.rms_norm(hs[l])
        og, _, gsel = ora.moe(xg, **oracle_args(l))
        if not near_tie(xg, l)[0]:
            np.testing.assert_array_equal(np.sort(sel[l]), np.sort(gsel[0]), err_msg=f"layer {l}")
        err = rel_l2(hs[l + 1] - hs[l], og)
        worst = max(worst, err)
        assert err < TOL and err < 2e-4, (l, err)
        # the oracle's own stack
        xn = ora.rms_norm(h)
        assert not near_tie(xn, l)[0], f"layer {l} has a near-tie; the free-running comparison would not hold"
        o, _, osel = ora.moe(xn, **oracle_args(l))
        np.testing.assert_array_equal(np.sort(sel[l]), np.sort(osel[0]), err_msg=f"free-running layer {l}")
        h = h + o
    drift = rel_l2(hs[-1], h)
    print(f"decode40: worst block error {worst:.2e}, free-running drift after 40 layers {drift:.2e}")
    assert drift < 1e-2, drift
    store.close()


def test_batch64_zipf_block_matches_oracle(ctx):
    """the whole 64-token block (f32, Zipf bias) on the default path (sliced float32 router, dispatch,
    grouped GEMMs from 16 tokens) against ora.moe on all 64 tokens."""
    import torch
    from willow_v2_b200 import moe
    store = moe.ExpertStore(1, ctx=ctx)
    store.fill_synthetic(SEED)
    bias = synth.zipf_bias(SEED)
    lw = layer_weights(0, bias)
    x = synth.hidden(SEED, 64, step=0)
    out, w, sel = moe.moe_forward(store, 0, torch.from_numpy(x).cuda(), lw, return_routing=True)
    torch.cuda.synchronize()
    ctx.check_device()
    ref, rw, rsel = ora.moe(x, **oracle_args(0, bias))
    ties = near_tie(x, 0, bias)
    sel = sel.cpu().numpy()
    for t in np.flatnonzero(~ties):
        np.testing.assert_array_equal(np.sort(sel[t]), np.sort(rsel[t]), err_msg=f"token {t}")
    keep = ~ties
    assert keep.sum() >= 60
    err = rel_l2(out.cpu().numpy()[keep], ref[keep])
    assert err < TOL and err < 1e-3, err
    store.close()


def test_prefill4096_tokens_match_oracle(ctx):
    """4096 bf16 tokens, uniform routing, tensor-core router + grouped GEMMs. Every token routed to
    experts 17 or 201 plus the first 64 tokens are compared with the oracle (dequantised experts, float32)."""
    import torch
    from willow_v2_b200 import moe
    store = moe.ExpertStore(1, ctx=ctx)
    store.fill_synthetic(SEED)
    lw = layer_weights(0).prepare(ctx, decode=False)
    xb = torch.from_numpy(synth.hidden(SEED, 4096, step=0)).to(torch.bfloat16)
    out, w, sel = moe.moe_forward(store, 0, xb.cuda(), lw, out_dtype=torch.float32, return_routing=True)
    torch.cuda.synchronize()
    ctx.check_device()
    sel = sel.cpu().numpy()
    chosen = np.flatnonzero(np.isin(sel, [17, 201]).any(axis=1))
    idx = np.union1d(chosen, np.arange(64))
    assert idx.size >= 256, idx.size
    x = xb.float().numpy()[idx]
    ref, _, rsel = ora.moe(x, **oracle_args(0))
    ties = near_tie(x, 0)
    for i in np.flatnonzero(~ties):
        np.testing.assert_array_equal(np.sort(sel[idx[i]]), np.sort(rsel[i]), err_msg=f"token {idx[i]}")
    keep = ~ties
    err = rel_l2(out.cpu().numpy()[idx][keep], ref[keep])
    assert err < TOL and err < 1e-3, err
    store.close()
