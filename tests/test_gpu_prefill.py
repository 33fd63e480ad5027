"""The prefill path (tcgen05 grouped GEMMs with fp16 tiles dequantised in shared memory) against the oracle and
against the dequant-GEMV path on the same inputs. Bound: 2e-3 relative L2 (BASELINE's, fp32 reference vs
fp32-accumulated low-precision outputs); fp16 operands measure ~4e-4 in numpy, so 1e-3 is asserted."""
import numpy as np
import pytest

from oracle import moe_oracle as ora
from willow_v2_b200 import synth

pytestmark = pytest.mark.gpu
SEED = 0
TOL = 2e-3


def rel_l2(a, b):
    a, b = np.asarray(a, dtype=np.float64), np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@pytest.fixture(scope="module")
def model():
    import torch
    from willow_v2_b200 import moe
    torch.cuda.set_device(0)
    ctx = moe.Context(0)
    store = moe.ExpertStore(2, ctx=ctx)
    store.fill_synthetic(SEED)
    torch.cuda.synchronize()
    return ctx, store


def layer_weights(layer, bias=None):
    import torch
    from willow_v2_b200 import moe
    return moe.LayerWeights(
        router_w=torch.from_numpy(synth.router_weight(SEED, layer)).cuda(),
        shared_gate=torch.from_numpy(synth.shared_gate_weight(SEED, layer)).cuda(),
        shared_gate_up=torch.from_numpy(synth.expert_gate_up(SEED, layer, 256).reshape(-1)).cuda(),
        shared_down=torch.from_numpy(synth.expert_down(SEED, layer, 256).reshape(-1)).cuda(),
        router_bias=None if bias is None else torch.from_numpy(bias).cuda())


def oracle_layer(layer, bias=None):
    def experts(e):
        return (ora.dequantize(synth.expert_gate_up(SEED, layer, e), "Q4_K", (1024, 2048)),
                ora.dequantize(synth.expert_down(SEED, layer, e), "Q6_K", (2048, 512)))
    return dict(router_w=synth.router_weight(SEED, layer), expert_weights=experts, shared=experts(256),
                shared_gate_w=synth.shared_gate_weight(SEED, layer), router_bias=bias)


def forward(ctx, store, layer, x, lw, path, out_dtype=None):
    from willow_v2_b200 import moe
    from willow_v2_b200.lib import lib
    prev = lib.wmoe_set_prefill_threshold(ctx.handle, 1 if path == "gemm" else 1 << 30)
    try:
        return moe.moe_forward(store, layer, x, lw, out_dtype=out_dtype, return_routing=True)
    finally:
        lib.wmoe_set_prefill_threshold(ctx.handle, prev)


@pytest.mark.parametrize("T,zipf", [(300, False), (1024, True)])
def test_gemm_path_matches_gemv_path_and_oracle(model, T, zipf):
    import torch
    ctx, store = model
    bias = synth.zipf_bias(SEED) if zipf else None
    lw = layer_weights(1, bias)
    x = torch.from_numpy(synth.hidden(SEED, T, step=50 + T)).cuda()
    g, gw, gsel = forward(ctx, store, 1, x, lw, "gemm")
    v, vw, vsel = forward(ctx, store, 1, x, lw, "gemv")
    torch.cuda.synchronize()
    ctx.check_device()
    assert torch.equal(gsel, vsel) and torch.equal(gw, vw)  # routing is shared by both paths
    err_paths = rel_l2(g.cpu().numpy(), v.cpu().numpy())
    idx = [0, 1, T // 2, T - 1]
    ref = ora.moe(x[idx].cpu().numpy(), **oracle_layer(1, bias))[0]
    err = rel_l2(g[idx].cpu().numpy(), ref)
    assert err < 1e-3 and err < TOL, err
    assert err_paths < 1e-3, err_paths
    if zipf:  # the hottest experts span several 128-token tiles
        counts = np.bincount(gsel.cpu().numpy().reshape(-1), minlength=256)
        assert counts.max() > 128


def test_gemm_path_bf16_input(model):
    import torch
    ctx, store = model
    lw = layer_weights(0)
    x = torch.from_numpy(synth.hidden(SEED, 512, step=61)).to(torch.bfloat16).cuda()
    g = forward(ctx, store, 0, x, lw, "gemm", out_dtype=torch.float32)[0]
    idx = [3, 100, 511]
    ref = ora.moe(x[idx].float().cpu().numpy(), **oracle_layer(0))[0]
    assert rel_l2(g[idx].cpu().numpy(), ref) < 1e-3


def test_gemm_path_config3_size(model):
    """BASELINE configs[3] shape: 4096 tokens, uniform routing (~128 tokens per expert). Sampled tokens against
    the oracle; the whole output against the GEMV path; token order does not change any token's result."""
    import torch
    ctx, store = model
    lw = layer_weights(0)
    x = torch.from_numpy(synth.hidden(SEED, 4096, step=62)).to(torch.bfloat16).cuda()
    g = forward(ctx, store, 0, x, lw, "gemm", out_dtype=torch.float32)[0]
    v = forward(ctx, store, 0, x, lw, "gemv", out_dtype=torch.float32)[0]
    perm = torch.randperm(4096, generator=torch.Generator().manual_seed(1)).cuda()
    gp = forward(ctx, store, 0, x[perm], lw, "gemm", out_dtype=torch.float32)[0]
    torch.cuda.synchronize()
    ctx.check_device()
    assert rel_l2(g.cpu().numpy(), v.cpu().numpy()) < 1e-3
    assert rel_l2(gp.cpu().numpy(), g[perm].cpu().numpy()) < 1e-3
    idx = [0, 2047, 4095]
    ref = ora.moe(x[idx].float().cpu().numpy(), **oracle_layer(0))[0]
    assert rel_l2(g[idx].cpu().numpy(), ref) < 1e-3


def routing_agrees(x, lw, bias, sel_a, sel_b, w_a, w_b):
    """Two routings of the same tokens agree: identical picks except where the float64 logits of the swapped
    experts are within 1e-5 (the parity rule), and weights within 1e-5 where the picks agree."""
    import torch
    logits = x.double() @ lw.router_w.double().T
    if bias is not None:
        logits = logits + torch.from_numpy(bias).cuda().double()
    a, b = sel_a.long(), sel_b.long()
    rows = (a.sort(1).values != b.sort(1).values).any(1)
    for t in rows.nonzero().flatten().tolist():
        only_a = set(a[t].tolist()) - set(b[t].tolist())
        only_b = set(b[t].tolist()) - set(a[t].tolist())
        gap = max(abs(logits[t, i] - logits[t, j]).item() for i in only_a for j in only_b)
        assert gap < 1e-5, (t, only_a, only_b, gap)
    same = ~rows
    assert torch.allclose(w_a[same], w_b[same], rtol=0, atol=1e-5)
    return int(rows.sum())


@pytest.mark.parametrize("T,zipf", [(4096, False), (1024, True), (37, False)])
def test_tensor_core_router_matches_float32_router(model, T, zipf):
    """bf16 tokens with the split router (tcgen05, K split) against the float32 CUDA-core router on the same
    inputs: same routing (up to 1e-5 logit ties), same outputs within the path tolerance."""
    import torch
    from willow_v2_b200 import moe
    ctx, store = model
    bias = synth.zipf_bias(SEED) if zipf else None
    lw = layer_weights(1, bias)
    lw_tc = moe.LayerWeights(**{f: getattr(lw, f) for f in ("router_w", "shared_gate", "shared_gate_up",
                                                             "shared_down", "router_bias")}).prepare(ctx)
    x = torch.from_numpy(synth.hidden(SEED, T, step=70 + T)).to(torch.bfloat16).cuda()
    g, gw, gsel = forward(ctx, store, 1, x, lw_tc, "gemm", out_dtype=torch.float32)
    v, vw, vsel = forward(ctx, store, 1, x, lw, "gemm", out_dtype=torch.float32)
    torch.cuda.synchronize()
    ctx.check_device()
    routing_agrees(x, lw, bias, gsel, vsel, gw, vw)
    assert rel_l2(g.cpu().numpy(), v.cpu().numpy()) < 1e-3
    idx = [0, T // 2, T - 1]
    ref = ora.moe(x[idx].float().cpu().numpy(), **oracle_layer(1, bias))[0]
    assert rel_l2(g[idx].cpu().numpy(), ref) < 1e-3


def test_split_router_terms_sum_to_router(model):
    """wmoe_split_router: three bf16 terms whose float64 sum is the float32 router to ~2^-24 relative."""
    import torch
    from willow_v2_b200 import moe
    ctx, _ = model
    r = torch.from_numpy(synth.router_weight(SEED, 3)).cuda()
    s = moe.split_router(r, ctx)
    torch.cuda.synchronize()
    assert s.shape == (3, 256, 2048) and s.dtype == torch.bfloat16
    assert torch.equal(s[0], r.to(torch.bfloat16))
    total = s.double().sum(0)
    assert ((total - r.double()).abs() <= r.double().abs() * 2.0 ** -23).all()
