"""Expert parallelism on one GPU: `world` ranks emulated in one process, each with its own store holding its block
of experts (wmoe_store_create_range); the all-to-all exchanges are done by slicing and concatenating the buffers
exactly as all_to_all_single would. The combined output must equal the single-GPU moe_forward bit for bit (same
routing, same per-row GEMM arithmetic, same combine order), and match the oracle."""
import numpy as np
import pytest

from oracle import moe_oracle as ora
from willow_v2_b200 import synth

pytestmark = pytest.mark.gpu
SEED = 0
LAYER = 0


def rel_l2(a, b):
    a, b = np.asarray(a, dtype=np.float64), np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@pytest.fixture(scope="module")
def base():
    import torch
    from willow_v2_b200 import moe
    torch.cuda.set_device(0)
    ctx = moe.Context(0)
    full = moe.ExpertStore(1, ctx=ctx)
    full.fill_synthetic(SEED)
    lw = moe.LayerWeights(
        router_w=torch.from_numpy(synth.router_weight(SEED, LAYER)).cuda(),
        shared_gate=torch.from_numpy(synth.shared_gate_weight(SEED, LAYER)).cuda(),
        shared_gate_up=torch.from_numpy(synth.expert_gate_up(SEED, LAYER, 256).reshape(-1)).cuda(),
        shared_down=torch.from_numpy(synth.expert_down(SEED, LAYER, 256).reshape(-1)).cuda()).prepare(ctx)
    torch.cuda.synchronize()
    return ctx, full, lw


def emulate(ctx, stores, xs, lw, world):
    """One expert-parallel layer over `world` emulated ranks; returns each rank's output."""
    from willow_v2_b200 import moe
    plans = [moe.ep_route_plan(ctx, world, xs[r], lw) for r in range(world)]
    counts = [p.counts.cpu().numpy() for p in plans]  # [2, world] per sender: rows, pairs to each rank
    row_off = [np.concatenate([[0], np.cumsum(c[0])]) for c in counts]
    pair_off = [np.concatenate([[0], np.cumsum(c[1])]) for c in counts]
    ys, recv_pairs_of = [], []
    for d in range(world):
        r_rows = [int(counts[s][0][d]) for s in range(world)]
        r_pairs = [int(counts[s][1][d]) for s in range(world)]
        import torch
        recv_buf = torch.cat([plans[s].send_buf[row_off[s][d]:row_off[s][d + 1]] for s in range(world)])
        recv_pl = torch.cat([plans[s].pair_list[pair_off[s][d]:pair_off[s][d + 1]] for s in range(world)])
        ys.append(moe.ep_experts(stores[d], LAYER, world, r_rows, r_pairs, recv_buf, recv_pl, xs[d], lw))
        recv_pairs_of.append(r_pairs)
    outs = []
    import torch
    for s in range(world):
        blocks = []
        for d in range(world):
            start = sum(recv_pairs_of[d][:s])
            blocks.append(ys[d][start:start + recv_pairs_of[d][s]])
        y_ret = torch.cat(blocks)
        P_r = sum(recv_pairs_of[s])
        outs.append(moe.ep_combine(ctx, plans[s], y_ret, ys[s][P_r:], torch.float32))
    return outs, plans


@pytest.mark.parametrize("world,tokens,zipf", [(1, 512, False), (2, 1024, False), (4, 2048, True), (8, 2048, False)])
def test_ep_emulated_ranks_match_single_gpu(base, world, tokens, zipf):
    import torch
    from willow_v2_b200 import moe
    from willow_v2_b200.lib import lib
    ctx, full, lw = base
    if zipf:
        lw = moe.LayerWeights(router_w=lw.router_w, shared_gate=lw.shared_gate, shared_gate_up=lw.shared_gate_up,
                              shared_down=lw.shared_down, router_split=lw.router_split,
                              router_bias=torch.from_numpy(synth.zipf_bias(SEED)).cuda())
    per = 256 // world
    stores = []
    for r in range(world):
        st = moe.ExpertStore(1, ctx=ctx, expert_range=(r * per, (r + 1) * per))
        st.fill_synthetic(SEED)
        stores.append(st)
    x = torch.from_numpy(synth.hidden(SEED, tokens, step=90 + world)).to(torch.bfloat16).cuda()
    xs = list(x.chunk(world))
    prev = lib.wmoe_set_prefill_threshold(ctx.handle, 1)  # the single-GPU reference on the GEMM path too
    try:
        ref, ref_w, ref_sel = moe.moe_forward(full, LAYER, x, lw, out_dtype=torch.float32, return_routing=True)
    finally:
        lib.wmoe_set_prefill_threshold(ctx.handle, prev)
    outs, plans = emulate(ctx, stores, xs, lw, world)
    torch.cuda.synchronize()
    ctx.check_device()
    out = torch.cat(outs)
    assert torch.equal(torch.cat([p.topk_idx for p in plans]), ref_sel)
    assert torch.equal(out, ref)
    counts = sum(p.counts.cpu() for p in plans)
    assert int(counts[1].sum()) == tokens * 8  # every pick sent exactly once
    assert int(counts[0].sum()) <= tokens * min(8, world)  # one row per (token, destination)
    idx = [0, tokens // 2, tokens - 1]
    bias = synth.zipf_bias(SEED) if zipf else None

    def experts(e):
        return (ora.dequantize(synth.expert_gate_up(SEED, LAYER, e), "Q4_K", (1024, 2048)),
                ora.dequantize(synth.expert_down(SEED, LAYER, e), "Q6_K", (2048, 512)))
    want = ora.moe(x[idx].float().cpu().numpy(), synth.router_weight(SEED, LAYER), experts, experts(256),
                   synth.shared_gate_weight(SEED, LAYER), router_bias=bias)[0]
    assert rel_l2(out[idx].cpu().numpy(), want) < 1e-3
    for st in stores:
        st.close()


def test_range_store_refuses_other_experts(base):
    import torch
    from willow_v2_b200 import moe
    from willow_v2_b200.lib import WmoeError
    ctx, full, lw = base
    st = moe.ExpertStore(1, ctx=ctx, expert_range=(64, 128))
    st.fill_synthetic(SEED)
    torch.cuda.synchronize()
    assert np.array_equal(st.download(0, 100), full.download(0, 100))
    with pytest.raises(WmoeError):
        st.download(0, 3)
    with pytest.raises(WmoeError):
        st.load_many(0, [3])
    st.close()
