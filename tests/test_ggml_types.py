"""Typed expert kernels over every ggml type of willow's Metal path (gguf/metal.py:295), against the oracle.

CPU: the numpy restatement (oracle/ggml_types.py) reproduces the golden values willow's own gguf/quants.py
produced (tests/golden/make_golden_types.py) bit for bit, and the library's row sizes match the block table.
GPU: wmoe_dequant is bit-identical to the oracle for every type (f32; bf16 = its round-to-nearest-even);
wmoe_gemv / gemv_batch / gemv_combine (through willow_v2_b200.ggml, the mirror of gguf/metal.py; integer dot
products on int16 activations) match the oracle's float32 products within the stated tolerances; GGMLWeight runs
F.linear on both paths (gemv, dequant + matmul)."""
import os

import numpy as np
import pytest

from conftest import REPO
from oracle import ggml_types as G

GOLDEN = os.path.join(REPO, "tests", "golden", "ggml_types.npz")
SEED = 5
TOL_F32 = 2e-5   # relative L2 of float32 outputs (same products, another summation order)
# the GEMV kernels take activations as int16 with a power-of-two scale per 32 values (exact for bf16 values within
# 2^7 of their block's largest; smaller ones round at 2^-15 of it): float32 outputs within this relative L2
TOL_GEMV = 2e-4
TOL_BF16 = 5e-3  # relative L2 of bf16 outputs (one bf16 rounding: <= 2^-9 relative per element)


def random_blocks(type_name: str, n: int, seed: int) -> np.ndarray:
    """n blocks of random bytes with the fp16 scales drawn from U[1e-3, 4e-3] (finite, like real weights)."""
    _, size = G.BLOCKS[type_name]
    rng = np.random.default_rng(seed)
    b = rng.integers(0, 256, (n, size), dtype=np.uint8)
    d_at = 208 if type_name == "Q6_K" else 0
    b[:, d_at:d_at + 2] = rng.uniform(1e-3, 4e-3, n).astype(np.float16).view(np.uint8).reshape(n, 2)
    if type_name == "Q4_K":
        b[:, 2:4] = rng.uniform(1e-3, 4e-3, n).astype(np.float16).view(np.uint8).reshape(n, 2)
    return b


def matrix(type_name: str, rows: int, k: int, seed: int) -> np.ndarray:
    elements, _ = G.BLOCKS[type_name]
    return random_blocks(type_name, rows * k // elements, seed).reshape(-1)


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


# ------------------------------------------------------------------------------------------------ CPU


@pytest.mark.parametrize("type_name", G.TYPES)
def test_oracle_matches_willow_golden(type_name):
    g = np.load(GOLDEN)
    blocks, want = g["blocks_" + type_name], g["values_" + type_name]
    got = G.DEQUANTIZERS[type_name](blocks).astype(np.float32)
    np.testing.assert_array_equal(got.view(np.uint32), want.astype(np.float32).view(np.uint32))


def test_row_bytes_match_the_block_table():
    from willow_v2_b200 import ggml
    from willow_v2_b200.lib import GGML_TYPES, lib
    for name in G.TYPES:
        elements, size = G.BLOCKS[name]
        assert ggml.BLOCKS[name] == (elements, size)
        for k in (256, 512, 2048):
            assert lib.wmoe_ggml_row_bytes(GGML_TYPES[name], k) == k // elements * size == ggml.row_bytes(name, k)
        assert lib.wmoe_ggml_row_bytes(GGML_TYPES[name], elements + 32 if elements > 32 else 16) == 0
    assert lib.wmoe_ggml_row_bytes(2, 256) == 0  # Q4_0: not a type of these kernels


def test_unsupported_types_are_refused_without_a_gpu():
    from willow_v2_b200 import ggml
    from willow_v2_b200.lib import ERR_INVALID, lib
    with pytest.raises(NotImplementedError, match="IQ1_S"):
        ggml.GGMLWeight(np.zeros(1, np.uint8), "IQ1_S", (1, 256))
    assert lib.wmoe_gemv(None, 8, None, 1, 256, None, 1, 1, None, 1, None) == ERR_INVALID
    assert lib.wmoe_gemv_combine(None, 8, None, None, 1, 1, 1, 256, None, None, 1, None, None) == ERR_INVALID
    assert lib.wmoe_batched_decode_experts(None, 12, 14, 2048, 512, None, None, None, 8, 8, None, None, None,
                                           None) == ERR_INVALID


def test_wrappers_refuse_bad_arguments_without_a_gpu():
    """The Python mirror of gguf/metal.py checks its arguments before any CUDA call: host tensors, too many tokens,
    short buffers, offsets, positions and perm entries outside their arrays."""
    import torch
    from willow_v2_b200 import ggml
    raw = torch.zeros(64 * ggml.row_bytes("Q8_0", 256), dtype=torch.uint8)
    x = torch.zeros(1, 256, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        ggml.gemv(raw, "Q8_0", (64, 256), x)
    with pytest.raises(ValueError, match="1..8 tokens"):
        ggml.gemv(raw, "Q8_0", (64, 256), torch.zeros(9, 256))
    with pytest.raises(ValueError, match="fewer bytes"):
        ggml.gemv(raw[:100], "Q8_0", (64, 256), x)
    out = torch.zeros(2, 64)
    with pytest.raises(ValueError, match="one position per offset"):
        ggml.gemv_batch(raw, "Q8_0", (64, 256), x, [0], [0, 1], out)
    with pytest.raises(ValueError, match="outside base"):
        ggml.gemv_batch(raw, "Q8_0", (64, 256), x, [2], [0], out)
    with pytest.raises(ValueError, match="position outside out"):
        ggml.gemv_batch(raw, "Q8_0", (64, 256), x, [0], [2], out)
    with pytest.raises(ValueError, match="CUDA"):
        ggml.gemv_batch(raw, "Q8_0", (64, 256), x, [0], [1], out)
    w = torch.ones(4, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="at least one"):
        ggml.gemv_combine(raw, "Q8_0", (64, 256), x, [], w, [])
    with pytest.raises(ValueError, match="perm entry outside"):
        ggml.gemv_combine(raw, "Q8_0", (64, 256), x, [0], w, [4])
    with pytest.raises(ValueError, match="CUDA"):
        ggml.dequantize_gpu(raw, "Q8_0", (64, 256))
    # the one-call expert step (engines/base.py:492-532) and expert_gate
    gu_b, dn_b = 2 * 128 * ggml.row_bytes("Q8_0", 256), 256 * ggml.row_bytes("Q8_0", 128)
    slab = torch.zeros(2 * (gu_b + dn_b), dtype=torch.uint8)
    xb = torch.zeros(256, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="at least one"):
        ggml.batched_decode_experts(slab, "Q8_0", "Q8_0", 128, xb, [0], [], w, [0])
    with pytest.raises(ValueError, match="gate_up offset"):
        ggml.batched_decode_experts(slab, "Q8_0", "Q8_0", 128, xb, [slab.numel()], [gu_b], w, [0])
    with pytest.raises(ValueError, match="down offset"):
        ggml.batched_decode_experts(slab, "Q8_0", "Q8_0", 128, xb, [0], [slab.numel() - 1], w, [0])
    with pytest.raises(ValueError, match="perm entry outside"):
        ggml.batched_decode_experts(slab, "Q8_0", "Q8_0", 128, xb, [0], [gu_b], w, [4])
    with pytest.raises(ValueError, match="CUDA"):
        ggml.batched_decode_experts(slab, "Q8_0", "Q8_0", 128, xb, [0], [gu_b], w, [3])
    with pytest.raises(ValueError, match="bf16"):
        ggml.expert_gate(torch.zeros(2, 64))
    with pytest.raises(ValueError, match="CUDA"):
        ggml.expert_gate(torch.zeros(2, 64, dtype=torch.bfloat16))
    with pytest.raises(NotImplementedError, match="Q4_0"):
        ggml.dequantize_gpu(raw, "Q4_0", (64, 256))
    # f16 activations widen to f32 (exact) rather than rounding to bf16
    h = torch.tensor([1.0 + 2.0 ** -10, -3.0009765625], dtype=torch.float16)
    assert ggml._act(h).dtype == torch.float32 and torch.equal(ggml._act(h), h.float())


def test_combine_oracle_rounds_like_torch_bf16():
    """The oracle's bf16 combine agrees with the same steps done in torch bf16 (engines/base.py:431-443)."""
    import torch
    rng = np.random.default_rng(3)
    k, rows, n = 256, 8, 3
    mats = [matrix("Q8_0", rows, k, 30 + i) for i in range(n)]
    x = G.bf16(rng.standard_normal((n, k)).astype(np.float32))
    w = G.bf16(rng.uniform(0, 1, 4).astype(np.float32))
    perm = [2, 0, 3]
    got = G.gemv_combine_bf16(mats, "Q8_0", (rows, k), x, w, perm)
    parts = [torch.from_numpy(G.dequantize(m, "Q8_0", (rows, k)) @ x[i]).to(torch.bfloat16) for i, m in enumerate(mats)]
    scaled = [p * torch.from_numpy(w)[perm[i]].to(torch.bfloat16) for i, p in enumerate(parts)]
    total = scaled[0]
    for s in scaled[1:]:
        total = total + s
    np.testing.assert_array_equal(got, total.float().numpy())


# ------------------------------------------------------------------------------------------------ GPU


@pytest.fixture(scope="module")
def ctx():
    import torch
    from willow_v2_b200 import moe
    torch.cuda.set_device(0)
    return moe.default_context()


@pytest.mark.gpu
@pytest.mark.parametrize("type_name", G.TYPES)
def test_dequant_is_bit_exact(ctx, type_name):
    import torch
    from willow_v2_b200 import ggml
    g = np.load(GOLDEN)
    blocks = np.concatenate([g["blocks_" + type_name], random_blocks(type_name, 300, SEED)])
    elements, _ = G.BLOCKS[type_name]
    raw = torch.from_numpy(blocks.reshape(-1).copy()).cuda()
    want = G.dequantize(blocks, type_name, (blocks.shape[0], elements))
    got = ggml.dequantize_gpu(raw, type_name, (blocks.shape[0], elements), torch.float32, ctx).cpu().numpy()
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    got_bf16 = ggml.dequantize_gpu(raw, type_name, (blocks.shape[0], elements), torch.bfloat16, ctx)
    finite = np.isfinite(want)
    np.testing.assert_array_equal(got_bf16.float().cpu().numpy()[finite], G.bf16(want)[finite])
    ctx.check_device()


@pytest.mark.gpu
@pytest.mark.parametrize("type_name", G.TYPES)
def test_gemv_matches_oracle(ctx, type_name):
    """gate_up-shaped [1024, 2048] (32 lanes per row) and down-shaped [2048, 512] (16 lanes) matrices, 1, 3 and 8
    tokens, bf16 and f32 activations."""
    import torch
    from willow_v2_b200 import ggml
    rng = np.random.default_rng(11)
    for rows, k in ((1024, 2048), (2048, 512), (64, 256)):
        raw_np = matrix(type_name, rows, k, SEED + rows)
        raw = torch.from_numpy(raw_np).cuda()
        w = G.dequantize(raw_np, type_name, (rows, k))
        for tokens in (1, 3, 8):
            x32 = rng.standard_normal((tokens, k)).astype(np.float32)
            xb = G.bf16(x32)
            y = ggml.gemv(raw, type_name, (rows, k), torch.from_numpy(xb).cuda().to(torch.bfloat16),
                          out_dtype=torch.float32, ctx=ctx)
            assert rel_l2(y.cpu().numpy(), xb @ w.T) < TOL_GEMV, (rows, k, tokens)
            yb = ggml.gemv(raw, type_name, (rows, k), torch.from_numpy(x32).cuda(), ctx=ctx)
            assert yb.dtype == torch.bfloat16
            assert rel_l2(yb.float().cpu().numpy(), x32 @ w.T) < TOL_BF16, (rows, k, tokens)
    ctx.check_device()


@pytest.mark.gpu
@pytest.mark.parametrize("type_name", ["IQ2_S", "Q5_0", "Q6_K"])
def test_gemv_batch_positions_and_combine(ctx, type_name):
    """Five experts in one slab at byte offsets: gemv_batch writes each to its position; gemv_combine's bf16
    result matches the oracle's bf16 restatement, its float32 mode the float32 sum."""
    import torch
    from willow_v2_b200 import ggml
    from willow_v2_b200.lib import F32, lib, check
    rows, k, n = 2048, 512, 5
    rb = G.row_bytes(type_name, k)
    mats = [matrix(type_name, rows, k, 70 + i) for i in range(n)]
    slab_np = np.zeros(n * rows * rb + 2 * 7, dtype=np.uint8)
    offsets = [2 * 7 + i * rows * rb for i in range(n)]  # even, not 16-aligned: exercises the staged head/tail
    for o, m in zip(offsets, mats):
        slab_np[o:o + m.size] = m
    slab = torch.from_numpy(slab_np).cuda()
    rng = np.random.default_rng(12)
    x = G.bf16(rng.standard_normal(k).astype(np.float32))
    positions = [3, 0, 6, 1, 5]
    out = torch.zeros(7, rows, dtype=torch.float32, device="cuda")
    ggml.gemv_batch(slab, type_name, (rows, k), torch.from_numpy(x).cuda().to(torch.bfloat16), offsets, positions,
                    out, ctx=ctx)
    got = out.cpu().numpy()
    for i, m in enumerate(mats):
        assert rel_l2(got[positions[i]], G.dequantize(m, type_name, (rows, k)) @ x) < TOL_GEMV, i
    assert not got[2].any() and not got[4].any()  # untouched positions

    xs = G.bf16(rng.standard_normal((n, k)).astype(np.float32))
    route = G.bf16(rng.uniform(0.02, 0.3, 8).astype(np.float32))
    perm = [4, 1, 7, 0, 2]
    y = ggml.gemv_combine(slab, type_name, (rows, k), torch.from_numpy(xs).cuda().to(torch.bfloat16), offsets,
                          torch.from_numpy(route).cuda().to(torch.bfloat16), perm, ctx=ctx)
    ref = G.gemv_combine_bf16(mats, type_name, (rows, k), xs, route, perm)
    yb = y.float().cpu().numpy().reshape(-1)
    # the same bf16 steps; a float32 dot product summed in another order can land on the other side of a bf16
    # rounding boundary, so a few elements may differ by a bf16 step
    assert np.mean(yb == ref) > 0.95 and rel_l2(yb, ref) < 5e-3
    # float32 mode: sum_i route[perm[i]] * (W_i x_i) without rounding
    ptrs = torch.tensor([slab.data_ptr() + o for o in offsets], dtype=torch.int64).cuda()
    pm = torch.tensor(perm, dtype=torch.int64).cuda()
    xs_t, rw_t = torch.from_numpy(xs).cuda(), torch.from_numpy(route).cuda()
    y32 = torch.empty(rows, dtype=torch.float32, device="cuda")
    check(ctx.handle, lib.wmoe_gemv_combine(ctx.handle, ggml._type_id(type_name), ggml._p(ptrs), ggml._p(pm), n, 8,
                                            rows, k, ggml._p(xs_t), ggml._p(rw_t), F32, ggml._p(y32),
                                            ggml._stream()))
    ref32 = sum(route[perm[i]] * (G.dequantize(m, type_name, (rows, k)) @ xs[i]) for i, m in enumerate(mats))
    assert rel_l2(y32.cpu().numpy(), ref32) < TOL_GEMV
    ctx.check_device()


@pytest.mark.gpu
def test_expert_gate_rounds_like_torch(ctx):
    """wmoe_expert_gate gives the bits of willow's expert_gate on bf16 tensors, F.silu(gate) * up
    (engines/base.py:99-102), over a wide range of values (large negative and positive gates, tiny ups)."""
    import torch
    import torch.nn.functional as F
    from willow_v2_b200 import ggml
    g = torch.Generator().manual_seed(3)
    gu = (torch.randn(64, 1024, generator=g) * torch.logspace(-3, 1.5, 1024)).to(torch.bfloat16).cuda()
    got = ggml.expert_gate(gu, ctx=ctx)
    want = F.silu(gu[:, :512]) * gu[:, 512:]
    torch.cuda.synchronize()
    assert torch.equal(got, want)


@pytest.mark.gpu
@pytest.mark.parametrize("gu_type,dn_type", [("Q4_K", "Q6_K"), ("IQ2_S", "IQ2_S"), ("Q8_0", "Q4_K")])
def test_batched_decode_experts(ctx, gu_type, dn_type):
    """wmoe_batched_decode_experts (engines/base.py:492-532 in one call) gives the bits of its three steps run
    through the Python API one after another: gemv_batch into bf16 rows, willow's expert_gate F.silu(gate) * up on
    bf16 tensors (engines/base.py:99-102), gemv_combine. The chain is also checked against the oracle's bf16
    restatement (the last bf16 rounding of a float32 dot product summed in another order may differ by a step)."""
    import torch
    import torch.nn.functional as F
    from willow_v2_b200 import ggml
    H, Fd, n = 2048, 512, 8
    gu_b = 2 * Fd * G.row_bytes(gu_type, H)
    dn_b = H * G.row_bytes(dn_type, Fd)
    gus = [matrix(gu_type, 2 * Fd, H, 300 + i) for i in range(n)]
    dns = [matrix(dn_type, H, Fd, 400 + i) for i in range(n)]
    slab_np = np.concatenate([np.concatenate([g, d]) for g, d in zip(gus, dns)])
    slab = torch.from_numpy(slab_np).cuda()
    offs = [i * (gu_b + dn_b) for i in range(n)]
    rng = np.random.default_rng(21)
    x = torch.from_numpy(rng.standard_normal(H).astype(np.float32)).to(torch.bfloat16).cuda()
    route = torch.from_numpy(rng.uniform(0.02, 0.3, 8).astype(np.float32)).to(torch.bfloat16).cuda()
    perm = [3, 0, 6, 1, 5, 2, 7, 4]
    y = ggml.batched_decode_experts(slab, gu_type, dn_type, Fd, x, offs, [o + gu_b for o in offs], route, perm,
                                    ctx=ctx)
    gate_up = torch.empty(n, 2 * Fd, dtype=torch.bfloat16, device="cuda")
    ggml.gemv_batch(slab, gu_type, (2 * Fd, H), x, offs, list(range(n)), gate_up, ctx=ctx)
    hidden = (F.silu(gate_up[:, :Fd]) * gate_up[:, Fd:]).contiguous()
    want = ggml.gemv_combine(slab, dn_type, (H, Fd), hidden, [o + gu_b for o in offs], route, perm, ctx=ctx)
    torch.cuda.synchronize()
    ctx.check_device()
    assert y.shape == (1, H) and y.dtype == torch.bfloat16
    assert torch.equal(y, want)
    # the oracle's chain
    xb = x.float().cpu().numpy()
    g = np.stack([G.bf16(G.dequantize(m, gu_type, (2 * Fd, H)) @ xb) for m in gus])
    gt = torch.from_numpy(g).to(torch.bfloat16)
    hid = (F.silu(gt[:, :Fd]) * gt[:, Fd:]).float().numpy()
    ref = G.gemv_combine_bf16(dns, dn_type, (H, Fd), hid, route.float().cpu().numpy(), perm)
    assert rel_l2(y.float().cpu().numpy().reshape(-1), ref) < 1e-2


@pytest.mark.gpu
def test_ggml_weight_linear_both_paths(ctx):
    import torch
    import torch.nn.functional as F
    from willow_v2_b200 import ggml
    rows, k = 512, 2048
    raw_np = matrix("IQ3_XXS", rows, k, 91)
    w = G.dequantize(raw_np, "IQ3_XXS", (rows, k))
    weight = ggml.GGMLWeight(torch.from_numpy(raw_np), "IQ3_XXS", (rows, k))  # CPU bytes: copied on first use
    rng = np.random.default_rng(4)
    for tokens in (2, 40):  # gemv path, then dequant + bf16 matmul
        x = torch.from_numpy(G.bf16(rng.standard_normal((1, tokens, k)).astype(np.float32))).cuda().to(torch.bfloat16)
        y = F.linear(x, weight)
        assert y.shape == (1, tokens, rows) and y.dtype == torch.bfloat16
        ref = x.float().cpu().numpy()[0] @ w.T
        assert rel_l2(y.float().cpu().numpy()[0], ref) < 1e-2, tokens
    ctx.check_device()


@pytest.mark.gpu
def test_bad_position_sets_device_status(ctx):
    """A position past n_out is caught on the device: nothing is written and the status word says so."""
    import torch
    from willow_v2_b200 import ggml
    from willow_v2_b200.lib import F32, WmoeError, lib, check
    rows, k = 64, 256
    raw = torch.from_numpy(matrix("Q8_0", rows, k, 5)).cuda()
    ptrs = torch.tensor([raw.data_ptr()], dtype=torch.int64).cuda()
    pos = torch.tensor([9], dtype=torch.int64).cuda()
    x = torch.ones(k, dtype=torch.float32, device="cuda")
    y = torch.zeros(2, rows, dtype=torch.float32, device="cuda")
    ctx.check_device()
    check(ctx.handle, lib.wmoe_gemv_batch(ctx.handle, 8, ggml._p(ptrs), ggml._p(pos), 1, 2, rows, k, ggml._p(x), F32,
                                          ggml._p(y), F32, ggml._stream()))
    with pytest.raises(WmoeError):
        ctx.check_device()
    assert not y.any()
