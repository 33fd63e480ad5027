"""The GGUF loader (willow_v2_b200/gguf_store.py, the role of gguf/reader.py + gguf/compiler.py for the MoE path).
Model files are written here with llama.cpp's own gguf-py writer: the parser must agree with gguf-py's reader on
every tensor, every expert blob must be the expert's slice of the stacked tensors (gate rows, up rows, down rows,
the pack layout of gguf/compiler.py:69-88), and on the GPU a store and layer weights loaded from a GGUF must give
bit-identical MoE outputs to the synthetic store they were written from."""
import os

import numpy as np
import pytest

gguf = pytest.importorskip("gguf")
from gguf import GGMLQuantizationType as Q  # noqa: E402

from willow_v2_b200 import gguf_store  # noqa: E402

ROW = {Q.Q4_K: 144, Q.Q6_K: 210, Q.Q8_0: 34, Q.IQ2_S: 82, Q.IQ4_NL: 18}
PER = {Q.Q4_K: 256, Q.Q6_K: 256, Q.Q8_0: 32, Q.IQ2_S: 256, Q.IQ4_NL: 32}


def _quant(rng, shape, qt):
    *outer, k = shape
    return rng.integers(0, 256, (*outer, k // PER[qt] * ROW[qt]), dtype=np.uint8)


def write_model(folder, layers=2, E=4, F=256, H=512, fused=False, files=1, down_type=Q.Q6_K, seed=0,
                gate_type=Q.Q4_K):
    """A qwen35moe GGUF (or `files` split files) with random quant bytes; returns the arrays written per layer."""
    rng = np.random.default_rng(seed)
    arrays = []
    per_file = -(-layers // files)
    paths = []
    for f in range(files):
        name = "m.gguf" if files == 1 else f"m-{f + 1:05d}-of-{files:05d}.gguf"
        path = os.path.join(folder, name)
        paths.append(path)
        w = gguf.GGUFWriter(path, "qwen35moe")
        w.add_block_count(layers)
        for layer in range(f * per_file, min(layers, (f + 1) * per_file)):
            a = dict(gate=_quant(rng, (E, F, H), gate_type), up=_quant(rng, (E, F, H), gate_type),
                     down=_quant(rng, (E, H, F), down_type), router=rng.standard_normal((E, H)).astype(np.float32),
                     sgate=rng.standard_normal(H).astype(np.float32), sg=_quant(rng, (F, H), Q.Q4_K),
                     su=_quant(rng, (F, H), Q.Q4_K), sd=_quant(rng, (H, F), Q.Q6_K))
            p = f"blk.{layer}."
            if fused:
                w.add_tensor(p + "ffn_gate_up_exps.weight", np.concatenate([a["gate"], a["up"]], axis=1),
                             raw_dtype=gate_type)
            else:
                w.add_tensor(p + "ffn_gate_exps.weight", a["gate"], raw_dtype=gate_type)
                w.add_tensor(p + "ffn_up_exps.weight", a["up"], raw_dtype=gate_type)
            w.add_tensor(p + "ffn_down_exps.weight", a["down"], raw_dtype=down_type)
            w.add_tensor(p + "ffn_gate_inp.weight", a["router"])
            w.add_tensor(p + "ffn_gate_inp_shexp.weight", a["sgate"])
            w.add_tensor(p + "ffn_gate_shexp.weight", a["sg"], raw_dtype=Q.Q4_K)
            w.add_tensor(p + "ffn_up_shexp.weight", a["su"], raw_dtype=Q.Q4_K)
            w.add_tensor(p + "ffn_down_shexp.weight", a["sd"], raw_dtype=Q.Q6_K)
            arrays.append(a)
        w.write_header_to_file()
        w.write_kv_data_to_file()
        w.write_tensors_to_file()
        w.close()
    return paths[0], arrays


def test_parser_matches_gguf_py(tmp_path):
    path, _ = write_model(str(tmp_path))
    meta, tensors = gguf_store.read_gguf(path)
    assert meta["general.architecture"] == "qwen35moe" and meta["qwen35moe.block_count"] == 2
    ref = gguf.GGUFReader(path)
    assert len(ref.tensors) == len(tensors)
    for t in ref.tensors:
        ours = tensors[t.name]
        assert ours.offset == t.data_offset, t.name
        assert ours.shape == tuple(int(d) for d in reversed(t.shape)), t.name
        assert ours.type == Q(t.tensor_type).name, t.name
        assert ours.nbytes == t.n_bytes, t.name


@pytest.mark.parametrize("fused,files", [(False, 1), (True, 1), (False, 2)])
def test_expert_blobs_are_the_pack_layout(tmp_path, fused, files):
    """blob(layer, e) = gate rows of e ‖ up rows of e ‖ down rows of e, for separate, fused and split-file
    models."""
    path, arrays = write_model(str(tmp_path), fused=fused, files=files)
    meta, tensors = gguf_store.read_gguf(path)
    lay = gguf_store.expert_layout(meta, tensors)
    assert (lay.layers, lay.experts, lay.hidden, lay.ffn) == (2, 4, 512, 256)
    files_ = gguf_store._Files()
    try:
        for layer, a in enumerate(arrays):
            for e in range(4):
                blob = gguf_store.expert_blob(files_, lay, layer, e)
                want = np.concatenate([a["gate"][e].ravel(), a["up"][e].ravel(), a["down"][e].ravel()])
                assert blob.size == lay.blob_bytes()
                np.testing.assert_array_equal(blob, want)
    finally:
        files_.close()


def test_q4k_down_layers_are_read(tmp_path):
    """llama.cpp's Q4_K_M files store some layers' ffn_down_exps as Q4_K: such a layer's blob is gate ‖ up ‖ down
    rows of 288 bytes."""
    path, arrays = write_model(str(tmp_path), down_type=Q.Q4_K)
    meta, tensors = gguf_store.read_gguf(path)
    lay = gguf_store.expert_layout(meta, tensors)
    assert lay.down_type(0) == "Q4_K" and lay.blob_bytes(0) == 2 * 256 * 512 // 256 * 144 + 512 * 256 // 256 * 144
    files_ = gguf_store._Files()
    try:
        blob = gguf_store.expert_blob(files_, lay, 1, 3)
        a = arrays[1]
        np.testing.assert_array_equal(blob, np.concatenate([a["gate"][3].ravel(), a["up"][3].ravel(),
                                                            a["down"][3].ravel()]))
    finally:
        files_.close()


def test_unsupported_layout_is_an_error(tmp_path):
    path, _ = write_model(str(tmp_path), down_type=Q.Q8_0)
    meta, tensors = gguf_store.read_gguf(path)
    with pytest.raises(gguf_store.GGUFError, match="ffn_down_exps"):
        gguf_store.expert_layout(meta, tensors)
    bad = tmp_path / "not.gguf"
    bad.write_bytes(b"NOPE" + bytes(64))
    with pytest.raises(gguf_store.GGUFError, match="not a GGUF"):
        gguf_store.read_gguf(str(bad))
    with pytest.raises(gguf_store.GGUFError, match="missing"):
        gguf_store.read_gguf(str(tmp_path / "x-00001-of-00003.gguf"))


@pytest.mark.parametrize("fused", [False, True])
def test_typed_layer_views(tmp_path, fused):
    """A layer of IQ2_S gate/up and IQ4_NL down experts read into one buffer: each expert's GGMLWeight views hold its
    gate ‖ up rows and its down rows, at byte offsets of one base (what gemv_batch / gemv_combine take)."""
    path, arrays = write_model(str(tmp_path), gate_type=Q.IQ2_S, down_type=Q.IQ4_NL, fused=fused)
    tl = gguf_store.typed_layer(path, 1, device="cpu")
    a = arrays[1]
    assert (tl.gate_up_type, tl.down_type, tl.hidden, tl.ffn) == ("IQ2_S", "IQ4_NL", 512, 256)
    assert tl.expert_bytes == 2 * 256 * 512 // 256 * 82 + 512 * 256 // 32 * 18
    for e, (gu, dn) in enumerate(tl.experts):
        assert (gu.type_name, gu.shape, dn.type_name, dn.shape) == ("IQ2_S", (512, 512), "IQ4_NL", (512, 256))
        np.testing.assert_array_equal(gu.raw.numpy(), np.concatenate([a["gate"][e].ravel(), a["up"][e].ravel()]))
        np.testing.assert_array_equal(dn.raw.numpy(), a["down"][e].ravel())
        base_gu, off_gu = gu.raw._base, gu.raw.storage_offset()
        assert base_gu is not None and base_gu.data_ptr() == tl.base.data_ptr()
        assert off_gu == e * tl.expert_bytes and dn.raw.storage_offset() == off_gu + gu.raw.numel()
    with pytest.raises(gguf_store.GGUFError, match="no ffn_down_exps|expected ffn_gate_exps"):
        gguf_store.typed_layer(path, 7, device="cpu")


def test_truncated_files_are_errors(tmp_path):
    """A file cut inside its header, or inside a tensor's data, raises GGUFError naming the problem."""
    path, _ = write_model(str(tmp_path), layers=1)
    data = open(path, "rb").read()
    head = tmp_path / "head.gguf"
    head.write_bytes(data[:200])
    with pytest.raises(gguf_store.GGUFError, match="truncated or corrupt header"):
        gguf_store.read_gguf(str(head))
    cut = tmp_path / "cut.gguf"
    cut.write_bytes(data[:-1000])
    with pytest.raises(gguf_store.GGUFError, match="runs past the end"):
        gguf_store.read_gguf(str(cut))


def test_typed_tensors_have_sizes(tmp_path):
    """Tensors of the typed kernels' ggml types get their byte sizes (the store still loads Q4_K / Q6_K experts
    only, and names the first tensor of another type)."""
    path, arrays = write_model(str(tmp_path), layers=1, down_type=Q.Q8_0)
    _, tensors = gguf_store.read_gguf(path)
    down = tensors["blk.0.ffn_down_exps.weight"]
    assert down.type == "Q8_0" and down.nbytes == arrays[0]["down"].size


@pytest.mark.gpu
def test_gguf_model_runs_like_the_store_it_came_from(tmp_path):
    """One full-size layer (256 experts of H 2048, F 512) written to a GGUF from the synthetic store and loaded back:
    the store blobs and the MoE outputs (decode kernel at 1 token, grouped GEMMs at 64) are bit-identical."""
    import torch
    from willow_v2_b200 import moe, synth
    torch.cuda.set_device(0)
    ctx = moe.Context(0)
    src = moe.ExpertStore(1, ctx=ctx)
    src.fill_synthetic(0)
    blobs = np.stack([src.download(0, e) for e in range(256)])
    gu_bytes = 1024 * 8 * 144
    w = gguf.GGUFWriter(str(tmp_path / "m.gguf"), "qwen35moe")
    w.add_block_count(1)
    w.add_tensor("blk.0.ffn_gate_exps.weight", blobs[:, :gu_bytes // 2].reshape(256, 512, 1152), raw_dtype=Q.Q4_K)
    w.add_tensor("blk.0.ffn_up_exps.weight", blobs[:, gu_bytes // 2:gu_bytes].reshape(256, 512, 1152),
                 raw_dtype=Q.Q4_K)
    w.add_tensor("blk.0.ffn_down_exps.weight", blobs[:, gu_bytes:].reshape(256, 2048, 420), raw_dtype=Q.Q6_K)
    w.add_tensor("blk.0.ffn_gate_inp.weight", synth.router_weight(0, 0))
    w.add_tensor("blk.0.ffn_gate_inp_shexp.weight", synth.shared_gate_weight(0, 0))
    sgu, sdn = synth.expert_gate_up(0, 0, 256), synth.expert_down(0, 0, 256)
    w.add_tensor("blk.0.ffn_gate_shexp.weight", sgu.reshape(1024, 1152)[:512], raw_dtype=Q.Q4_K)
    w.add_tensor("blk.0.ffn_up_shexp.weight", sgu.reshape(1024, 1152)[512:], raw_dtype=Q.Q4_K)
    w.add_tensor("blk.0.ffn_down_shexp.weight", sdn.reshape(2048, 420), raw_dtype=Q.Q6_K)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    store, layers = gguf_store.load(str(tmp_path / "m.gguf"), ctx=ctx)
    for e in (0, 77, 255):
        np.testing.assert_array_equal(store.download(0, e), blobs[e])
    ref_lw = moe.LayerWeights(router_w=torch.from_numpy(synth.router_weight(0, 0)).cuda(),
                              shared_gate=torch.from_numpy(synth.shared_gate_weight(0, 0)).cuda(),
                              shared_gate_up=torch.from_numpy(sgu.reshape(-1)).cuda(),
                              shared_down=torch.from_numpy(sdn.reshape(-1)).cuda()).prepare(ctx)
    for T in (1, 64):
        x = torch.from_numpy(synth.hidden(0, T, step=5)).cuda()
        a = moe.moe_forward(store, 0, x, layers[0])
        b = moe.moe_forward(src, 0, x, ref_lw)
        torch.cuda.synchronize()
        assert torch.equal(a, b), T
    ctx.check_device()
    store.close()
    src.close()
