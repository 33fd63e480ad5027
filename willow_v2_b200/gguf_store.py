"""Loads a qwen35moe GGUF file (llama.cpp's format) into this library: every (layer, expert) becomes one store blob
(gate rows, then up rows, then down rows: the expert-pack layout of gguf/compiler.py:69-88,139-197), and each layer's
router, shared expert and shared-expert gate become a moe.LayerWeights.

It replaces, for the MoE path, willow's header reader (gguf/reader.py:106-171) and the expert scan and gate/up fusion
of its pack compiler (gguf/compiler.py:29-88). There is no pack step: the expert bytes go from the memory-mapped
GGUF file straight into the HBM store (or into its pinned host copy when the store is capped). The bytes are not
converted, so the store holds exactly the file's Q4_K / Q6_K blocks.

    from willow_v2_b200 import gguf_store
    store, layers = gguf_store.load(path)                  # every layer's experts + LayerWeights
    out = moe.moe_forward(store, 0, x, layers[0])

The parser needs no GPU (read_gguf, expert_layout); loading does.
"""
import mmap
import os
import re
import struct
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import numpy as np

GGUF_MAGIC = b"GGUF"
DEFAULT_ALIGNMENT = 32  # when the file does not set general.alignment

# ggml type ids whose sizes this loader knows, with (values per block, bytes per block) (gguf/reader.py:14-48): the
# store's Q4_K / Q6_K, the float types of routers and gates, and the other types the typed kernels run
TYPES = {0: ("F32", 1, 4), 1: ("F16", 1, 2), 6: ("Q5_0", 32, 22), 8: ("Q8_0", 32, 34), 12: ("Q4_K", 256, 144),
         14: ("Q6_K", 256, 210), 18: ("IQ3_XXS", 256, 98), 20: ("IQ4_NL", 32, 18), 21: ("IQ3_S", 256, 110),
         22: ("IQ2_S", 256, 82), 23: ("IQ4_XS", 256, 136), 30: ("BF16", 1, 2), 42: ("Q2_0", 64, 18)}
# other ids are still parsed (the header must be walked), their sizes unknown to this loader
_SCALARS = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "?", 10: "Q", 11: "q", 12: "d"}
_STRING, _ARRAY = 8, 9
_SPLIT = re.compile(r"^(.*)-(\d{5})-of-(\d{5})\.gguf$")
_EXPERT = re.compile(r"^blk\.(\d+)\.ffn_(gate|up|down|gate_up)_exps\.weight$")


@dataclass
class Tensor:
    """One tensor of the file: data at `offset` (absolute) in `path`; shape outermost first (the reverse of ggml's
    ne); `type` the ggml type name, or `ggml<id>` for a type this loader has no block size for."""
    name: str
    path: str
    offset: int
    type: str
    shape: Tuple[int, ...]

    @property
    def nbytes(self) -> int:
        for name, per, size in TYPES.values():
            if name == self.type:
                if self.shape[-1] % per:
                    raise ValueError(f"{self.name}: row length {self.shape[-1]} is not a multiple of {per}")
                return int(np.prod(self.shape)) // per * size
        raise ValueError(f"{self.name}: ggml type {self.type} is not one this loader reads")


class GGUFError(ValueError):
    pass


def _read_header(path: str):
    """(metadata, {name: Tensor}) of one file. A truncated or corrupt header, or tensor data that runs past the end of
    the file, raises GGUFError."""
    with open(path, "rb") as f:
        mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
    file_size = len(mm)
    try:
        buf = memoryview(mm)
        pos = 0

        def take(fmt):
            nonlocal pos
            vals = struct.unpack_from("<" + fmt, buf, pos)
            pos += struct.calcsize("<" + fmt)
            return vals if len(vals) > 1 else vals[0]

        def string():
            nonlocal pos
            n = take("Q")
            s = bytes(buf[pos:pos + n]).decode("utf-8", errors="replace")
            pos += n
            return s

        def value(t):
            nonlocal pos
            if t == _STRING:
                return string()
            if t == _ARRAY:
                item, count = take("IQ")
                if item in _SCALARS:
                    fmt = f"{count}{_SCALARS[item]}"
                    vals = list(struct.unpack_from("<" + fmt, buf, pos))
                    pos += struct.calcsize("<" + fmt)
                    return vals
                return [value(item) for _ in range(count)]
            if t not in _SCALARS:
                raise GGUFError(f"{path}: unknown metadata value type {t}")
            return take(_SCALARS[t])

        if bytes(buf[:4]) != GGUF_MAGIC:
            raise GGUFError(f"{path} is not a GGUF file")
        pos = 4
        try:
            version, n_tensors, n_kv = take("IQQ")
            if version < 2:
                raise GGUFError(f"{path} is GGUF version {version}; versions 2 and 3 are supported")
            meta = {}
            for _ in range(n_kv):
                key = string()
                meta[key] = value(take("I"))
            infos = []
            for _ in range(n_tensors):
                name = string()
                n_dims = take("I")
                ne = take(f"{n_dims}Q") if n_dims > 1 else (take("Q"),)
                type_id, offset = take("IQ")
                infos.append((name, tuple(reversed(ne)), type_id, offset))
        except struct.error as e:
            raise GGUFError(f"{path}: truncated or corrupt header ({e})") from None
        align = int(meta.get("general.alignment", DEFAULT_ALIGNMENT))
        data_start = (pos + align - 1) // align * align
    finally:
        buf.release()
        mm.close()
    tensors = {}
    for name, shape, type_id, offset in infos:
        type_name = TYPES[type_id][0] if type_id in TYPES else f"ggml{type_id}"
        t = Tensor(name, path, data_start + offset, type_name, shape)
        if type_id in TYPES and t.offset + t.nbytes > file_size:
            raise GGUFError(f"{name}: its data runs past the end of {path} "
                            f"({t.offset + t.nbytes} > {file_size} bytes)")
        tensors[name] = t
    return meta, tensors


def split_paths(path: str) -> List[str]:
    """Every file of a split model (<name>-00001-of-00003.gguf) given any one of them, else [path]."""
    m = _SPLIT.match(os.path.basename(path))
    if not m:
        return [path]
    base, _, count = m.groups()
    folder = os.path.dirname(path)
    paths = [os.path.join(folder, f"{base}-{i:05d}-of-{count}.gguf") for i in range(1, int(count) + 1)]
    missing = [p for p in paths if not os.path.exists(p)]
    if missing:
        raise GGUFError(f"split GGUF is missing {len(missing)} of {count} files, e.g. {missing[0]}")
    return paths


def read_gguf(path: str):
    """(metadata of the first file, {name: Tensor} over every split file), like gguf/reader.py:162-171."""
    meta, tensors = None, {}
    for p in split_paths(path):
        m, t = _read_header(p)
        meta = m if meta is None else meta
        tensors.update(t)
    return meta, tensors


@dataclass
class ExpertLayout:
    """Where each layer's stacked expert tensors live. gate_up[layer] is one fused tensor or a (gate, up) pair."""
    layers: int
    experts: int
    hidden: int
    ffn: int
    gate_up: Dict[int, Tuple[Tensor, ...]] = field(default_factory=dict)
    down: Dict[int, Tensor] = field(default_factory=dict)

    def down_type(self, layer: int) -> str:
        return self.down[layer].type

    def blob_bytes(self, layer: int = 0) -> int:
        per = 144 if self.down_type(layer) == "Q4_K" else 210
        return 2 * self.ffn * self.hidden // 256 * 144 + self.hidden * self.ffn // 256 * per


def num_layers(meta: dict) -> int:
    """Decoder layers: block_count minus trailing multi-token-prediction layers (gguf/compiler.py:24-27)."""
    arch = meta["general.architecture"]
    return int(meta[f"{arch}.block_count"]) - int(meta.get(f"{arch}.nextn_predict_layers", 0))


def expert_layout(meta: dict, tensors: Dict[str, Tensor]) -> ExpertLayout:
    """Finds every layer's blk.N.ffn_{gate,up,down}_exps (or a fused ffn_gate_up_exps) and checks what this library's
    kernels run: gate/up Q4_K [E, F, H], down Q6_K or Q4_K [E, H, F] (the type may differ per layer, as in llama.cpp's
    Q4_K_M files), the same E, F, H on every layer, H and F multiples of 256. Raises GGUFError naming the first
    tensor that does not fit."""
    n_layers = num_layers(meta)
    parts: Dict[int, Dict[str, Tensor]] = {}
    for name, t in tensors.items():
        m = _EXPERT.match(name)
        if m and int(m.group(1)) < n_layers:
            parts.setdefault(int(m.group(1)), {})[m.group(2)] = t
    if not parts:
        raise GGUFError("no MoE expert tensors (expected names like blk.N.ffn_gate_exps.weight)")
    if sorted(parts) != list(range(n_layers)):
        raise GGUFError(f"expert tensors in layers {sorted(parts)}, expected 0..{n_layers - 1} (dense layers are not "
                        "supported)")
    dims = None
    lay = None
    for layer in range(n_layers):
        p = parts[layer]
        if "gate_up" in p:
            gu = (p["gate_up"],)
        elif "gate" in p and "up" in p:
            gu = (p["gate"], p["up"])
        else:
            raise GGUFError(f"layer {layer}: expected ffn_gate_exps and ffn_up_exps (or ffn_gate_up_exps)")
        if "down" not in p:
            raise GGUFError(f"layer {layer}: no ffn_down_exps")
        for t in gu:
            if t.type != "Q4_K" or len(t.shape) != 3:
                raise GGUFError(f"{t.name}: {t.type} {t.shape}; the kernels run Q4_K [experts, ffn, hidden]")
        down = p["down"]
        if down.type not in ("Q6_K", "Q4_K") or len(down.shape) != 3:
            raise GGUFError(f"{down.name}: {down.type} {down.shape}; the kernels run Q6_K or Q4_K "
                            "[experts, hidden, ffn]")
        E, rows, H = gu[0].shape
        F = rows // 2 if len(gu) == 1 else rows
        if len(gu) == 2 and gu[1].shape != gu[0].shape:
            raise GGUFError(f"layer {layer}: gate {gu[0].shape} and up {gu[1].shape} differ")
        if down.shape != (E, H, F):
            raise GGUFError(f"{down.name}: shape {down.shape}, expected {(E, H, F)}")
        if H % 256 or F % 256:
            raise GGUFError(f"layer {layer}: hidden {H} and ffn {F} must be multiples of 256")
        if dims is None:
            dims = (E, H, F)
            lay = ExpertLayout(n_layers, E, H, F)
        elif dims != (E, H, F):
            raise GGUFError(f"layer {layer}: experts/hidden/ffn {(E, H, F)} differ from layer 0's {dims}")
        lay.gate_up[layer] = gu
        lay.down[layer] = down
    return lay


class _Files:
    """Memory maps of the model's files, opened once."""

    def __init__(self):
        self.maps = {}

    def view(self, t: Tensor, start: int, size: int) -> np.ndarray:
        if t.path not in self.maps:
            with open(t.path, "rb") as f:
                self.maps[t.path] = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        return np.frombuffer(self.maps[t.path], dtype=np.uint8, count=size, offset=t.offset + start)

    def close(self):
        for m in self.maps.values():
            try:
                m.close()
            except BufferError:  # a caller still holds a view; the map goes with it
                pass
        self.maps = {}


def expert_blob(files: _Files, lay: ExpertLayout, layer: int, expert: int) -> np.ndarray:
    """The store blob of one expert: its gate rows, its up rows, its down rows (each the expert's equal slice of the
    stacked tensor; quant blocks never cross rows, so the slices split cleanly)."""
    pieces = []
    for t in lay.gate_up[layer]:
        per = t.nbytes // lay.experts
        pieces.append(files.view(t, expert * per, per))
    d = lay.down[layer]
    per = d.nbytes // lay.experts
    pieces.append(files.view(d, expert * per, per))
    return np.concatenate(pieces)


def load_experts(path: str, ctx=None, cap_bytes: int = 0, expert_range: Optional[Tuple[int, int]] = None):
    """An ExpertStore holding the file's routed experts (all of them, or expert_range's of every layer)."""
    from . import moe
    meta, tensors = read_gguf(path)
    lay = expert_layout(meta, tensors)
    store = moe.ExpertStore(lay.layers, lay.experts, lay.hidden, lay.ffn, cap_bytes=cap_bytes, ctx=ctx,
                            expert_range=expert_range)
    lo, hi = expert_range or (0, lay.experts)
    files = _Files()
    try:
        for layer in range(lay.layers):
            store.set_down_type(layer, lay.down_type(layer))
            for e in range(lo, hi):
                store.upload(layer, e, expert_blob(files, lay, layer, e))
    finally:
        files.close()
    return store


def _float_tensor(files: _Files, t: Tensor) -> np.ndarray:
    n = int(np.prod(t.shape))
    raw = files.view(t, 0, t.nbytes)
    if t.type == "F32":
        return raw.view(np.float32).reshape(t.shape).copy()
    if t.type == "F16":
        return raw.view(np.float16).astype(np.float32).reshape(t.shape)
    if t.type == "BF16":
        return (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32).reshape(t.shape)
    raise GGUFError(f"{t.name}: {t.type}; expected F32, F16 or BF16")


def layer_weights(path: str, ctx=None, prepare: bool = True, tensors_of=None):
    """moe.LayerWeights for every layer: router blk.N.ffn_gate_inp.weight [E, H] and shared-expert gate
    ffn_gate_inp_shexp.weight [H] as float32, the shared expert's ffn_{gate,up}_shexp (Q4_K [F, H]) fused into
    gate_up bytes and ffn_down_shexp ([H, F], of the layer's down type) (the names of
    engines/qwen36/loader.py:37-41)."""
    import torch
    from . import moe
    meta, tensors = tensors_of or read_gguf(path)
    lay = expert_layout(meta, tensors)
    files = _Files()
    out = []
    try:
        for layer in range(lay.layers):
            p = f"blk.{layer}."
            need = ["ffn_gate_inp.weight", "ffn_gate_inp_shexp.weight", "ffn_gate_shexp.weight",
                    "ffn_up_shexp.weight", "ffn_down_shexp.weight"]
            missing = [n for n in need if p + n not in tensors]
            if missing:
                raise GGUFError(f"layer {layer}: missing {', '.join(p + n for n in missing)}")
            router = _float_tensor(files, tensors[p + "ffn_gate_inp.weight"])
            gate_vec = _float_tensor(files, tensors[p + "ffn_gate_inp_shexp.weight"]).reshape(-1)
            if router.shape != (lay.experts, lay.hidden) or gate_vec.shape != (lay.hidden,):
                raise GGUFError(f"layer {layer}: router {router.shape} / shared gate {gate_vec.shape}, expected "
                                f"{(lay.experts, lay.hidden)} / {(lay.hidden,)}")
            sg, su, sd = (tensors[p + n] for n in need[2:])
            # the kernels read the shared expert's down matrix with the layer's down type
            for t, typ, shape in ((sg, "Q4_K", (lay.ffn, lay.hidden)), (su, "Q4_K", (lay.ffn, lay.hidden)),
                                  (sd, lay.down_type(layer), (lay.hidden, lay.ffn))):
                if t.type != typ or tuple(t.shape) != shape:
                    raise GGUFError(f"{t.name}: {t.type} {t.shape}; the kernels run {typ} {shape}")
            gate_up = np.concatenate([files.view(sg, 0, sg.nbytes), files.view(su, 0, su.nbytes)])
            down = files.view(sd, 0, sd.nbytes).copy()
            lw = moe.LayerWeights(router_w=torch.from_numpy(router).cuda(),
                                  shared_gate=torch.from_numpy(np.ascontiguousarray(gate_vec)).cuda(),
                                  shared_gate_up=torch.from_numpy(gate_up).cuda(),
                                  shared_down=torch.from_numpy(down).cuda())
            out.append(lw.prepare(ctx) if prepare else lw)
    finally:
        files.close()
    return out


# the ggml types of the typed expert kernels (willow_v2_b200/ggml.py, gguf/metal.py:295)
TYPED = ("Q5_0", "Q8_0", "IQ4_NL", "IQ4_XS", "IQ3_XXS", "IQ3_S", "IQ2_S", "Q2_0", "Q4_K", "Q6_K")


@dataclass
class TypedLayer:
    """One layer's routed experts, of any type the typed kernels run, in one uint8 buffer in the pack layout (per
    expert: gate rows, up rows, down rows; gguf/compiler.py:69-88), and each expert's (gate_up, down) as
    ggml.GGMLWeight views of that buffer. One buffer with byte offsets is what the batched decode kernels take
    (gemv_batch, gemv_combine; engines/base.py:492-532), as willow's store hands out GGMLWeight views of its GPU
    slots (gguf/store.py:425-437)."""
    base: object                 # torch uint8 tensor [experts * expert_bytes]
    experts: list                # [(gate_up GGMLWeight [2F, H], down GGMLWeight [H, F])] per expert
    gate_up_type: str
    down_type: str
    hidden: int
    ffn: int
    expert_bytes: int


def typed_layer(path: str, layer: int, device="cuda", parsed=None) -> TypedLayer:
    """Reads one layer's ffn_{gate,up,down}_exps (or ffn_gate_up_exps) whatever their type among TYPED into one
    buffer on `device`. Raises GGUFError naming a tensor of another type or shape."""
    import torch
    from .ggml import GGMLWeight
    meta, tensors = parsed or read_gguf(path)
    parts = {}
    for name, t in tensors.items():
        m = _EXPERT.match(name)
        if m and int(m.group(1)) == layer:
            parts[m.group(2)] = t
    if "gate_up" in parts:
        gu = (parts["gate_up"],)
    elif "gate" in parts and "up" in parts:
        gu = (parts["gate"], parts["up"])
    else:
        raise GGUFError(f"layer {layer}: expected ffn_gate_exps and ffn_up_exps (or ffn_gate_up_exps)")
    if "down" not in parts:
        raise GGUFError(f"layer {layer}: no ffn_down_exps")
    down = parts["down"]
    for t in (*gu, down):
        if t.type not in TYPED or len(t.shape) != 3:
            raise GGUFError(f"{t.name}: {t.type} {t.shape}; the typed kernels run {', '.join(TYPED)} "
                            "[experts, rows, k]")
    if len(gu) == 2 and (gu[0].type != gu[1].type or gu[0].shape != gu[1].shape):
        raise GGUFError(f"layer {layer}: gate {gu[0].type} {gu[0].shape} and up {gu[1].type} {gu[1].shape} differ")
    E, rows, H = gu[0].shape
    F = rows // 2 if len(gu) == 1 else rows
    if down.shape != (E, H, F):
        raise GGUFError(f"{down.name}: shape {down.shape}, expected {(E, H, F)}")
    if H % 32 or F % 32:
        raise GGUFError(f"layer {layer}: hidden {H} and ffn {F} must be multiples of 32")
    gu_b = sum(t.nbytes for t in gu) // E
    dn_b = down.nbytes // E
    eb = gu_b + dn_b
    host = np.empty(E * eb, dtype=np.uint8)
    files = _Files()
    try:
        for e in range(E):
            at = e * eb
            for t in gu:
                per = t.nbytes // E
                host[at:at + per] = files.view(t, e * per, per)
                at += per
            host[at:at + dn_b] = files.view(down, e * dn_b, dn_b)
    finally:
        files.close()
    base = torch.from_numpy(host).to(device)
    experts = [(GGMLWeight(base[e * eb:e * eb + gu_b], gu[0].type, (2 * F, H)),
                GGMLWeight(base[e * eb + gu_b:(e + 1) * eb], down.type, (H, F))) for e in range(E)]
    return TypedLayer(base, experts, gu[0].type, down.type, H, F, eb)


def load(path: str, ctx=None, cap_bytes: int = 0, expert_range: Optional[Tuple[int, int]] = None):
    """(ExpertStore, [LayerWeights per layer]) for a qwen35moe GGUF."""
    parsed = read_gguf(path)
    store = load_experts(path, ctx=ctx, cap_bytes=cap_bytes, expert_range=expert_range)
    return store, layer_weights(path, ctx=ctx or store.ctx, tensors_of=parsed)
