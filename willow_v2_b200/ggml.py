"""Typed expert kernels over ggml blocks: the B200 counterpart of willow's gguf/metal.py, for every type its Metal
path runs (gguf/metal.py:295: Q5_0, Q8_0, IQ4_NL, IQ4_XS, IQ3_XXS, IQ3_S, IQ2_S, Q2_0, Q4_K, Q6_K).

  row_bytes(type_name, k)                                   gguf/metal.py:323-325
  gemv(raw, type_name, shape, x)                            gguf/metal.py:327-334 (tokens <= MAX_TOKENS)
  gemv_batch(base, type_name, shape, x, offsets, positions, out)    gguf/metal.py:336-343
  gemv_combine(base, type_name, shape, x, offsets, weights, perm)   gguf/metal.py:345-355
  dequantize_gpu(raw, type_name, shape)                     gguf/metal.py:357-363
  GGMLWeight                                                gguf/metal.py:365-408 (F.linear on ggml blocks)

Arguments mean what they mean there. bf16 in and out, summed in float32; gemv_combine rounds to bf16 at every
step like engines/base.py:431-443. The kernels are CUDA (libwmoe.so, csrc/ggml_gemv.cu); a missing library raises
on import, and a type outside TYPES raises NotImplementedError as willow's quants.dequantize does.
"""
import ctypes
from typing import Optional

import torch
import torch.nn.functional as F

from . import lib as _lib
from .lib import check, lib

MAX_TOKENS = 8  # gemv handles up to this many tokens; more are dequantized to bf16 and multiplied by torch
TYPES = ("Q5_0", "Q8_0", "IQ4_NL", "IQ4_XS", "IQ3_XXS", "IQ3_S", "IQ2_S", "Q2_0", "Q4_K", "Q6_K")
# (elements, bytes) per block (gguf/reader.py:14-48)
BLOCKS = {"Q5_0": (32, 22), "Q8_0": (32, 34), "IQ4_NL": (32, 18), "IQ4_XS": (256, 136), "IQ3_XXS": (256, 98),
          "IQ3_S": (256, 110), "IQ2_S": (256, 82), "Q2_0": (64, 18), "Q4_K": (256, 144), "Q6_K": (256, 210)}
_DTYPES = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16, torch.float16: _lib.F16}


def _type_id(type_name: str) -> int:
    if type_name not in _lib.GGML_TYPES:
        raise NotImplementedError(f"ggml type {type_name} has no CUDA kernel (supported: {', '.join(TYPES)})")
    return _lib.GGML_TYPES[type_name]


def _ctx():
    from .moe import default_context
    return default_context()


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _p(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _act(x: torch.Tensor) -> torch.Tensor:
    """Activations as the kernels take them: bf16 or f32, contiguous (16-byte aligned rows). Other float types widen
    to f32, which holds every f16 value exactly."""
    if x.dtype not in (torch.bfloat16, torch.float32):
        x = x.to(torch.float32)
    return x.contiguous()


def _on_gpu(*tensors):
    """The kernels read these through device addresses: every one must be a CUDA tensor on one device."""
    devs = {t.device for t in tensors}
    if any(not t.is_cuda for t in tensors) or len(devs) != 1:
        raise ValueError(f"expected CUDA tensors on one device, got {sorted(str(d) for d in devs)}")


class _Staging:
    """The small int64 arrays the batched kernels take (matrix addresses, output positions, routing order) go to the
    GPU through a ring of pinned host chunks, each copied asynchronously into its device chunk on the current
    stream: a call makes no host synchronisation (a pageable torch.tensor(...).to(device) would wait for the GPU
    on every call). A chunk is written again only after the event recorded behind the kernel that read its last
    contents has completed; with 64 chunks that wait is all but never taken."""
    CHUNKS, WORDS = 64, 1024

    def __init__(self, device: torch.device):
        self.host = torch.empty(self.CHUNKS, self.WORDS, dtype=torch.int64).pin_memory()
        self.host_np = self.host.numpy()
        self.dev = torch.empty(self.CHUNKS, self.WORDS, dtype=torch.int64, device=device)
        self.events = [None] * self.CHUNKS
        self.next = 0
        self.chunk = -1

    def put(self, *arrays):
        """Device int64 views of the given integer sequences (one chunk for all of them)."""
        sizes = [len(a) for a in arrays]
        if sum(sizes) > self.WORDS:  # beyond a chunk: a plain (synchronising) upload
            self.chunk = -1
            return [torch.tensor(list(a), dtype=torch.int64).to(self.dev.device) for a in arrays]
        c = self.chunk = self.next
        self.next = (c + 1) % self.CHUNKS
        if self.events[c] is not None:
            self.events[c].synchronize()
        h, off, views = self.host_np[c], 0, []
        for a, n in zip(arrays, sizes):
            h[off:off + n] = a
            views.append((off, n))
            off += n
        self.dev[c, :off].copy_(self.host[c, :off], non_blocking=True)
        return [self.dev[c, o:o + n] for o, n in views]

    def done(self):
        """Marks the chunk of the last put as read by the kernel just launched on the current stream."""
        if self.chunk >= 0:
            ev = torch.cuda.Event()
            ev.record()
            self.events[self.chunk] = ev


_STAGING = {}


def _staging(device: torch.device) -> _Staging:
    key = device.index if device.index is not None else torch.cuda.current_device()
    if key not in _STAGING:
        _STAGING[key] = _Staging(torch.device("cuda", key))
    return _STAGING[key]


def available() -> bool:
    return torch.cuda.is_available()


def row_bytes(type_name: str, k: int) -> int:
    elements, size = BLOCKS[type_name]
    return k // elements * size


def dequantize_gpu(raw: torch.Tensor, type_name: str, shape: tuple, dtype: torch.dtype = torch.bfloat16,
                   ctx=None) -> torch.Tensor:
    """raw (uint8, on the GPU) -> dtype [shape] on the GPU; float32 bit-identical to gguf/quants.py:dequantize."""
    gtype = _type_id(type_name)
    elements, size = BLOCKS[type_name]
    _on_gpu(raw)
    assert raw.dtype == torch.uint8 and raw.is_contiguous()
    nblocks = raw.numel() // size
    numel = 1
    for s in shape:
        numel *= int(s)
    if nblocks * size != raw.numel() or nblocks * elements != numel:
        raise ValueError(f"{raw.numel()} bytes of {type_name} do not hold a tensor of shape {tuple(shape)}")
    out = torch.empty(tuple(shape), dtype=dtype, device=raw.device)
    ctx = ctx or _ctx()
    check(ctx.handle, lib.wmoe_dequant(ctx.handle, gtype, _p(raw), nblocks, _p(out), _DTYPES[dtype], _stream()))
    return out


def gemv(raw: torch.Tensor, type_name: str, shape: tuple, x: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16,
         ctx=None) -> torch.Tensor:
    """raw: the weight's bytes (uint8, on the GPU); x: [tokens <= MAX_TOKENS, k] -> out_dtype [tokens, rows]."""
    rows, k = shape
    x = _act(x.reshape(-1, k))
    if not 1 <= x.shape[0] <= MAX_TOKENS:
        raise ValueError(f"gemv takes 1..{MAX_TOKENS} tokens, got {x.shape[0]}")
    if raw.numel() < rows * row_bytes(type_name, k):
        raise ValueError("raw holds fewer bytes than the [rows, k] matrix")
    _on_gpu(raw, x)
    y = torch.empty(x.shape[0], rows, dtype=out_dtype, device=raw.device)
    ctx = ctx or _ctx()
    check(ctx.handle, lib.wmoe_gemv(ctx.handle, _type_id(type_name), _p(raw), rows, k, _p(x), _DTYPES[x.dtype],
                                    x.shape[0], _p(y), _DTYPES[out_dtype], _stream()))
    return y


def gemv_batch(base: torch.Tensor, type_name: str, shape: tuple, x: torch.Tensor, offsets: list, positions: list,
               out: torch.Tensor, ctx=None):
    """Several experts' weights, all [rows, k] of type_name at byte offsets in base (uint8, on the GPU), times one
    token x ([1, k] or [k]): writes expert i's result to row positions[i] of out ([n, rows], bf16 or f32)."""
    rows, k = shape
    if len(offsets) != len(positions):
        raise ValueError("one position per offset")
    if not offsets:
        return
    rb = row_bytes(type_name, k)
    for o in offsets:
        if o < 0 or o + rows * rb > base.numel():
            raise ValueError(f"offset {o} puts a [{rows}, {k}] {type_name} matrix outside base")
    if any(not 0 <= p < out.shape[0] for p in positions):
        raise ValueError("a position outside out")
    assert out.is_contiguous() and out.shape[-1] == rows
    x = _act(x.reshape(k))
    _on_gpu(base, x, out)
    stage = _staging(base.device)
    b0 = base.data_ptr()
    ptrs, pos = stage.put([b0 + int(o) for o in offsets], [int(q) for q in positions])
    ctx = ctx or _ctx()
    try:
        check(ctx.handle, lib.wmoe_gemv_batch(ctx.handle, _type_id(type_name), _p(ptrs), _p(pos), len(offsets),
                                              out.shape[0], rows, k, _p(x), _DTYPES[x.dtype], _p(out),
                                              _DTYPES[out.dtype], _stream()))
    finally:
        stage.done()


def gemv_combine(base: torch.Tensor, type_name: str, shape: tuple, x: torch.Tensor, offsets: list,
                 weights: torch.Tensor, perm: list, ctx=None) -> torch.Tensor:
    """sum over i of weights[perm[i]] * (W_i x[i]), in order of i, rounded to bf16 at each step like torch's bf16
    ops. W_i: [rows, k] of type_name at byte offsets[i] in base; x: bf16 [n, k]; weights: bf16 [top_k], on the GPU.
    -> bf16 [1, rows]."""
    rows, k = shape
    n = len(offsets)
    if n == 0 or len(perm) != n:
        raise ValueError("one perm entry per offset, at least one")
    rb = row_bytes(type_name, k)
    for o in offsets:
        if o < 0 or o + rows * rb > base.numel():
            raise ValueError(f"offset {o} puts a [{rows}, {k}] {type_name} matrix outside base")
    if any(not 0 <= p < weights.numel() for p in perm):
        raise ValueError("a perm entry outside weights")
    x = x.reshape(n, k).to(torch.bfloat16).contiguous()
    w = weights.reshape(-1).to(torch.bfloat16).contiguous()
    _on_gpu(base, x, w)
    stage = _staging(base.device)
    b0 = base.data_ptr()
    ptrs, pm = stage.put([b0 + int(o) for o in offsets], [int(q) for q in perm])
    y = torch.empty(1, rows, dtype=torch.bfloat16, device=base.device)
    ctx = ctx or _ctx()
    try:
        check(ctx.handle, lib.wmoe_gemv_combine(ctx.handle, _type_id(type_name), _p(ptrs), _p(pm), n, w.numel(),
                                                rows, k, _p(x), _p(w), _lib.BF16, _p(y), _stream()))
    finally:
        stage.done()
    return y


def expert_gate(gate_up: torch.Tensor, ctx=None) -> torch.Tensor:
    """willow's expert_gate (engines/base.py:99-102) on bf16 [n, 2 * ffn] rows -> bf16 [n, ffn] (wmoe_expert_gate),
    rounded as torch's bf16 F.silu(gate) * up."""
    if gate_up.dtype != torch.bfloat16 or gate_up.dim() != 2 or gate_up.shape[1] % 2:
        raise ValueError("expert_gate takes bf16 [n, 2 * ffn]")
    gate_up = gate_up.contiguous()
    _on_gpu(gate_up)
    n, ffn = gate_up.shape[0], gate_up.shape[1] // 2
    out = torch.empty(n, ffn, dtype=torch.bfloat16, device=gate_up.device)
    ctx = ctx or _ctx()
    check(ctx.handle, lib.wmoe_expert_gate(ctx.handle, _p(gate_up), n, ffn, _p(out), _stream()))
    return out


def batched_decode_experts(base: torch.Tensor, gate_up_type: str, down_type: str, ffn: int, x: torch.Tensor,
                           gate_up_offsets, down_offsets, routing_weights: torch.Tensor, perm,
                           ctx=None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One decode token's routed experts in one library call (wmoe_batched_decode_experts), as
    engines/base.py:492-532 batched_decode_experts runs them when the experts sit in one buffer: gate_up_offsets[i]
    is expert i's [2 * ffn, hidden] gate_up matrix of gate_up_type and down_offsets[i] its [hidden, ffn] down matrix
    of down_type, byte offsets in base (uint8, on the GPU); x bf16 [hidden]; routing_weights bf16 [top_k], perm[i]
    the slot of expert i's weight in it. Returns bf16 [1, hidden] (written into out when given), the value of
    gemv_batch, expert_gate and gemv_combine run one after another."""
    n = len(gate_up_offsets)
    if n == 0 or len(down_offsets) != n or len(perm) != n:
        raise ValueError("one down offset and one perm entry per gate_up offset, at least one")
    if x.dtype != torch.bfloat16 or not x.is_contiguous():
        x = x.to(torch.bfloat16).contiguous()
    hidden = x.numel()
    w = routing_weights
    if w.dtype != torch.bfloat16 or not w.is_contiguous():
        w = w.to(torch.bfloat16).contiguous()
    gu_bytes = 2 * ffn * row_bytes(gate_up_type, hidden)
    dn_bytes = hidden * row_bytes(down_type, ffn)
    size = base.numel()
    if min(gate_up_offsets) < 0 or max(gate_up_offsets) + gu_bytes > size:
        raise ValueError("a gate_up offset puts its matrix outside base")
    if min(down_offsets) < 0 or max(down_offsets) + dn_bytes > size:
        raise ValueError("a down offset puts its matrix outside base")
    if min(perm) < 0 or max(perm) >= w.numel():
        raise ValueError("a perm entry outside routing_weights")
    dev = base.device
    if not (base.is_cuda and x.device == dev and w.device == dev):
        raise ValueError("base, x and routing_weights must be CUDA tensors on one device")
    if out is None:
        out = torch.empty(1, hidden, dtype=torch.bfloat16, device=dev)
    elif out.dtype != torch.bfloat16 or out.numel() != hidden or not out.is_contiguous() or out.device != dev:
        raise ValueError("out must be a contiguous bf16 tensor of hidden values on base's device")
    b0 = base.data_ptr()
    gu = (ctypes.c_uint64 * n)(*[b0 + o for o in gate_up_offsets])
    dn = (ctypes.c_uint64 * n)(*[b0 + o for o in down_offsets])
    pm = (ctypes.c_int64 * n)(*perm)
    ctx = ctx or _ctx()
    check(ctx.handle, lib.wmoe_batched_decode_experts(ctx.handle, _type_id(gate_up_type), _type_id(down_type), hidden,
                                                      ffn, gu, dn, pm, n, w.numel(), x.data_ptr(), w.data_ptr(),
                                                      out.data_ptr(), torch.cuda.current_stream(dev).cuda_stream))
    return out


class GGMLWeight:
    """A [rows, k] weight kept as its ggml blocks on the GPU, used in place of a bf16 tensor: F.linear(x, weight)
    runs the CUDA kernels above (through __torch_function__). raw is a uint8 tensor; a CPU tensor is copied to the
    GPU on first use."""

    @classmethod
    def __torch_function__(cls, func, types, args=(), kwargs=None):
        bias = (kwargs or {}).get("bias", args[2] if len(args) > 2 else None)
        if func is F.linear and len(args) > 1 and isinstance(args[1], GGMLWeight) and bias is None:
            return args[1].linear(args[0])
        return NotImplemented

    def __init__(self, raw: torch.Tensor, type_name: str, shape: tuple):
        _type_id(type_name)
        self.raw, self.type_name, self.shape = raw, type_name, tuple(shape)
        self.nbytes = raw.numel()

    def to_gpu(self, device=None):
        if not self.raw.is_cuda:
            self.raw = self.raw.to(device or torch.device("cuda", torch.cuda.current_device()), non_blocking=True)

    def location(self):
        """(the GPU buffer holding this weight's bytes, as a uint8 tensor; their byte offset in it), for the
        batched kernels."""
        self.to_gpu()
        base = self.raw if self.raw._base is None else self.raw._base
        return base, self.raw.storage_offset() - base.storage_offset()

    def linear(self, x: torch.Tensor) -> torch.Tensor:
        self.to_gpu()
        flat = x.reshape(-1, x.shape[-1])
        if not flat.is_cuda:
            flat = flat.to(self.raw.device)
        if flat.shape[0] <= MAX_TOKENS:
            y = gemv(self.raw, self.type_name, self.shape, flat).to(x.dtype)
        else:
            y = F.linear(flat.to(torch.bfloat16), dequantize_gpu(self.raw, self.type_name, self.shape)).to(x.dtype)
        return y.view(*x.shape[:-1], y.shape[-1]).to(x.device)
