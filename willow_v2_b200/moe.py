"""The host side of the B200 MoE block: thin PyTorch-facing wrappers over libwmoe.so that mirror willow's own
interfaces, so willow's engine can call them unchanged.

  dequantize(raw, type_name, shape, dtype)   gguf/quants.py:207-227 (every type of ggml.TYPES), on the GPU
  route(x, router_w, top_k, ...)             engines/base.py:91-97 route, after the router linear (base.py:448)
  dispatch(selected, experts)                engines/base.py:456-467 grouping + store.py:482-484 record_usage
  ExpertStore                                gguf/store.py:41-536 (HBM slots; capped LRU over pinned host memory)
  moe_forward / CudaMoE.moe                  engines/base.py:445-490 Engine.moe
  decode_stack                               engines/qwen36/model.py:17-22, the per-layer x + moe(rms_norm(x))

Tensors are torch CUDA tensors; kernels run on torch's current stream. Errors raise WmoeError with the library's
message (willow raises Python exceptions the same way: quants.py:214-216, store.py:77-81).
"""
import ctypes
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from . import lib as _lib
from .lib import check, lib

_DTYPES = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16, torch.float16: _lib.F16}
_GGML = {"Q4_K": (_lib.GGML_Q4_K, 144), "Q6_K": (_lib.GGML_Q6_K, 210)}


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


class Context:
    """One libwmoe context on a CUDA device (scratch buffers, device status word, launch counter)."""

    def __init__(self, device: Optional[int] = None):
        self.device = torch.cuda.current_device() if device is None else int(device)
        handle = ctypes.c_void_p()
        code = lib.wmoe_init(self.device, ctypes.byref(handle))
        if code != _lib.OK:
            raise _lib.WmoeError(code, f"wmoe_init failed on device {self.device}")
        self.handle = handle

    @property
    def launches(self) -> int:
        return int(lib.wmoe_launch_count(self.handle))

    def set_decode_kernel(self, enable: bool) -> bool:
        return bool(lib.wmoe_set_decode_kernel(self.handle, int(enable)))

    def set_min_expert_weight(self, weight: float):
        """willow's min_expert_weight (engines/base.py:413-429): routings of this context drop each token's picks of
        renormalised weight below `weight` except its top one, scaling the kept ones back to the former total;
        dropped picks are returned as -1 (weight 0). 0 turns it off."""
        check(self.handle, lib.wmoe_set_min_expert_weight(self.handle, float(weight)))

    def device_status(self) -> int:
        """Reads and clears the device status word (0 = fine; see lib.STATUS_NAMES)."""
        v = ctypes.c_int()
        check(self.handle, lib.wmoe_device_status(self.handle, ctypes.byref(v), _stream()))
        return v.value

    def check_device(self):
        v = self.device_status()
        if v:
            raise _lib.WmoeError(_lib.ERR_DEVICE, _lib.STATUS_NAMES.get(v, f"device status {v}"))

    def ep_set_timeout(self, ms: int) -> int:
        """Bound of every host wait on the expert-parallel communicator (wmoe_ep_set_timeout); returns the old one."""
        return int(lib.wmoe_ep_set_timeout(self.handle, int(ms)))

    def ep_finalize(self):
        """Frees the NCCL communicator of ep_init (every rank, before the process group goes away)."""
        check(self.handle, lib.wmoe_ep_finalize(self.handle))

    def close(self):
        if self.handle:
            lib.wmoe_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_default_ctx = {}


def default_context() -> Context:
    dev = torch.cuda.current_device()
    if dev not in _default_ctx:
        _default_ctx[dev] = Context(dev)
    return _default_ctx[dev]


def dequantize(raw: torch.Tensor, type_name: str, shape: tuple, dtype: torch.dtype = torch.bfloat16,
               ctx: Optional[Context] = None) -> torch.Tensor:
    """raw: uint8 CUDA tensor holding one ggml tensor's bytes (any type of ggml.TYPES) -> a new tensor of shape and
    dtype (float32 bit-identical to gguf/quants.py:dequantize; bf16/f16 rounded to nearest even from it)."""
    from .ggml import dequantize_gpu
    return dequantize_gpu(raw, type_name, shape, dtype, ctx)


def route(x: torch.Tensor, router_w: torch.Tensor, top_k: int = 8, bias: Optional[torch.Tensor] = None,
          shared_gate: Optional[torch.Tensor] = None, ctx: Optional[Context] = None):
    """x [T, H] (f32/bf16) -> (weights f32 [T, top_k], selected int32 [T, top_k], shared gate sigmoid f32 [T] or
    None, logits f32 [T, E]). The router linear in fp32, softmax, top-k and renormalisation of engines/base.py:91-97
    (norm_topk_prob=True)."""
    ctx = ctx or default_context()
    T, H = x.shape
    E = router_w.shape[0]
    w = torch.empty(T, top_k, dtype=torch.float32, device=x.device)
    sel = torch.empty(T, top_k, dtype=torch.int32, device=x.device)
    s = torch.empty(T, dtype=torch.float32, device=x.device) if shared_gate is not None else None
    logits = torch.empty(T, E, dtype=torch.float32, device=x.device)
    check(ctx.handle, lib.wmoe_route(ctx.handle, _ptr(x.contiguous()), _DTYPES[x.dtype], T, H, E, top_k,
                                     _ptr(router_w), _ptr(bias), _ptr(shared_gate), _ptr(w), _ptr(sel), _ptr(s),
                                     _ptr(logits), _stream()))
    return w, sel, s, logits


def dispatch(selected: torch.Tensor, experts: int, usage: Optional[torch.Tensor] = None,
             ctx: Optional[Context] = None):
    """selected int32 [T, k] -> (counts int32 [E], offsets int32 [E+1], perm int32 [T*k]): the picks grouped by
    expert, tokens ascending within an expert; perm holds token*k + slot. usage (int64 [E]) accumulates counts."""
    ctx = ctx or default_context()
    T, k = selected.shape
    dev = selected.device
    counts = torch.empty(experts, dtype=torch.int32, device=dev)
    offsets = torch.empty(experts + 1, dtype=torch.int32, device=dev)
    perm = torch.empty(T * k, dtype=torch.int32, device=dev)
    check(ctx.handle, lib.wmoe_dispatch(ctx.handle, _ptr(selected.contiguous()), T, k, experts, _ptr(counts),
                                        _ptr(offsets), _ptr(perm), _ptr(usage), _stream()))
    return counts, offsets, perm


class ExpertStore:
    """Routed experts of every layer in HBM (the role of gguf/store.py:ExpertStore). Each expert is one blob, the
    pack layout: gate_up (Q4_K [2F, H], gate rows then up rows) followed by down (Q6_K [H, F]).
    cap_bytes = 0 keeps every blob resident; otherwise at most cap_bytes of device slots, the blobs in pinned
    host memory, misses copied on a side stream with least-recently-used eviction."""

    def __init__(self, layers: int, experts: int = 256, hidden: int = 2048, ffn: int = 512, cap_bytes: int = 0,
                 ctx: Optional[Context] = None, expert_range: Optional[tuple] = None):
        """expert_range (begin, end): hold only those experts of every layer (one rank's block under expert
        parallelism, wmoe_store_create_range); default all."""
        self.ctx = ctx or default_context()
        self.layers, self.experts, self.hidden, self.ffn = layers, experts, hidden, ffn
        self.expert_range = tuple(expert_range) if expert_range is not None else (0, experts)
        held = self.expert_range[1] - self.expert_range[0]
        handle = ctypes.c_void_p()
        check(self.ctx.handle, lib.wmoe_store_create_range(self.ctx.handle, layers, experts, self.expert_range[0],
                                                           self.expert_range[1], hidden, ffn, cap_bytes,
                                                           ctypes.byref(handle)))
        self.handle = handle
        self.blob_bytes = int(lib.wmoe_store_blob_bytes(handle))
        self.gate_up_bytes = 2 * ffn * hidden // 256 * 144
        self.capped = cap_bytes != 0 and cap_bytes < layers * held * ((self.blob_bytes + 255) // 256 * 256)

    def set_down_type(self, layer: int, type_name: str):
        """The layer's down-matrix type: "Q6_K" (default) or "Q4_K" (some layers of llama.cpp's Q4_K_M files).
        Set before uploading the layer; its blob is then layer_blob_bytes(layer) long."""
        check(self.ctx.handle, lib.wmoe_store_set_down_type(self.handle, layer, _GGML[type_name][0]))

    def layer_blob_bytes(self, layer: int) -> int:
        return int(lib.wmoe_store_layer_blob_bytes(self.handle, layer))

    def upload(self, layer: int, expert: int, blob):
        """blob: the expert's bytes (numpy uint8 / bytes, or a CPU uint8 tensor), layer_blob_bytes(layer) long."""
        arr = np.ascontiguousarray(np.frombuffer(blob, dtype=np.uint8) if isinstance(blob, (bytes, bytearray))
                                   else (blob.numpy() if isinstance(blob, torch.Tensor) else blob), dtype=np.uint8)
        want = self.layer_blob_bytes(layer)
        if arr.size != want:
            raise ValueError(f"expert blob is {arr.size} bytes, expected {want}")
        check(self.ctx.handle, lib.wmoe_store_upload(self.handle, layer, expert,
                                                     arr.ctypes.data_as(ctypes.c_void_p), _stream()))
        torch.cuda.current_stream().synchronize()  # the host buffer may be freed after this returns

    def fill_synthetic(self, seed: int, layer_begin: int = 0, layer_end: Optional[int] = None):
        """Generates every blob of the layer range on the device (the generator of willow_v2_b200.synth)."""
        end = self.layers if layer_end is None else layer_end
        check(self.ctx.handle, lib.wmoe_store_fill_synthetic(self.handle, seed, layer_begin, end, _stream()))

    def load_many(self, layer: int, experts):
        """Makes the experts of a layer resident (store.py:132-137's role); a no-op when nothing is capped."""
        ids = np.ascontiguousarray(np.asarray(list(experts), dtype=np.int32))
        check(self.ctx.handle, lib.wmoe_store_prepare(self.handle, layer, ids.ctypes.data_as(ctypes.c_void_p),
                                                      int(ids.size), _stream()))

    def prefetch(self, layer: int, experts=None):
        """Starts copying experts of a coming layer (store.py:204-219) without making the compute stream wait;
        experts None: the experts the layer has been routed to before, most used first (all of the layer's experts
        this store holds when there is no history). A no-op when nothing is capped."""
        if experts is None:
            check(self.ctx.handle, lib.wmoe_store_prefetch(self.handle, layer, None, 0, _stream()))
            return
        ids = np.ascontiguousarray(np.asarray(list(experts), dtype=np.int32))
        check(self.ctx.handle, lib.wmoe_store_prefetch(self.handle, layer, ids.ctypes.data_as(ctypes.c_void_p),
                                                       int(ids.size), _stream()))

    def choose_hot(self, share: float = 0.75):
        """Keeps `share` of the slots for the experts routed the most tokens so far (store.py:464-480, HOT_SHARE)."""
        check(self.ctx.handle, lib.wmoe_store_choose_hot(self.handle, float(share)))

    def download(self, layer: int, expert: int) -> np.ndarray:
        """The expert's bytes as the store holds them (uint8 [layer_blob_bytes(layer)])."""
        out = np.empty(self.layer_blob_bytes(layer), dtype=np.uint8)
        check(self.ctx.handle, lib.wmoe_store_download(self.handle, layer, expert,
                                                       out.ctypes.data_as(ctypes.c_void_p), _stream()))
        return out

    def blob_ptr(self, layer: int, expert: int) -> Optional[int]:
        return lib.wmoe_store_blob(self.handle, layer, expert)

    def stats(self) -> dict:
        vals = [ctypes.c_uint64() for _ in range(6)]
        check(self.ctx.handle, lib.wmoe_store_stats(self.handle, *[ctypes.byref(v) for v in vals[:4]]))
        check(self.ctx.handle, lib.wmoe_store_prefetch_stats(self.handle, *[ctypes.byref(v) for v in vals[4:]]))
        return dict(zip(("hits", "misses", "bytes_in", "evictions", "prefetched", "prefetch_used"),
                        (v.value for v in vals)))

    def close(self):
        if self.handle:
            lib.wmoe_store_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def add_rmsnorm(x: torch.Tensor, y: Optional[torch.Tensor] = None, eps: float = 1e-6,
                out_dtype: torch.dtype = torch.bfloat16, ctx: Optional[Context] = None):
    """The layer glue of engines/qwen36/model.py:17-22 (rms_norm of engines/base.py:27-32, weight 1): returns
    (x + y as float32, rms_norm(x + y) as out_dtype); y (the previous MoE output, f32 or bf16) may be None. x is
    updated in place (float32 [T, H])."""
    ctx = ctx or default_context()
    if x.dtype != torch.float32 or not x.is_contiguous():
        raise ValueError("add_rmsnorm: x must be a contiguous float32 tensor")
    T, H = x.shape
    xn = torch.empty(T, H, dtype=out_dtype, device=x.device)
    y_c = None if y is None else y.contiguous()
    check(ctx.handle, lib.wmoe_add_rmsnorm(ctx.handle, _ptr(x), _ptr(y_c), _DTYPES[y.dtype] if y is not None else 0,
                                           T, H, float(eps), _ptr(x), _ptr(xn), _DTYPES[out_dtype], _stream()))
    return x, xn


def guess_next_layer(store: ExpertStore, residual: torch.Tensor, lw_next: "LayerWeights", layer_next: int,
                     top_k: int = 8, eps: float = 1e-6, guess_input: Optional[torch.Tensor] = None) -> list:
    """Decode on a capped store (engines/base.py:392-406, with engines/qwen36/model.py:30-31's guess input): runs
    the next layer's router on rms_norm(residual), the residual stream before the current layer's experts (or on
    guess_input, the engine's own normalised form of it), and starts copying the experts it picks for every token
    (ExpertStore.prefetch), so they are resident or on their way when that layer runs; the current layer's experts
    compute meanwhile. Returns the guessed expert ids (those this store holds). Usually most of them are the experts
    the layer then picks. Guesses the context's min_expert_weight drops are not copied (base.py:424-425)."""
    if guess_input is None:
        x = residual.float().contiguous().clone()
        _, xn = add_rmsnorm(x, None, eps, out_dtype=torch.float32, ctx=store.ctx)
    else:
        xn = guess_input.float().contiguous()
    w, sel, _, _ = route(xn, lw_next.router_w, top_k, bias=lw_next.router_bias, ctx=store.ctx)
    lo, hi = store.expert_range
    picked = sel[w > 0]
    guess = [e for e in torch.unique(picked).tolist() if lo <= e < hi]
    store.prefetch(layer_next, guess)
    return guess


def pack_router(router_w: torch.Tensor, shared_gate: torch.Tensor, ctx: Optional[Context] = None) -> torch.Tensor:
    """The router [E, H] and shared gate [H] transposed into one f32 [H, 264] matrix (wmoe_pack_router): the
    decode kernel reads each CTA's rows of it as one contiguous block."""
    ctx = ctx or default_context()
    E, H = router_w.shape
    out = torch.empty(H, _lib.ROUTER_STRIDE, dtype=torch.float32, device=router_w.device)
    check(ctx.handle, lib.wmoe_pack_router(ctx.handle, _ptr(router_w.contiguous()), _ptr(shared_gate.contiguous()),
                                           E, H, _ptr(out), _stream()))
    return out


def split_router(router_w: torch.Tensor, ctx: Optional[Context] = None) -> torch.Tensor:
    """The router [E, H] as three bf16 terms [3, E, H] summing to it (wmoe_split_router): with it, the router
    logits of bf16 tokens run on the tensor cores at float32 accuracy."""
    ctx = ctx or default_context()
    E, H = router_w.shape
    out = torch.empty(3, E, H, dtype=torch.bfloat16, device=router_w.device)
    check(ctx.handle, lib.wmoe_split_router(ctx.handle, _ptr(router_w.contiguous()), E, H, _ptr(out), _stream()))
    return out


@dataclass
class LayerWeights:
    """One layer's non-routed MoE weights on the GPU: router f32 [E, H], optional routing bias f32 [E], shared
    expert gate vector f32 [H], shared expert gate_up (Q4_K bytes, uint8) and down (Q6_K bytes, uint8), and two
    prepared forms of the router made once by prepare(): packed (decode) and split into bf16 terms (prefill)."""
    router_w: torch.Tensor
    shared_gate: torch.Tensor
    shared_gate_up: torch.Tensor
    shared_down: torch.Tensor
    router_bias: Optional[torch.Tensor] = None
    router_packed: Optional[torch.Tensor] = None
    router_split: Optional[torch.Tensor] = None

    def prepare(self, ctx: Optional[Context] = None, decode: bool = True, prefill: bool = True) -> "LayerWeights":
        if decode and self.router_packed is None:
            self.router_packed = pack_router(self.router_w, self.shared_gate, ctx)
        if prefill and self.router_split is None:
            self.router_split = split_router(self.router_w, ctx)
        return self

    def as_struct(self) -> _lib.LayerWeights:
        opt = lambda t: None if t is None else t.data_ptr()
        return _lib.LayerWeights(self.router_w.data_ptr(), opt(self.router_bias), self.shared_gate.data_ptr(),
                                 self.shared_gate_up.data_ptr(), self.shared_down.data_ptr(), opt(self.router_packed),
                                 opt(self.router_split))


def moe_forward(store: ExpertStore, layer: int, x: torch.Tensor, lw: LayerWeights, top_k: int = 8,
                out_dtype: Optional[torch.dtype] = None, return_routing: bool = False):
    """One MoE block (engines/base.py:445-491) on x [T, H] (f32 or bf16) -> out [T, H] (x's dtype by default);
    with return_routing also (weights f32 [T, k], selected int32 [T, k]). Uses the prepared router forms that lw
    holds (LayerWeights.prepare)."""
    ctx = store.ctx
    x = x.contiguous()
    T = x.shape[0]
    out = torch.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device)
    sel = torch.empty(T, top_k, dtype=torch.int32, device=x.device) if return_routing else None
    w = torch.empty(T, top_k, dtype=torch.float32, device=x.device) if return_routing else None
    weights = lw.as_struct()
    check(ctx.handle, lib.wmoe_moe_forward_layer(ctx.handle, store.handle, layer, _ptr(x), _DTYPES[x.dtype], T,
                                                 top_k, ctypes.byref(weights), _ptr(out), _DTYPES[out.dtype],
                                                 _ptr(sel), _ptr(w), _stream()))
    return (out, w, sel) if return_routing else out


@dataclass
class EPPlan:
    """A rank's routing and send plan for one layer under expert parallelism (wmoe_ep_route_plan)."""
    topk_w: torch.Tensor       # f32 [T, k]
    topk_idx: torch.Tensor     # int32 [T, k]
    shared_s: torch.Tensor     # f32 [T]
    counts: torch.Tensor       # int32 [2, world]: rows, pairs to each rank
    send_buf: torch.Tensor     # fp16 [T * min(k, world), H] (first sum(rows) used)
    pair_list: torch.Tensor    # int32 [T * k, 2] (first sum(pairs) used)
    ret_index: torch.Tensor    # int32 [T, k]


def ep_route_plan(ctx: Context, world: int, x: torch.Tensor, lw: LayerWeights, experts: int = 256,
                  top_k: int = 8) -> EPPlan:
    """Step 1 of an expert-parallel layer on one rank (see include/wmoe.h): route x [T, H] and build what goes to
    each of the world ranks."""
    x = x.contiguous()
    T, H = x.shape
    dev = x.device
    rows = T * min(top_k, world)
    plan = EPPlan(topk_w=torch.empty(T, top_k, dtype=torch.float32, device=dev),
                  topk_idx=torch.empty(T, top_k, dtype=torch.int32, device=dev),
                  shared_s=torch.empty(T, dtype=torch.float32, device=dev),
                  counts=torch.zeros(2, world, dtype=torch.int32, device=dev),
                  send_buf=torch.empty(rows, H, dtype=torch.float16, device=dev),
                  pair_list=torch.empty(T * top_k, 2, dtype=torch.int32, device=dev),
                  ret_index=torch.empty(T, top_k, dtype=torch.int32, device=dev))
    weights = lw.as_struct()
    send_tok = torch.empty(max(rows, 1), dtype=torch.int32, device=dev)
    check(ctx.handle, lib.wmoe_ep_route_plan(ctx.handle, world, _ptr(x), _DTYPES[x.dtype], T, top_k, experts, H,
                                             ctypes.byref(weights), _ptr(plan.topk_w), _ptr(plan.topk_idx),
                                             _ptr(plan.shared_s), _ptr(plan.counts[0]), _ptr(plan.counts[1]),
                                             _ptr(send_tok), _ptr(plan.pair_list), _ptr(plan.ret_index),
                                             _ptr(plan.send_buf), _stream()))
    return plan


def ep_experts(store: ExpertStore, layer: int, world: int, recv_rows, recv_pairs, recv_buf: torch.Tensor,
               recv_pair_list: torch.Tensor, x: torch.Tensor, lw: LayerWeights) -> torch.Tensor:
    """Step 3: this rank's experts on the received rows (recv_rows / recv_pairs: per-source counts, host ints),
    plus the shared expert on its own tokens x. -> y fp16 [sum(recv_pairs) + T, H]."""
    ctx = store.ctx
    x = x.contiguous()
    T, H = x.shape
    rr = (ctypes.c_int32 * world)(*[int(v) for v in recv_rows])
    rp = (ctypes.c_int32 * world)(*[int(v) for v in recv_pairs])
    y = torch.empty(sum(int(v) for v in recv_pairs) + T, H, dtype=torch.float16, device=x.device)
    weights = lw.as_struct()
    check(ctx.handle, lib.wmoe_ep_experts(ctx.handle, store.handle, layer, world, rr, rp, _ptr(recv_buf),
                                          _ptr(recv_pair_list), _ptr(x), _DTYPES[x.dtype], T, ctypes.byref(weights),
                                          _ptr(y), _stream()))
    return y


def ep_combine(ctx: Context, plan: EPPlan, y_returned: torch.Tensor, y_shared: torch.Tensor,
               out_dtype: torch.dtype) -> torch.Tensor:
    """Step 5: the rank's outputs from the returned result rows and its shared-expert rows."""
    T, k = plan.topk_idx.shape
    H = y_shared.shape[1]
    out = torch.empty(T, H, dtype=out_dtype, device=y_shared.device)
    check(ctx.handle, lib.wmoe_ep_combine(ctx.handle, T, k, H, _ptr(plan.topk_idx), _ptr(plan.topk_w),
                                          _ptr(plan.ret_index), _ptr(plan.shared_s), _ptr(y_returned),
                                          _ptr(y_shared), _ptr(out), _DTYPES[out_dtype], _stream()))
    return out


class GpuEPOps:
    """The three per-rank steps of an expert-parallel layer, on this library's kernels."""

    @staticmethod
    def route_plan(store: ExpertStore, x: torch.Tensor, lw: LayerWeights, world: int, top_k: int) -> EPPlan:
        return ep_route_plan(store.ctx, world, x, lw, store.experts, top_k)

    @staticmethod
    def experts(store: ExpertStore, layer: int, world: int, recv_rows, recv_pairs, recv_buf, recv_pair_list, x, lw):
        return ep_experts(store, layer, world, recv_rows, recv_pairs, recv_buf, recv_pair_list, x, lw)

    @staticmethod
    def combine(store: ExpertStore, plan: EPPlan, y_returned, y_shared, out_dtype):
        return ep_combine(store.ctx, plan, y_returned, y_shared, out_dtype)


def moe_forward_ep(store, layer: int, x: torch.Tensor, lw: LayerWeights, group=None, top_k: int = 8,
                   out_dtype: Optional[torch.dtype] = None, return_routing: bool = False, ops=GpuEPOps,
                   stats: Optional[dict] = None):
    """One MoE block on this rank's tokens x [T, H] with the experts split over the ranks of `group`
    (torch.distributed; NCCL on GPUs): store holds this rank's block (ExpertStore(expert_range=...)). Same result
    as moe_forward on one GPU with every expert. The exchange: counts, then rows and pair lists, then result rows
    back, each one all_to_all_single. stats (optional dict, GPU only): CUDA events recorded after each stage
    (stats["events"]: [(stage, event)], the first "start") and the rows / pairs sent and received."""
    import torch.distributed as dist
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    per = store.experts // world
    if tuple(store.expert_range) != (rank * per, (rank + 1) * per):
        raise ValueError(f"rank {rank} of {world} must hold experts [{rank * per}, {(rank + 1) * per})")
    events = [] if stats is not None else None

    def mark(name):
        if events is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            events.append((name, ev))

    x = x.contiguous()
    mark("start")
    plan = ops.route_plan(store, x, lw, world, top_k)
    mark("route_plan")
    # counts: what this rank sends to each rank -> what each rank sends here (one host read for the sizes)
    send_counts = plan.counts.t().contiguous()  # [world, (rows, pairs)]
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=group)
    c = torch.cat([send_counts, recv_counts]).cpu()
    s_rows, s_pairs = c[:world, 0].tolist(), c[:world, 1].tolist()
    r_rows, r_pairs = c[world:, 0].tolist(), c[world:, 1].tolist()
    mark("counts")
    H = x.shape[1]
    recv_buf = plan.send_buf.new_empty(sum(r_rows), *plan.send_buf.shape[1:])
    recv_pairs = plan.pair_list.new_empty(sum(r_pairs), 2)
    dist.all_to_all_single(recv_buf, plan.send_buf[:sum(s_rows)], output_split_sizes=r_rows,
                           input_split_sizes=s_rows, group=group)
    dist.all_to_all_single(recv_pairs, plan.pair_list[:sum(s_pairs)], output_split_sizes=r_pairs,
                           input_split_sizes=s_pairs, group=group)
    mark("dispatch_a2a")
    y = ops.experts(store, layer, world, r_rows, r_pairs, recv_buf, recv_pairs, x, lw)
    mark("experts")
    P_r = sum(r_pairs)
    y_ret = y.new_empty(sum(s_pairs), H)
    dist.all_to_all_single(y_ret, y[:P_r].contiguous(), output_split_sizes=s_pairs, input_split_sizes=r_pairs,
                           group=group)
    mark("combine_a2a")
    out = ops.combine(store, plan, y_ret, y[P_r:], out_dtype or x.dtype)
    mark("combine")
    if stats is not None:
        stats.update(events=events, rows_out=sum(s_rows), pairs_out=sum(s_pairs), rows_in=sum(r_rows),
                     pairs_in=P_r, tokens=x.shape[0])
    return (out, plan.topk_w, plan.topk_idx) if return_routing else out


def ep_init(ctx: Context, group=None):
    """Creates the library's own NCCL communicator over the ranks of a torch.distributed group (wmoe_ep_init): rank 0
    makes the id, every rank receives it through the group. Needed once per context before moe_forward_ep_native."""
    import torch.distributed as dist
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    buf = (ctypes.c_uint8 * _lib.EP_ID_BYTES)()
    if rank == 0:
        check(ctx.handle, lib.wmoe_ep_unique_id(buf))
    obj = [bytes(buf)]
    dist.broadcast_object_list(obj, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
    uid = (ctypes.c_uint8 * _lib.EP_ID_BYTES).from_buffer_copy(obj[0])
    check(ctx.handle, lib.wmoe_ep_init(ctx.handle, uid, rank, world))


def moe_forward_ep_native(store: ExpertStore, layer: int, x: torch.Tensor, lw: LayerWeights, top_k: int = 8,
                          out_dtype: Optional[torch.dtype] = None, return_routing: bool = False):
    """moe_forward_ep in one library call (wmoe_moe_forward_ep) over the communicator of ep_init: one all-gather of
    the transfer counts, then the rows, pair lists and result rows copied by the copy engines into the peers'
    exchange windows (CUDA IPC), each exchange closed by a one-int all-reduce. Raises WmoeError (WMOE_ERR_NCCL) when a
    rank has left or NCCL failed; every later call of the context does so until ep_finalize and a new ep_init."""
    ctx = store.ctx
    x = x.contiguous()
    T = x.shape[0]
    out = torch.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device)
    sel = torch.empty(T, top_k, dtype=torch.int32, device=x.device) if return_routing else None
    w = torch.empty(T, top_k, dtype=torch.float32, device=x.device) if return_routing else None
    weights = lw.as_struct()
    check(ctx.handle, lib.wmoe_moe_forward_ep(ctx.handle, store.handle, layer, _ptr(x), _DTYPES[x.dtype], T, top_k,
                                              ctypes.byref(weights), _ptr(out), _DTYPES[out.dtype], _ptr(sel),
                                              _ptr(w), _stream()))
    return (out, w, sel) if return_routing else out


def decode_stack(store: ExpertStore, layers: list, h: torch.Tensor, eps: float = 1e-6, layer_begin: int = 0,
                 out: Optional[torch.Tensor] = None, return_routing: bool = False, pack: bool = True):
    """One decode token through len(layers) stacked blocks, h <- h + moe(rms_norm(h)) per layer, in one persistent
    launch. h: f32 [H] (or [1, H]) on the GPU. pack: give each layer a packed router first (the fast layout)."""
    ctx = store.ctx
    h = h.reshape(-1).contiguous()
    assert h.dtype == torch.float32
    out = torch.empty_like(h) if out is None else out
    for lw in layers:
        if pack and lw.router_packed is None:
            lw.router_packed = pack_router(lw.router_w, lw.shared_gate, ctx)
    arr = (_lib.LayerWeights * len(layers))(*[lw.as_struct() for lw in layers])
    sel = torch.empty(len(layers), 8, dtype=torch.int32, device=h.device) if return_routing else None
    check(ctx.handle, lib.wmoe_decode_stack(ctx.handle, store.handle, layer_begin, len(layers),
                                            ctypes.cast(arr, ctypes.c_void_p), ctypes.c_float(eps), _ptr(h),
                                            _ptr(out), _ptr(sel), _stream()))
    return (out, sel) if return_routing else out


def prefill_stack(store: ExpertStore, layers: list, h: torch.Tensor, eps: float = 1e-6, layer_begin: int = 0,
                  x_dtype: torch.dtype = torch.bfloat16, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """T tokens through len(layers) stacked blocks, h <- h + moe(rms_norm(h)) per layer (wmoe_prefill_stack): the
    residual add and the next layer's RMSNorm run in each layer's combine kernel. h: f32 [T, H] on the GPU; each
    block takes its input in x_dtype (bf16: the tensor-core router of LayerWeights.prepare). After ep_init each layer
    runs over the context's communicator, the store holding this rank's block of the experts (every rank passes its
    own tokens); a capped store prefetches each next layer. out may be h."""
    ctx = store.ctx
    h = h.contiguous()
    if h.dtype != torch.float32 or h.dim() != 2:
        raise ValueError("prefill_stack: h must be a float32 [T, H] tensor")
    out = torch.empty_like(h) if out is None else out
    arr = (_lib.LayerWeights * len(layers))(*[lw.as_struct() for lw in layers])
    check(ctx.handle, lib.wmoe_prefill_stack(ctx.handle, store.handle, layer_begin, len(layers),
                                             ctypes.cast(arr, ctypes.c_void_p), ctypes.c_float(eps), _ptr(h),
                                             h.shape[0], _DTYPES[x_dtype], _ptr(out), _stream()))
    return out


class CudaMoE:
    """Mixin that replaces willow's Engine.moe (engines/base.py:445-490) with the B200 kernels:

        class B200Qwen35(CudaMoE, Qwen35MoEEngine): ...
        engine = B200Qwen35(...)            # willow's loader as usual
        engine.wmoe_attach(gguf_path)       # routed experts into HBM, shared experts' GGUF bytes

    Weights by willow's own names through self.w(...): the router ``{prefix}layers.{L}.mlp.gate.weight`` and the
    shared-expert gate ``.mlp.shared_expert_gate.weight`` (willow keeps them dequantised, bf16 or f32: they are
    widened to f32 exactly), and ``.mlp.gate.bias`` when present. willow's loader dequantises the shared expert, so
    its GGUF bytes come from the file (wmoe_attach), or from ``.mlp.shared_expert.gate_up_proj.qweight`` (Q4_K,
    gate rows then up rows) and ``.mlp.shared_expert.down_proj.qweight`` when the engine keeps them. Routed experts
    come from self.experts, an ExpertStore of this module.

    The engine's settings keep their meaning:
    * min_expert_weight (main.py:37,108): routed picks below it are dropped as skip_small_experts does
      (base.py:413-429);
    * residual with prefetch_top_k (base.py:392-406,450,473-474): for a decode token on a capped store, the next
      layer's router runs on the engine's router_guess_input(residual, layer + 1) and the experts it picks start
      copying into HBM (ExpertStore.prefetch) while this layer computes.
    Returns the block's output in x's dtype, like Engine.moe."""

    top_k = 8

    def wmoe_attach(self, gguf_path: str, cap_bytes: int = 0, ctx: Optional[Context] = None):
        """Reads the GGUF's routed experts into an ExpertStore (self.experts; capped at cap_bytes of HBM when given)
        and keeps each layer's shared-expert bytes on the GPU for moe_layer_weights."""
        from . import gguf_store
        store, lws = gguf_store.load(gguf_path, ctx=ctx, cap_bytes=cap_bytes)
        self.experts = store
        self._wmoe_shared = {layer: (lw.shared_gate_up, lw.shared_down) for layer, lw in enumerate(lws)}
        self.__dict__.pop("_wmoe_layers", None)
        return store

    def moe_layer_weights(self, layer: int) -> LayerWeights:
        """The layer's weights with their prepared router forms, made on first use and kept."""
        cache = self.__dict__.setdefault("_wmoe_layers", {})
        if layer not in cache:
            p = f"{self.prefix}layers.{layer}.mlp"
            dev = torch.device("cuda", self.experts.ctx.device)
            f32 = lambda t: t.to(device=dev, dtype=torch.float32).contiguous()
            shared = getattr(self, "_wmoe_shared", {}).get(layer)
            if shared is None:
                shared = (self.w(p + ".shared_expert.gate_up_proj.qweight"),
                          self.w(p + ".shared_expert.down_proj.qweight"))
            bias = self.weights.get(p + ".gate.bias")
            cache[layer] = LayerWeights(router_w=f32(self.w(p + ".gate.weight")),
                                        shared_gate=f32(self.w(p + ".shared_expert_gate.weight").reshape(-1)),
                                        shared_gate_up=shared[0].to(dev).contiguous(),
                                        shared_down=shared[1].to(dev).contiguous(),
                                        router_bias=None if bias is None else f32(bias)).prepare(self.experts.ctx)
        return cache[layer]

    def moe(self, x: torch.Tensor, layer: int, residual: torch.Tensor = None) -> torch.Tensor:
        lw = self.moe_layer_weights(layer)
        ctx = self.experts.ctx
        ctx.set_min_expert_weight(float(getattr(self, "min_expert_weight", 0.0) or 0.0))
        shape = x.shape
        flat = x.reshape(-1, shape[-1])
        out = moe_forward(self.experts, layer, flat, lw, self.top_k)
        # willow starts the next layer's guessed reads after this layer's (base.py:471-474); here they are queued
        # behind this layer's kernels on the same stream, and the copies run on the store's side stream
        following = layer + 1
        k = int(getattr(self, "prefetch_top_k", 0) or 0)
        if (residual is not None and k and self.experts.capped and flat.shape[0] == 1
                and following < getattr(self, "num_layers", self.experts.layers)):
            guess_in = self.router_guess_input(residual.reshape(-1, shape[-1]), following) \
                if hasattr(self, "router_guess_input") else None
            guess_next_layer(self.experts, residual.reshape(-1, shape[-1]), self.moe_layer_weights(following),
                             following, top_k=min(k, self.top_k), guess_input=guess_in)
        return out.view(shape)
