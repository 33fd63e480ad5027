"""ctypes binding of libwmoe.so (include/wmoe.h). Importing this module loads the library and fails loudly when it
is missing: there is no CPU fallback. Build it with ``python -m willow_v2_b200.build``."""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libwmoe.so")

OK = 0
ERR_INVALID, ERR_CUDA, ERR_CAPACITY, ERR_DEVICE, ERR_UNSUPPORTED, ERR_IO, ERR_NCCL = -1, -2, -3, -4, -5, -6, -7
F32, BF16, F16 = 0, 1, 2
GGML_Q4_K, GGML_Q6_K = 12, 14
# ggml type ids of every type wmoe_dequant and the typed kernels (wmoe_gemv*) run (gguf/reader.py:14-48)
GGML_TYPES = {"Q5_0": 6, "Q8_0": 8, "Q4_K": 12, "Q6_K": 14, "IQ3_XXS": 18, "IQ4_NL": 20, "IQ3_S": 21, "IQ2_S": 22,
              "IQ4_XS": 23, "Q2_0": 42}
STATUS_NAMES = {1: "expert id out of range", 2: "expert not resident", 3: "grid barrier timed out",
                4: "bad segment", 5: "value out of the range of an fp16 intermediate"}

# every symbol include/wmoe.h declares, with (restype, argtypes)
_p, _i, _sz, _u64, _f = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.c_uint64, ctypes.c_float
_pp = ctypes.POINTER(ctypes.c_void_p)
SIGNATURES = {
    "wmoe_init": (_i, [_i, _pp]),
    "wmoe_destroy": (None, [_p]),
    "wmoe_last_error": (ctypes.c_char_p, [_p]),
    "wmoe_launch_count": (_u64, [_p]),
    "wmoe_set_decode_kernel": (_i, [_p, _i]),
    "wmoe_set_trace": (_i, [_p, _p, _sz]),
    "wmoe_set_prefill_threshold": (_i, [_p, _i]),
    "wmoe_set_min_expert_weight": (_i, [_p, _f]),
    "wmoe_ep_set_timeout": (_i, [_p, _i]),
    "wmoe_set_profiling": (_i, [_p, _i]),
    "wmoe_phase_ms": (_i, [_p, _i, _i, ctypes.POINTER(_f)]),
    "wmoe_decode_ctas": (_i, [_p]),
    "wmoe_device_status": (_i, [_p, ctypes.POINTER(_i), _p]),
    "wmoe_dequant": (_i, [_p, _i, _p, _sz, _p, _i, _p]),
    "wmoe_route": (_i, [_p, _p, _i, _i, _i, _i, _i, _p, _p, _p, _p, _p, _p, _p, _p]),
    "wmoe_dispatch": (_i, [_p, _p, _i, _i, _i, _p, _p, _p, _p, _p]),
    "wmoe_pack_router": (_i, [_p, _p, _p, _i, _i, _p, _p]),
    "wmoe_split_router": (_i, [_p, _p, _i, _i, _p, _p]),
    "wmoe_store_create": (_i, [_p, _i, _i, _i, _i, _sz, _pp]),
    "wmoe_store_create_range": (_i, [_p, _i, _i, _i, _i, _i, _i, _sz, _pp]),
    "wmoe_store_destroy": (None, [_p]),
    "wmoe_store_upload": (_i, [_p, _i, _i, _p, _p]),
    "wmoe_store_fill_synthetic": (_i, [_p, _u64, _i, _i, _p]),
    "wmoe_store_blob_bytes": (_sz, [_p]),
    "wmoe_store_prepare": (_i, [_p, _i, _p, _i, _p]),
    "wmoe_store_prefetch": (_i, [_p, _i, _p, _i, _p]),
    "wmoe_store_set_down_type": (_i, [_p, _i, _i]),
    "wmoe_store_layer_blob_bytes": (_sz, [_p, _i]),
    "wmoe_store_choose_hot": (_i, [_p, ctypes.c_double]),
    "wmoe_store_prefetch_stats": (_i, [_p, ctypes.POINTER(_u64), ctypes.POINTER(_u64)]),
    "wmoe_add_rmsnorm": (_i, [_p, _p, _p, _i, _i, _i, ctypes.c_float, _p, _p, _i, _p]),
    "wmoe_store_download": (_i, [_p, _i, _i, _p, _p]),
    "wmoe_store_blob": (_p, [_p, _i, _i]),
    "wmoe_store_stats": (_i, [_p, ctypes.POINTER(_u64), ctypes.POINTER(_u64), ctypes.POINTER(_u64),
                              ctypes.POINTER(_u64)]),
    "wmoe_moe_forward": (_i, [_p, _p, _i, _p, _i, _i, _i, _p, _p, _p, _p, _p, _p, _i, _p, _p, _p]),
    "wmoe_moe_forward_layer": (_i, [_p, _p, _i, _p, _i, _i, _i, _p, _p, _i, _p, _p, _p]),
    "wmoe_decode_stack": (_i, [_p, _p, _i, _i, _p, _f, _p, _p, _p, _p]),
    "wmoe_decode_stack_noalloc": (_i, [_p, _p, _i, _i, _p, _f, _p, _p, _p, _p]),
    "wmoe_prefill_stack": (_i, [_p, _p, _i, _i, _p, _f, _p, _i, _i, _p, _p]),
    "wmoe_ggml_row_bytes": (_sz, [_i, _i]),
    "wmoe_gemv": (_i, [_p, _i, _p, _i, _i, _p, _i, _i, _p, _i, _p]),
    "wmoe_gemv_batch": (_i, [_p, _i, _p, _p, _i, _i, _i, _i, _p, _i, _p, _i, _p]),
    "wmoe_gemv_combine": (_i, [_p, _i, _p, _p, _i, _i, _i, _i, _p, _p, _i, _p, _p]),
    "wmoe_expert_gate": (_i, [_p, _p, _i, _i, _p, _p]),
    "wmoe_batched_decode_experts": (_i, [_p, _i, _i, _i, _i, _p, _p, _p, _i, _i, _p, _p, _p, _p]),
    "wmoe_ep_route_plan": (_i, [_p, _i, _p, _i, _i, _i, _i, _i, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p]),
    "wmoe_ep_experts": (_i, [_p, _p, _i, _i, _p, _p, _p, _p, _p, _i, _i, _p, _p, _p]),
    "wmoe_ep_combine": (_i, [_p, _i, _i, _i, _p, _p, _p, _p, _p, _p, _p, _i, _p]),
    "wmoe_ep_unique_id": (_i, [_p]),
    "wmoe_ep_init": (_i, [_p, _p, _i, _i]),
    "wmoe_ep_finalize": (_i, [_p]),
    "wmoe_ep_set_chunks": (_i, [_p, _i]),
    "wmoe_ep_uses_copy_engines": (_i, [_p]),
    "wmoe_moe_forward_ep": (_i, [_p, _p, _i, _p, _i, _i, _i, _p, _p, _i, _p, _p, _p]),
}


class LayerWeights(ctypes.Structure):
    """wmoe_layer_weights: device pointers of one layer's router, bias, shared gate, shared expert and the two
    prepared router forms."""
    _fields_ = [("router_w", _p), ("router_bias", _p), ("shared_gate", _p), ("shared_gate_up", _p),
                ("shared_down", _p), ("router_packed", _p), ("router_split", _p)]


ROUTER_STRIDE = 264  # WMOE_ROUTER_STRIDE
PHASES = ("router", "dispatch", "gather", "gate_up", "down", "combine")  # WMOE_PHASES, in order
EP_PHASES = ("route_plan", "counts", "first_rows", "experts", "last_results", "combine")  # wmoe_moe_forward_ep
MAX_RANKS = 8  # WMOE_MAX_RANKS
EP_ID_BYTES = 128  # WMOE_EP_ID_BYTES


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `python -m willow_v2_b200.build`")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


class WmoeError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code


def check(ctx, code: int):
    if code != OK:
        msg = lib.wmoe_last_error(ctx)
        raise WmoeError(code, msg.decode() if msg else "unknown error")
