"""The C ABI boundary without a GPU: the library loads and exports every symbol include/wmoe.h declares, and the
host-side pieces of the synthetic generator agree with numpy."""
import ctypes
import os
import re

import numpy as np
import pytest

from conftest import REPO

HEADER = os.path.join(REPO, "include", "wmoe.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(wmoe_[a-z_0-9]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from willow_v2_b200 import lib as L
    syms = declared_symbols()
    assert len(syms) >= 20
    for name in syms:
        assert hasattr(L.lib, name), name
    # the ctypes table covers exactly the header
    assert sorted(L.SIGNATURES) == syms


def test_library_rejects_bad_arguments_without_a_gpu():
    from willow_v2_b200 import lib as L
    # null output handle: refused before touching CUDA
    assert L.lib.wmoe_init(0, None) == L.ERR_INVALID
    assert L.lib.wmoe_dequant(None, L.GGML_Q4_K, None, 0, None, L.F32, None) == L.ERR_INVALID
    assert L.lib.wmoe_prefill_stack(None, None, 0, 1, None, L.ctypes.c_float(1e-6), None, 4, L.BF16, None,
                                    None) == L.ERR_INVALID
    assert L.lib.wmoe_expert_gate(None, None, 1, 512, None, None) == L.ERR_INVALID
    assert L.lib.wmoe_ep_uses_copy_engines(None) == -1
    assert L.lib.wmoe_store_blob_bytes(None) == 0
    assert L.lib.wmoe_launch_count(None) == 0


def test_layer_weights_struct_matches_header():
    """The ctypes mirror of wmoe_layer_weights has the header's fields, in order, all pointers."""
    import re
    from willow_v2_b200 import lib as L
    text = open(os.path.join(REPO, "include", "wmoe.h")).read()
    body = re.search(r"typedef struct wmoe_layer_weights \{(.*?)\} wmoe_layer_weights;", text, re.S).group(1)
    names = re.findall(r"\*\s*(\w+);", body)
    assert names == [f[0] for f in L.LayerWeights._fields_]
    assert ctypes.sizeof(L.LayerWeights) == len(names) * ctypes.sizeof(ctypes.c_void_p)


def f64_to_f16_rne(v: float) -> int:
    """The integer algorithm of csrc/synth.cuh (positive normal values), in Python."""
    b = np.array([v], dtype=np.float64).view(np.uint64)[0].item()
    e = ((b >> 52) & 0x7FF) - 1023
    m = b & ((1 << 52) - 1)
    h = ((e + 15) << 10) | (m >> 42)
    rem, half = m & ((1 << 42) - 1), 1 << 41
    if rem > half or (rem == half and (h & 1)):
        h += 1
    return h


def test_fp16_rounding_of_generator_matches_numpy():
    rng = np.random.default_rng(1)
    u = rng.integers(0, 1 << 24, 20000).astype(np.float64)
    vals = u * (3e-3 / 16777216.0) + 1e-3
    # exact ties and values right at binade edges
    vals = np.concatenate((vals, [2.0 ** -10, 2.0 ** -9, 2.0 ** -9 * (1 + 2.0 ** -11),
                                  2.0 ** -9 * (1 + 3 * 2.0 ** -11)]))
    ref = vals.astype(np.float16).view(np.uint16)
    got = np.array([f64_to_f16_rne(float(v)) for v in vals], dtype=np.uint16)
    np.testing.assert_array_equal(got, ref)


def test_header_cites_reference_for_each_entry_point():
    text = open(HEADER).read()
    for sym in ("wmoe_dequant", "wmoe_route", "wmoe_dispatch", "wmoe_moe_forward", "wmoe_decode_stack",
                "wmoe_store_*", "wmoe_gemv_batch", "wmoe_gemv", "wmoe_gemv_combine", "wmoe_ggml_row_bytes"):
        assert re.search(re.escape(sym) + r"\s+\S+\.py:\d+", text), sym


@pytest.mark.parametrize("path", ["willow_v2_b200/moe.py", "willow_v2_b200/lib.py", "bench.py"])
def test_product_code_never_imports_the_oracle(path):
    full = os.path.join(REPO, path)
    if not os.path.exists(full):
        pytest.skip("not written yet")
    src = open(full).read()
    if path == "bench.py":
        # only the CPU-baseline leg may use it, inside a function
        assert "import oracle" not in src.split("def cpu_baseline")[0]
    else:
        assert "oracle" not in src
