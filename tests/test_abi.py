"""libk2b loads and exports every entry point include/k2b.h declares; the host
side of each entry point rejects bad sizes before touching the GPU.  No GPU."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "k2b.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(k2b?_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from k2b._native import LIB_PATH, lib as load

    if not os.path.exists(LIB_PATH):
        pytest.skip("libk2b not built (run __graft_entry__.build())")
    return load()


def test_header_declares_expected_entry_points():
    names = declared_symbols()
    for n in ("k2b_norm_quant", "k2b_qkv", "k2b_attention", "k2b_forward_blocks", "k2_norm_mod_quant4",
              "k2_int4_qkv", "k2_int4_swiglu", "k2_int4_gated_residual", "k2_int4_qk_norm_rope"):
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    from k2b._native import LIB_PATH, SIGNATURES

    out = subprocess.run(["nm", "-D", "--defined-only", LIB_PATH], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [n for n in declared_symbols() if n not in exported]
    assert not missing, missing
    # and the ctypes binding table covers them all
    assert not [n for n in declared_symbols() if n not in SIGNATURES]
    # nothing else leaks out of the library
    extra = [n for n in exported if n.startswith("k2")] 
    assert sorted(extra) == declared_symbols()


def test_version_and_layout_queries(lib):
    assert lib.k2b_version().startswith(b"k2b")
    assert lib.k2b_block_slots() == 19
    assert lib.k2b_block_workspace_bytes(4050, 6144, 48, 12, 16384) > 0
    assert lib.k2b_block_workspace_bytes(0, 6144, 48, 12, 16384) == -1
    assert lib.k2b_static_workspace_bytes() == 64 << 20


@pytest.mark.parametrize("call", [
    lambda L: L.k2b_norm_quant(None, None, None, None, None, None, 0, 6144, 1, -1, 1, ctypes.c_float(1e-6), None),
    lambda L: L.k2b_norm_quant(None, None, None, None, None, None, 4, 6000, 4, -1, 1, ctypes.c_float(1e-6), None),
    lambda L: L.k2b_rotate_quant(None, None, None, 4, 100, None),
    lambda L: L.k2b_gemm_f32(None, None, None, None, None, 128, 256, 100, None),
    lambda L: L.k2b_gemm_f32(None, None, None, None, None, 128, 100, 128, None),
    lambda L: L.k2b_swiglu_quant(None, None, None, None, None, None, None, None, 128, 100, 128, None),
    lambda L: L.k2b_attention(None, None, None, None, None, 1, 3, 1, 16, 16, 128, *([8] * 9), 0, None),
    lambda L: L.k2b_attention(None, None, None, None, None, 1, 4, 2, 16, 16, 64, *([8] * 9), 0, None),
    lambda L: L.k2b_prepare_weight(None, None, None, None, 0, 128, 1, 1, 0, 1, None),
    lambda L: L.k2_norm_mod_quant4(None, None, None, None, None, None, 4, 6144, 4, -1, 1, ctypes.c_float(1e-6), 256, 2,
                                   None),
    lambda L: L.k2_int4_qkv(*([None] * 17), 128, 256, 256, 128, 1, ctypes.c_float(1e-6), ctypes.c_float(1e-6), None),
    lambda L: L.k2b_forward_blocks(None, 1, None, None, None, 0, 1, 1, 6144, 48, 12, 16384, ctypes.c_float(1e-6),
                                   ctypes.c_float(1e-6), None, None),
])
def test_invalid_arguments_are_rejected_on_the_host(lib, call):
    """cudaErrorInvalidValue (1), returned before any launch (kernels/norm_quant.cu:92 convention)."""
    assert call(lib) == 1


# Every symbol the reference's runtime resolves from its kernel libraries with
# dlopen(RTLD_NOW | RTLD_LOCAL) + dlsym, each failing with "Missing native
# symbol" (native_runtime.cpp:34-48): configure() (:514-521), configure_joint()
# (:524-528), configure_norm_quant() (:529).
REFERENCE_SYMBOLS = {
    "configure: kernels": ["k2_quant4", "k2_quant8", "k2_gemm4", "k2_dequant8", "k2_fp8", "k2_norm",
                           "k2_elementwise", "k2_rope"],
    "configure: epilogue": ["k2_int4_gated_residual"],
    "configure: qk": ["k2_int4_qk_norm_rope"],
    "configure_joint": ["k2_int4_swiglu", "k2_int4_qkv", "k2_int4_residual_norm"],
    "configure_norm_quant": ["k2_norm_mod_quant4"],
}


def test_reference_runtime_resolves_every_symbol():
    """libk2b opened the way the reference's configure() opens its libraries
    resolves every name each configure* call loads."""
    import os

    from k2b._native import LIB_PATH

    h = ctypes.CDLL(LIB_PATH, mode=os.RTLD_NOW | os.RTLD_LOCAL)
    missing = [n for names in REFERENCE_SYMBOLS.values() for n in names if not hasattr(h, n)]
    assert not missing, missing
