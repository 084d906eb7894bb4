"""ctypes binding of libk2b (include/k2b.h).

The library is the only compute path: if it is missing or fails to load, every
op raises.  There is no eager / PyTorch / CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libk2b.so")

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_LL = ctypes.c_longlong

# name -> (restype, argtypes); mirrors include/k2b.h
SIGNATURES = {
    "k2b_version": (ctypes.c_char_p, []),
    "k2b_device_error": (_I, [_I, _P]),
    "k2b_selftest_wait": (_I, [_I, _LL, _P, _P]),
    "k2b_norm_quant": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _P]),
    "k2b_rotate_quant": (_I, [_P, _P, _P, _I, _I, _P]),
    "k2b_prepare_weight": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P]),
    "k2b_gemm_f32": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _P]),
    "k2b_gemm_bf16": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _P]),
    "k2b_qkv": (_I, [_P] * 17 + [_I, _I, _I, _I, _I, _F, _F, _P]),
    "k2b_gated_residual": (_I, [_P] * 7 + [_I, _I, _I, _I, _P]),
    "k2b_gated_add": (_I, [_P] * 4 + [_I, _I, _I, _I, _P]),
    "k2b_reduce_gated_add": (_I, [_P, _I, ctypes.c_longlong, _P, _P, _P, _I, _I, _I, _I, _P]),
    "k2b_gemm_f32_scatter": (_I, [_P] * 5 + [_I] * 6 + [_P]),
    "k2b_ipc_alloc": (_I, [ctypes.c_longlong, _P, _P]),
    "k2b_ipc_open": (_I, [_P, _P]),
    "k2b_ipc_close": (_I, [_P]),
    "k2b_ipc_free": (_I, [_P]),
    "k2b_norm_quant_rows": (_I, [_P] * 6 + [_I, _I, _I, _I, _I, _I, _F, _P]),
    "k2b_swiglu_quant": (_I, [_P] * 8 + [_I, _I, _I, _P]),
    "k2b_swiglu_bf16": (_I, [_P] * 7 + [_I, _I, _I, _P]),
    "k2b_attention": (_I, [_P] * 5 + [_I] * 6 + [_LL] * 9 + [_I, _P]),
    "k2b_attention_quant": (_I, [_P] * 5 + [_I] * 6 + [_LL] * 9 + [_P]),
    "k2b_block_slots": (_I, []),
    "k2b_block_workspace_bytes": (_LL, [_I] * 5),
    "k2b_forward_blocks": (_I, [_P, _I, _P, _P, _P, _LL, _I, _I, _I, _I, _I, _I, _F, _F, _P, _P]),
    "k2b_static_workspace_bytes": (_LL, []),
    "k2b_forward_blocks_static": (_I, [_P, _I, _P, _P, _I, _I, _I, _I, _I, _I, _F, _F, _P]),
    "k2_norm_mod_quant4": (_I, [_P] * 6 + [_I] * 5 + [_F, _I, _I, _P]),
    "k2_int4_qkv": (_I, [_P] * 17 + [_I] * 5 + [_F, _F, _P]),
    "k2_int4_swiglu": (_I, [_P] * 7 + [_I] * 4 + [_P]),
    "k2_int4_gated_residual": (_I, [_P] * 7 + [_I] * 5 + [_P]),
    "k2_int4_qk_norm_rope": (_I, [_P] * 7 + [_I] * 4 + [_F, _P]),
    "k2b_norm_mod": (_I, [_P] * 5 + [_I] * 5 + [_F, _P]),
    "k2b_elementwise": (_I, [_P] * 4 + [_LL, _I, _I, _P]),
    "k2b_rope": (_I, [_P] * 5 + [_I] * 6 + [_P]),
    "k2_int4_residual_norm": (_I, [_P] * 12 + [_I] * 4 + [_F, _P]),
    "k2_norm": (None, [_P] * 5 + [_I] * 5 + [_F, _I, _P]),
    "k2_quant4": (None, [_P] * 3 + [ctypes.c_int64] * 2 + [_I, _I, _P]),
    "k2_elementwise": (None, [_P] * 4 + [ctypes.c_int64, _I, _I, _I, _P]),
    "k2_rope": (None, [_P] * 5 + [_I] * 7 + [_P]),
    "k2b_shim_status": (_I, [_I]),
    "k2_quant8": (None, [_P] * 3 + [ctypes.c_int64] * 2 + [_I, _I, _P]),
    "k2b_gemm8": (_I, [_P, _P, _I, _P, _P, _I, _P, _P, _I, _I, _I, _P]),
    "k2b_lora_gemm": (_I, [_I] + [_P] * 7 + [_I, _P, _P, _I, _F, _P, _I, _I, _I, _P]),
    "k2b_lora_swiglu": (_I, [_I] + [_P] * 8 + [_I, _F, _P, _P, _I, _F, _P, _I, _I, _I, _P]),
    "k2b_gemm_f8": (_I, [_P, _P, _I, _P, _P, _I, _P, _P, _I, _I, _I, _I, _I, _P]),
    "k2b_ref_qkv": (_I, [_P] * 17 + [_I, _I, _I, _I, _I, _F, _F, _P]),
    "k2b_ref_gated_residual": (_I, [_P] * 7 + [_I, _I, _I, _I, _P]),
    "k2b_ref_qkv8": (_I, [_P] * 17 + [_I, _I, _I, _I, _I, _F, _F, _P]),
    "k2b_ref_quant4_e4m3": (_I, [_P, _P, _P, ctypes.c_longlong, ctypes.c_longlong, _I, _P]),
    "k2b_ref_norm_quant4_e4m3": (_I, [_P] * 6 + [_I, _I, _I, _I, _I, _F, _I, _P]),
    "k2b_ref_swiglu8": (_I, [_P] * 7 + [_I, _I, _I, _P]),
    "k2b_ref_gated_residual8": (_I, [_P] * 7 + [_I, _I, _I, _I, _P]),
    "k2_gemm4": (None, [_P] * 6 + [ctypes.c_int64] * 3 + [_I, _P]),
    "k2_dequant8": (None, [_P] * 5 + [ctypes.c_int64] * 3 + [_I, _P]),
    "k2_fp8": (None, [_P, _P, _P, ctypes.c_int64, _I, _I, ctypes.c_bool, _P]),
    "k2b_norm_quant_e4m3": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _P]),
    "k2b_attention_quant_e4m3": (_I, [_P] * 5 + [_I] * 6 + [_LL] * 9 + [_P]),
    "k2b_gemm_f32_e4m3": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _P]),
    "k2b_qkv_e4m3": (_I, [_P] * 17 + [_I, _I, _I, _I, _I, _F, _F, _P]),
    "k2b_gated_residual_e4m3": (_I, [_P] * 7 + [_I, _I, _I, _I, _P]),
    "k2b_swiglu_quant_e4m3": (_I, [_P] * 8 + [_I, _I, _I, _P]),
    "k2b_gemm_bf16_e4m3": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _P]),
    "k2b_swiglu_bf16_e4m3": (_I, [_P] * 7 + [_I, _I, _I, _P]),
    "k2b_swiglu_quant_a8": (_I, [_P] * 8 + [_I, _I, _I, _P]),
    "k2b_gemm_f32_scatter_e4m3": (_I, [_P] * 5 + [_I] * 6 + [_P]),
    "k2b_expand_e4m3": (_I, [_P, _P, ctypes.c_longlong, _P]),
}

_lib = None
_lock = threading.Lock()


class K2BError(RuntimeError):
    """A libk2b entry point returned a non-zero status."""


def lib() -> ctypes.CDLL:
    """Load libk2b (building it first if this is a source tree without it)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                build_py = os.path.join(os.path.dirname(os.path.dirname(LIB_PATH)), "..", "build.py")
                if not os.path.exists(build_py):
                    raise K2BError(f"libk2b not built: {LIB_PATH} is missing")
                import importlib.util

                spec = importlib.util.spec_from_file_location("_k2b_build", build_py)
                mod = importlib.util.module_from_spec(spec)
                spec.loader.exec_module(mod)
                mod.build()
            L = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise K2BError(f"{what} failed with status {rc}")
