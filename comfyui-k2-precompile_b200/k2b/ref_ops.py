"""Torch-level wrappers over libk2b's reference-contract kernels.

The reference's runtime quantises and projects with one fp32 scale per
activation row and per weight channel (native_runtime.cpp:262-311):

* format 1, INT4: ConvRot (groups 16/64/256) + per-row INT4, packed [m, k/2]
  with the even column in the low nibble; the checkpoint's packed weights
  [n, k/2] with fp32 per-channel scales are streamed as stored;
* format 2, INT8: ConvRot (or none, group 0) + per-row int8 [m, k]; int8
  weights [n, k]; int32 accumulation, T(acc * xs * ws + bias);
* formats 3 / 4, FP8 e4m3 / e5m2: x / s with one fp32 scale s (the
  binding's input scale, or amax / fmax); fp8 weights [n, k] with their scale.

Every projection here is the tcgen05 pair GEMM with the whole of k in one
accumulator and the dequant (and the reference's fused epilogue) in the
epilogue.  Outputs are bf16 (the reference computes in the activation dtype;
this build serves bf16 activations only).  Nothing here computes on the CPU;
``K2BError`` carries a kernel's non-zero status.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence, Tuple

import torch

from ._native import K2BError, check, lib
from .ops import _cuda, _need, _p, _stream

FP8_FORMATS = {3: (torch.float8_e4m3fn, 5, 448.0), 4: (torch.float8_e5m2, 6, 57344.0)}
GROUPS4 = (16, 64, 256)


def _shim(name: str) -> None:
    """Raise on the status a void reference-named export left behind."""
    rc = int(lib().k2b_shim_status(1))
    if rc:
        raise K2BError(f"{name} failed with CUDA status {rc}")


def _bf16(x: torch.Tensor, what: str) -> None:
    _need(x.dtype == torch.bfloat16, f"{what}: bf16 activations expected (fp16 / fp32 are not served)")


# ------------------------------------------------------------- quantisers

def quant4(x: torch.Tensor, group: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """k2_quant4: x bf16 [m, k] -> (int8 [m, k/2] packed codes, fp32 [m, 1])."""
    _cuda(x)
    _bf16(x, "quant4")
    _need(group in GROUPS4, f"quant4: ConvRot group {group} not in {GROUPS4}")
    m, k = x.shape
    _need(k % group == 0 and k % 8 == 0, "quant4: k must be a multiple of the group")
    q = torch.empty((m, k // 2), dtype=torch.int8, device=x.device)
    s = torch.empty((m, 1), dtype=torch.float32, device=x.device)
    if m:
        lib().k2b_shim_status(1)
        lib().k2_quant4(_p(x), _p(q), _p(s), m, k, group, 2, _stream())
        _shim("k2_quant4")
    return q, s


def quant8(x: torch.Tensor, group: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """k2_quant8: x bf16 [m, k] -> (int8 [m, k], fp32 [m, 1]); group 0 = no
    rotation."""
    _cuda(x)
    _bf16(x, "quant8")
    _need(group == 0 or group in GROUPS4, f"quant8: ConvRot group {group} not in (0,) + {GROUPS4}")
    m, k = x.shape
    _need(k % 8 == 0 and (group == 0 or k % group == 0), "quant8: k must be a multiple of the group")
    q = torch.empty((m, k), dtype=torch.int8, device=x.device)
    s = torch.empty((m, 1), dtype=torch.float32, device=x.device)
    if m:
        lib().k2b_shim_status(1)
        lib().k2_quant8(_p(x), _p(q), _p(s), m, k, group, 2, _stream())
        _shim("k2_quant8")
    return q, s


def norm_quant4(x: torch.Tensor, w: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor, *, length: int,
                cut: int = -1, eps: float = 1e-6, group: int = 256) -> Tuple[torch.Tensor, torch.Tensor]:
    """k2_norm_mod_quant4: RMSNorm + modulation + ConvRot + per-row INT4 of
    x bf16 [rows, K] (latents of ``length`` rows, modulation rows [nb, K])."""
    _cuda(x, w, scale, shift)
    _bf16(x, "norm_quant4")
    _need(scale.dtype == torch.bfloat16 and shift.dtype == torch.bfloat16 and w.dtype == torch.float32,
          "norm_quant4: fp32 norm weight and bf16 modulation expected")
    _need(group in GROUPS4, f"norm_quant4: ConvRot group {group} not in {GROUPS4}")
    rows, K = x.shape
    batch = max(1, rows // max(1, length))
    nb = scale.numel() // K
    _need(w.numel() == K and scale.shape[-1] == K and shift.numel() == scale.numel(), "norm_quant4: width mismatch")
    _need(nb >= (2 * batch if cut >= 0 else batch), "norm_quant4: modulation rows do not cover the batch")
    q = torch.empty((rows, K // 2), dtype=torch.int8, device=x.device)
    s = torch.empty((rows, 1), dtype=torch.float32, device=x.device)
    if rows:
        check(lib().k2_norm_mod_quant4(_p(x), _p(w), _p(scale), _p(shift), _p(q), _p(s), rows, K, length, cut, batch,
                                       ctypes.c_float(eps), group, 2, _stream()), "k2_norm_mod_quant4")
    return q, s


def fp8_scale(x: torch.Tensor, fmt: int) -> torch.Tensor:
    """The reference's dynamic FP8 input scale (native_runtime.cpp:273-279):
    fp32(bf16(amax|x| / fmax)), at least the smallest normal fp32."""
    fmax = FP8_FORMATS[fmt][2]
    return (x.abs().amax() / fmax).to(torch.float32).clamp_min(torch.finfo(torch.float32).tiny).reshape(1)


def fp8_quant(x: torch.Tensor, fmt: int, scale: torch.Tensor) -> torch.Tensor:
    """k2_fp8 (quantise): x bf16 [m, k] -> fp8 [m, k] = fp8(x / scale[0])."""
    _cuda(x, scale)
    _bf16(x, "fp8_quant")
    _need(fmt in FP8_FORMATS and scale.dtype == torch.float32 and scale.numel() >= 1, "fp8_quant: format / scale")
    dt, code, _ = FP8_FORMATS[fmt]
    q = torch.empty(x.shape, dtype=dt, device=x.device)
    if x.numel():
        lib().k2b_shim_status(1)
        lib().k2_fp8(_p(x), _p(q), _p(scale), x.numel(), 2, code, True, _stream())
        _shim("k2_fp8")
    return q


# ------------------------------------------------------------ projections

def _proj_shapes(a: torch.Tensor, xs: torch.Tensor, w: torch.Tensor, ws: torch.Tensor, packed: bool):
    m = int(a.shape[0])
    k = int(a.shape[1]) * (2 if packed else 1)
    n = int(w.shape[0])
    _need(int(w.shape[1]) * (2 if packed else 1) == k, "projection: activation / weight k mismatch")
    _need(k % 128 == 0 and n % 128 == 0, "projection: k and n must be multiples of 128")
    _need(xs.dtype == torch.float32 and ws.dtype == torch.float32, "projection: fp32 scales expected")
    return m, n, k


def gemm4(a: torch.Tensor, xs: torch.Tensor, w: torch.Tensor, ws: torch.Tensor,
          bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """k2_gemm4: packed a [m, k/2] (xs fp32 [m]) x packed w [n, k/2] (ws fp32
    [n]) -> bf16 [m, n] = T(acc * xs * ws [+ bias fp32])."""
    _cuda(a, xs, w, ws, bias)
    m, n, k = _proj_shapes(a, xs, w, ws, True)
    _need(xs.numel() == m and ws.numel() == n, "gemm4: per-row / per-channel scales expected")
    _need(bias is None or (bias.dtype == torch.float32 and bias.numel() == n), "gemm4: fp32 bias [n]")
    out = torch.empty((m, n), dtype=torch.bfloat16, device=a.device)
    if m:
        lib().k2b_shim_status(1)
        lib().k2_gemm4(_p(a), _p(w), _p(xs), _p(ws), _p(bias), _p(out), m, n, k, 2, _stream())
        _shim("k2_gemm4")
    return out


def gemm8(a: torch.Tensor, xs: torch.Tensor, w: torch.Tensor, ws: torch.Tensor,
          bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """INT8 projection (the reference's _int_mm + k2_dequant8): int8 a [m, k]
    (xs fp32 [m]) x int8 w [n, k] (ws fp32 [n] or [1]) -> bf16 [m, n]."""
    _cuda(a, xs, w, ws, bias)
    _need(a.dtype == torch.int8 and w.dtype == torch.int8, "gemm8: int8 operands expected")
    m, n, k = _proj_shapes(a, xs, w, ws, False)
    _need(xs.numel() == m and ws.numel() in (1, n), "gemm8: scale shapes")
    _need(bias is None or (bias.dtype == torch.float32 and bias.numel() == n), "gemm8: fp32 bias [n]")
    out = torch.empty((m, n), dtype=torch.bfloat16, device=a.device)
    if m:
        check(lib().k2b_gemm8(_p(a), _p(xs), 1, _p(w), _p(ws), 1 if ws.numel() == n else 0, _p(bias), _p(out), m, n,
                              k, _stream()), "k2b_gemm8")
    return out


def gemm_f8(a: torch.Tensor, xs: torch.Tensor, w: torch.Tensor, ws: torch.Tensor,
            bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """FP8 projection (the reference's _scaled_mm): fp8 a [m, k] with one
    scale xs [1] (or per row [m]) x fp8 w [n, k] with ws [1] or [n]."""
    _cuda(a, xs, w, ws, bias)
    fmts = {torch.float8_e4m3fn: 0, torch.float8_e5m2: 1}
    _need(a.dtype in fmts and w.dtype in fmts, "gemm_f8: e4m3 / e5m2 operands expected")
    m, n, k = _proj_shapes(a, xs, w, ws, False)
    _need(xs.numel() in (1, m) and ws.numel() in (1, n), "gemm_f8: scale shapes")
    _need(bias is None or (bias.dtype == torch.float32 and bias.numel() == n), "gemm_f8: fp32 bias [n]")
    out = torch.empty((m, n), dtype=torch.bfloat16, device=a.device)
    if m:
        check(lib().k2b_gemm_f8(_p(a), _p(xs), 1 if xs.numel() == m and m > 1 else 0, _p(w), _p(ws),
                                1 if ws.numel() == n and n > 1 else 0, _p(bias), _p(out), m, n, k, fmts[a.dtype],
                                fmts[w.dtype], _stream()), "k2b_gemm_f8")
    return out


def qkv(a: torch.Tensor, xs: torch.Tensor, w: Sequence[torch.Tensor], s: Sequence[torch.Tensor], nq: torch.Tensor,
        nk: torch.Tensor, freqs: torch.Tensor, *, length: int, eps_q: float = 1e-6, eps_k: float = 1e-6,
        sigmoid_gate: bool = True):
    """Joint Q/K/V(/gate) INT4 projection (k2_int4_qkv over a stream of
    latents of ``length`` tokens): Q and K per-head RMSNorm + RoPE, V plain,
    the gate sigmoided (``sigmoid_gate``) or returned as T(p).  w / s: the
    four (or three) packed weights and their fp32 per-channel scales."""
    _cuda(a, xs, nq, nk, freqs, *w, *s)
    m = int(a.shape[0])
    k = int(a.shape[1]) * 2
    qn, kn = int(w[0].shape[0]), int(w[1].shape[0])
    _need(int(w[2].shape[0]) == kn and (len(w) < 4 or int(w[3].shape[0]) == qn), "qkv: weight widths")
    _need(all(int(t.shape[1]) * 2 == k for t in w) and k % 128 == 0, "qkv: weight k")
    _need(nq.numel() == 128 and nk.numel() == 128 and nq.dtype == torch.float32 and nk.dtype == torch.float32,
          "qkv: fp32 [128] q/k norm weights expected")
    _need(freqs.dtype == torch.float32 and freqs.numel() == length * 64 * 4, "qkv: freqs fp32 [length, 64, 2, 2]")
    _need(length > 0 and m % length == 0, "qkv: rows must be a whole number of latents")
    outs = [torch.empty((m, int(t.shape[0])), dtype=torch.bfloat16, device=a.device) for t in w]
    if m == 0:
        return tuple(outs) + ((None,) if len(w) == 3 else ())
    gate = len(w) == 4 and sigmoid_gate
    check(lib().k2b_ref_qkv(_p(a), _p(xs), _p(w[0]), _p(s[0]), _p(w[1]), _p(s[1]), _p(w[2]), _p(s[2]),
                            _p(w[3] if gate else None), _p(s[3] if gate else None), _p(nq), _p(nk), _p(freqs),
                            _p(outs[0]), _p(outs[1]), _p(outs[2]), _p(outs[3] if gate else None), m, length, qn, kn, k,
                            ctypes.c_float(eps_q), ctypes.c_float(eps_k), _stream()), "k2b_ref_qkv")
    if len(w) == 4 and not sigmoid_gate:
        outs[3] = gemm4(a, xs, w[3], s[3])
    return tuple(outs) + ((None,) if len(w) == 3 else ())


def swiglu(a: torch.Tensor, xs: torch.Tensor, wg: torch.Tensor, sg: torch.Tensor, wu: torch.Tensor,
           su: torch.Tensor) -> torch.Tensor:
    """k2_int4_swiglu: h = T(T(silu(T(p_g))) * T(p_u)), bf16 [m, n]."""
    _cuda(a, xs, wg, sg, wu, su)
    m, n, k = _proj_shapes(a, xs, wg, sg, True)
    _need(tuple(wu.shape) == tuple(wg.shape) and su.numel() == n and sg.numel() == n, "swiglu: gate / up shapes")
    h = torch.empty((m, n), dtype=torch.bfloat16, device=a.device)
    if m:
        check(lib().k2_int4_swiglu(_p(a), _p(wg), _p(wu), _p(xs), _p(sg), _p(su), _p(h), m, n, k, 0, _stream()),
              "k2_int4_swiglu")
    return h


def gated_residual(a: torch.Tensor, xs: torch.Tensor, w: torch.Tensor, ws: torch.Tensor, gate: torch.Tensor,
                   residual: torch.Tensor, *, length: int) -> torch.Tensor:
    """k2_int4_gated_residual over latents of ``length`` rows:
    out = T(resid + T(T(p) * gate[row // length])), gate bf16 [batch, n]."""
    _cuda(a, xs, w, ws, gate, residual)
    m, n, k = _proj_shapes(a, xs, w, ws, True)
    _need(gate.dtype == torch.bfloat16 and residual.dtype == torch.bfloat16, "gated_residual: bf16 gate / residual")
    _need(length > 0 and m % length == 0 and gate.numel() == (m // length) * n and residual.numel() == m * n,
          "gated_residual: gate rows must cover the latents")
    out = torch.empty((m, n), dtype=torch.bfloat16, device=a.device)
    if m:
        check(lib().k2b_ref_gated_residual(_p(a), _p(xs), _p(w), _p(ws), _p(gate), _p(residual), _p(out), m, length,
                                           n, k, _stream()), "k2b_ref_gated_residual")
    return out


def lora_gemm4(a: torch.Tensor, xs: torch.Tensor, w: torch.Tensor, ws: torch.Tensor, t: torch.Tensor,
               up: torch.Tensor, strength: float, bias: Optional[torch.Tensor] = None,
               gate: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None, *,
               length: Optional[int] = None) -> torch.Tensor:
    """k2_gemm4 (or the gated residual) with one LoRA pair in the epilogue:
    p' = T(T(acc * xs * ws [+ bias]) + T(T(t up^T) * s))."""
    from .ops import _lora_args

    _cuda(a, xs, w, ws, t, up, bias, gate, residual)
    m, n, k = _proj_shapes(a, xs, w, ws, True)
    r = _lora_args(t, up, m, n)
    _need((gate is None) == (residual is None) and (bias is None or gate is None), "lora_gemm4: arguments")
    length = m if length is None else length
    out = torch.empty((m, n), dtype=torch.bfloat16, device=a.device)
    if m:
        check(lib().k2b_lora_gemm(1, _p(a), _p(xs), _p(w), _p(ws), _p(bias), _p(gate), _p(residual), length, _p(t),
                                  _p(up), r, ctypes.c_float(strength), _p(out), m, n, k, _stream()), "k2b_lora_gemm")
    return out


# ------------------------------------------- byte-operand forms (INT4 codes)
# A and W as e4m3 code bytes: the same exact integer sums as the packed forms
# above, without their in-CTA unpacking (about 1.6x faster at Krea2 sizes).

def codes_e4m3(packed: torch.Tensor) -> torch.Tensor:
    """Packed INT4 codes (int8 / uint8 [r, k/2]) -> float8_e4m3fn [r, k]
    holding the same codes (k2b_expand_e4m3)."""
    from .ops import expand_e4m3

    return expand_e4m3(packed.view(torch.uint8)).view(torch.float8_e4m3fn)


def quant4_e4m3(x: torch.Tensor, group: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """quant4 with the codes as e4m3 bytes: (float8_e4m3fn [m, k], fp32 [m, 1])
    (k2b_ref_quant4_e4m3; k % 512 == 0)."""
    _cuda(x)
    _bf16(x, "quant4_e4m3")
    _need(group in GROUPS4, f"quant4_e4m3: ConvRot group {group} not in {GROUPS4}")
    m, k = x.shape
    _need(k % 512 == 0, "quant4_e4m3: k must be a multiple of 512")
    q = torch.empty((m, k), dtype=torch.float8_e4m3fn, device=x.device)
    s = torch.empty((m, 1), dtype=torch.float32, device=x.device)
    if m:
        check(lib().k2b_ref_quant4_e4m3(_p(x), _p(q), _p(s), m, k, group, _stream()), "k2b_ref_quant4_e4m3")
    return q, s


def norm_quant4_e4m3(x: torch.Tensor, w: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor, *, length: int,
                     cut: int = -1, eps: float = 1e-6, group: int = 256) -> Tuple[torch.Tensor, torch.Tensor]:
    """norm_quant4 with the codes as e4m3 bytes (k2b_ref_norm_quant4_e4m3)."""
    _cuda(x, w, scale, shift)
    _bf16(x, "norm_quant4_e4m3")
    _need(scale.dtype == torch.bfloat16 and shift.dtype == torch.bfloat16 and w.dtype == torch.float32,
          "norm_quant4_e4m3: fp32 norm weight and bf16 modulation expected")
    _need(group in GROUPS4, f"norm_quant4_e4m3: ConvRot group {group} not in {GROUPS4}")
    rows, K = x.shape
    _need(K % 512 == 0 and w.numel() == K and scale.shape[-1] == K and shift.numel() == scale.numel(),
          "norm_quant4_e4m3: widths")
    batch = max(1, rows // max(1, length))
    _need(scale.numel() // K >= (2 * batch if cut >= 0 else batch), "norm_quant4_e4m3: modulation rows")
    q = torch.empty((rows, K), dtype=torch.float8_e4m3fn, device=x.device)
    s = torch.empty((rows, 1), dtype=torch.float32, device=x.device)
    if rows:
        check(lib().k2b_ref_norm_quant4_e4m3(_p(x), _p(w), _p(scale), _p(shift), _p(q), _p(s), rows, K, length, cut,
                                             batch, ctypes.c_float(eps), group, _stream()), "k2b_ref_norm_quant4_e4m3")
    return q, s


def _codes8(a8: torch.Tensor, w8: Sequence[torch.Tensor], xs: torch.Tensor, ws: Sequence[torch.Tensor]):
    _cuda(a8, xs, *w8, *ws)
    _need(a8.dtype == torch.float8_e4m3fn and all(w.dtype == torch.float8_e4m3fn for w in w8),
          "e4m3 code bytes expected (codes_e4m3)")
    m, k = int(a8.shape[0]), int(a8.shape[1])
    _need(k % 128 == 0 and all(int(w.shape[1]) == k and int(w.shape[0]) % 128 == 0 for w in w8),
          "projection: k and n must be multiples of 128")
    _need(xs.dtype == torch.float32 and xs.numel() == m and
          all(s.dtype == torch.float32 and s.numel() == int(w.shape[0]) for s, w in zip(ws, w8)),
          "per-row / per-channel fp32 scales expected")
    return m, k


def qkv8(a8, xs, w8, s, nq, nk, freqs, *, length: int, eps_q: float = 1e-6, eps_k: float = 1e-6):
    """qkv() with code bytes (k2b_ref_qkv8); the gate (4th weight) sigmoided."""
    m, k = _codes8(a8, w8, xs, s)
    _cuda(nq, nk, freqs)
    qn, kn = int(w8[0].shape[0]), int(w8[1].shape[0])
    _need(int(w8[2].shape[0]) == kn and (len(w8) < 4 or int(w8[3].shape[0]) == qn), "qkv8: weight widths")
    _need(freqs.dtype == torch.float32 and freqs.numel() == length * 256 and length > 0 and m % length == 0,
          "qkv8: freqs fp32 [length, 64, 2, 2], whole latents")
    outs = [torch.empty((m, int(w.shape[0])), dtype=torch.bfloat16, device=a8.device) for w in w8]
    if m:
        g = len(w8) == 4
        check(lib().k2b_ref_qkv8(_p(a8), _p(xs), _p(w8[0]), _p(s[0]), _p(w8[1]), _p(s[1]), _p(w8[2]), _p(s[2]),
                                 _p(w8[3] if g else None), _p(s[3] if g else None), _p(nq), _p(nk), _p(freqs),
                                 _p(outs[0]), _p(outs[1]), _p(outs[2]), _p(outs[3] if g else None), m, length, qn, kn,
                                 k, ctypes.c_float(eps_q), ctypes.c_float(eps_k), _stream()), "k2b_ref_qkv8")
    return tuple(outs) + ((None,) if len(w8) == 3 else ())


def swiglu8(a8, xs, wg8, sg, wu8, su) -> torch.Tensor:
    """swiglu() with code bytes (k2b_ref_swiglu8)."""
    m, k = _codes8(a8, [wg8, wu8], xs, [sg, su])
    n = int(wg8.shape[0])
    _need(tuple(wu8.shape) == tuple(wg8.shape), "swiglu8: gate / up shapes")
    h = torch.empty((m, n), dtype=torch.bfloat16, device=a8.device)
    if m:
        check(lib().k2b_ref_swiglu8(_p(a8), _p(wg8), _p(wu8), _p(xs), _p(sg), _p(su), _p(h), m, n, k, _stream()),
              "k2b_ref_swiglu8")
    return h


def gated_residual8(a8, xs, w8, ws, gate, residual, *, length: int) -> torch.Tensor:
    """gated_residual() with code bytes (k2b_ref_gated_residual8)."""
    m, k = _codes8(a8, [w8], xs, [ws])
    n = int(w8.shape[0])
    _cuda(gate, residual)
    _need(gate.dtype == torch.bfloat16 and residual.dtype == torch.bfloat16 and length > 0 and m % length == 0 and
          gate.numel() == (m // length) * n and residual.numel() == m * n, "gated_residual8: shapes")
    out = torch.empty((m, n), dtype=torch.bfloat16, device=a8.device)
    if m:
        check(lib().k2b_ref_gated_residual8(_p(a8), _p(xs), _p(w8), _p(ws), _p(gate), _p(residual), _p(out), m, length,
                                            n, k, _stream()), "k2b_ref_gated_residual8")
    return out
