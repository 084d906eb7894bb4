"""Torch-level wrappers over the libk2b C ABI.

Each op validates devices, dtypes, shapes and contiguity the way the reference's
C++ side does before it dlsym-calls a kernel (TORCH_CHECK-style errors,
native_runtime.cpp:262-271, 399-423), allocates outputs with torch.empty
(the kernels never allocate), launches on torch's current CUDA stream, and
raises ``K2BError`` on a non-zero status.  Nothing here computes on the CPU.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional, Tuple

import torch

from ._native import K2BError, check, lib

GROUP = 128
HEAD_DIM = 128


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _p(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def _cuda(*ts: Optional[torch.Tensor]) -> None:
    dev = None
    for t in ts:
        if t is None:
            continue
        _need(t.is_cuda, "k2b ops need CUDA tensors")
        _need(t.is_contiguous(), "k2b ops need contiguous tensors")
        dev = t.device if dev is None else dev
        _need(t.device == dev, "k2b op inputs must share one device")


# ------------------------------------------------------------------ weights

@dataclass
class PreparedWeight:
    """Device-resident INT4 weight in the GEMM's streaming layout."""

    w: torch.Tensor      # uint8 [n, k]: the INT4 codes as e4m3 bytes, column order
    scale: torch.Tensor  # fp32 [k/128, n]

    @property
    def n(self) -> int:
        return int(self.w.shape[0])

    @property
    def k(self) -> int:
        return int(self.w.shape[1])


def prepare_weight(packed: torch.Tensor, scales: torch.Tensor) -> PreparedWeight:
    """Packed INT4 [n, k/2] (uint8) + fp16 group scales [n, k/128] ->
    PreparedWeight.  Registration-time step (weights stay resident)."""
    _cuda(packed, scales)
    _need(packed.dtype == torch.uint8 and scales.dtype == torch.float16, "packed u8 + fp16 scales expected")
    n, k2 = packed.shape
    k = 2 * k2
    _need(k % GROUP == 0 and tuple(scales.shape) == (n, k // GROUP), "weight scale shape mismatch")
    w = torch.empty((n, k), dtype=torch.uint8, device=packed.device)
    s = torch.empty((k // GROUP, n), dtype=torch.float32, device=packed.device)
    check(lib().k2b_prepare_weight(_p(packed), _p(scales), _p(w), _p(s), n, k, n, n, 0, n, _stream()),
          "k2b_prepare_weight")
    return PreparedWeight(w, s)


# --------------------------------------------------------------- norm_quant

def norm_quant(x: torch.Tensor, w: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor, *,
               length: Optional[int] = None, cut: int = -1, eps: float = 1e-6
               ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Fused RMSNorm + adaLN + H128 + group-128 INT4 (k2_native::norm_quant).

    x bf16 [..., K] (rows = prod of leading dims; ``length`` rows per latent,
    default = x.shape[-2] for 3-D x else all rows); w fp32 [K] in the "w+1"
    form; scale/shift bf16 [nb, K] (any shape ending in K).
    Returns (q uint8 [rows, K/2], s fp16 [rows, K/128])."""
    _cuda(x, w, scale, shift)
    _need(x.dtype == torch.bfloat16 and scale.dtype == torch.bfloat16 and shift.dtype == torch.bfloat16,
          "norm_quant: bf16 activations and modulation expected")
    _need(w.dtype == torch.float32, "norm_quant: fp32 norm weight expected")
    K = int(x.shape[-1])
    rows = x.numel() // K
    if length is None:
        length = (int(x.shape[-2]) if x.dim() == 3 else rows) or 1
    batch = max(1, rows // length)
    _need(w.numel() == K and scale.shape[-1] == K and shift.shape[-1] == K, "norm_quant: width mismatch")
    nb = scale.numel() // K
    _need(nb >= (2 * batch if cut >= 0 else batch) and shift.numel() == scale.numel(),
          "norm_quant: modulation rows do not cover the batch")
    q = torch.empty((rows, K // 2), dtype=torch.uint8, device=x.device)
    s = torch.empty((rows, K // GROUP), dtype=torch.float16, device=x.device)
    if rows == 0:  # empty batch: empty outputs, no launch
        return q, s
    check(lib().k2b_norm_quant(_p(x), _p(w), _p(scale), _p(shift), _p(q), _p(s), rows, K, length, cut, batch,
                               ctypes.c_float(eps), _stream()), "k2b_norm_quant")
    return q, s


def norm_quant_rows(x: torch.Tensor, w: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor, *,
                    base_row: int, length: int, batch: int, cut: int = -1, eps: float = 1e-6,
                    out: Optional[Tuple[torch.Tensor, torch.Tensor]] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """norm_quant of rows [base_row, base_row + rows) of a stream of ``batch``
    latents of ``length`` rows: x bf16 [rows, K] holds just those rows, and the
    modulation row of each follows its index in the whole stream.  ``out``
    (q, s) may name views to write into (e.g. this rank's slot of an
    all-gather buffer)."""
    _cuda(x, w, scale, shift)
    _need(x.dtype == torch.bfloat16 and scale.dtype == torch.bfloat16 and shift.dtype == torch.bfloat16 and
          w.dtype == torch.float32, "norm_quant_rows: bf16 x/modulation, fp32 w expected")
    K = int(x.shape[-1])
    rows = x.numel() // K
    _need(base_row >= 0 and base_row + rows <= batch * length, "norm_quant_rows: rows outside the stream")
    _need(w.numel() == K and scale.shape[-1] == K and shift.numel() == scale.numel() and
          scale.numel() // K >= (2 * batch if cut >= 0 else batch), "norm_quant_rows: modulation shape")
    if out is None:
        q = torch.empty((rows, K // 2), dtype=torch.uint8, device=x.device)
        s = torch.empty((rows, K // GROUP), dtype=torch.float16, device=x.device)
    else:
        q, s = out
        _cuda(q, s)
        _need(q.dtype == torch.uint8 and s.dtype == torch.float16 and q.numel() == rows * K // 2 and
              s.numel() == rows * K // GROUP, "norm_quant_rows: output shapes")
    if rows:
        check(lib().k2b_norm_quant_rows(_p(x), _p(w), _p(scale), _p(shift), _p(q), _p(s), base_row, rows, K, length,
                                        cut, batch, ctypes.c_float(eps), _stream()), "k2b_norm_quant_rows")
    return q, s


def gated_add(p: torch.Tensor, gate: torch.Tensor, residual: torch.Tensor, *, base_row: int, length: int,
              out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out = bf16(residual + bf16(bf16(p) * gate[(base_row + row) // length]))
    for a reduced fp32 projection p [rows, n] (k2b_gated_add)."""
    _cuda(p, gate, residual, out)
    _need(p.dtype == torch.float32 and gate.dtype == torch.bfloat16 and residual.dtype == torch.bfloat16,
          "gated_add: fp32 p, bf16 gate/residual expected")
    n = int(p.shape[-1])
    rows = p.numel() // n
    _need(residual.numel() == rows * n and gate.shape[-1] == n, "gated_add: shapes")
    _need(rows == 0 or (base_row + rows - 1) // length < gate.numel() // n, "gated_add: gate rows do not cover")
    if out is None:
        out = torch.empty((rows, n), dtype=torch.bfloat16, device=p.device)
    _need(out.dtype == torch.bfloat16 and out.numel() == rows * n, "gated_add: out shape")
    check(lib().k2b_gated_add(_p(p), _p(gate), _p(residual), _p(out), base_row, rows, n, length, _stream()),
          "k2b_gated_add")
    return out


def reduce_gated_add(slots_ptr: int, nslots: int, slot_stride: int, gate: torch.Tensor, residual: torch.Tensor, *,
                     base_row: int, length: int, out: torch.Tensor) -> torch.Tensor:
    """out = gated_add of p = ((s_0 + s_1) + ...) over ``nslots`` fp32 slots
    of a receive buffer (``slots_ptr``: this rank's first row in slot 0,
    ``slot_stride`` floats between slots), k2b_reduce_gated_add."""
    _cuda(gate, residual, out)
    _need(gate.dtype == torch.bfloat16 and residual.dtype == torch.bfloat16 and out.dtype == torch.bfloat16,
          "reduce_gated_add: bf16 gate/residual/out expected")
    n = int(residual.shape[-1])
    rows = residual.numel() // n
    _need(out.numel() == rows * n and gate.shape[-1] == n and 1 <= nslots <= 8, "reduce_gated_add: shapes")
    check(lib().k2b_reduce_gated_add(ctypes.c_void_p(slots_ptr), nslots, slot_stride, _p(gate), _p(residual), _p(out),
                                     base_row, rows, n, length, _stream()), "k2b_reduce_gated_add")
    return out


def norm_mod(x: torch.Tensor, w: torch.Tensor, scale: Optional[torch.Tensor] = None,
             shift: Optional[torch.Tensor] = None, *, length: Optional[int] = None, cut: int = -1,
             eps: float = 1e-6) -> torch.Tensor:
    """bf16 RMSNorm (+ adaLN when scale/shift are given), the rounding points
    of norm_quant without the quantisation (k2_native::norm_mod, k2_norm).
    Returns bf16 shaped like x."""
    _cuda(x, w, scale, shift)
    _need((scale is None) == (shift is None), "norm_mod: scale and shift go together")
    _need(x.dtype == torch.bfloat16 and w.dtype == torch.float32, "norm_mod: bf16 x, fp32 w expected")
    K = int(x.shape[-1])
    rows = x.numel() // K
    _need(w.numel() == K, "norm_mod: width mismatch")
    if length is None:
        length = (int(x.shape[-2]) if x.dim() == 3 else rows) or 1
    batch = max(1, rows // length)
    if scale is not None:
        _need(scale.dtype == torch.bfloat16 and shift.dtype == torch.bfloat16 and scale.shape[-1] == K and
              shift.numel() == scale.numel(), "norm_mod: bf16 modulation [nb, K] expected")
        _need(scale.numel() // K >= (2 * batch if cut >= 0 else batch), "norm_mod: modulation rows do not cover the batch")
    y = torch.empty_like(x)
    if rows == 0:
        return y
    check(lib().k2b_norm_mod(_p(x), _p(w), _p(scale), _p(shift), _p(y), rows, K, length, cut, batch,
                             ctypes.c_float(eps), _stream()), "k2b_norm_mod")
    return y


def elementwise(a: torch.Tensor, b: Optional[torch.Tensor], r: Optional[torch.Tensor], mode: int,
                width: int = 0) -> torch.Tensor:
    """k2_elementwise (kernels/native_dispatch.cu:63-70): mode 0 silu(a)[*b],
    1 sigmoid(a)[*b], 2 r + b*a[i % width] (bf16, each step rounded)."""
    _cuda(a, b, r)
    for t in (a, b, r):
        _need(t is None or t.dtype == torch.bfloat16, "elementwise: bf16 expected")
    out_like = r if mode == 2 else a
    _need(out_like is not None, "elementwise: mode 2 needs a residual")
    y = torch.empty_like(out_like)
    check(lib().k2b_elementwise(_p(a), _p(b), _p(r), _p(y), y.numel(), mode, width, _stream()), "k2b_elementwise")
    return y


def rope(q: torch.Tensor, k: torch.Tensor, freqs: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """k2_native::rope (native_runtime.cpp:312-317): q [B,Hq,L,D], k [B,Hk,L,D]
    bf16, freqs fp32 [fb, ..., L, D/2, 2, 2] with fb = 1 or B."""
    _cuda(q, k, freqs)
    _need(q.dtype == torch.bfloat16 and k.dtype == torch.bfloat16 and freqs.dtype == torch.float32, "rope: dtypes")
    B, Hq, L, D = q.shape
    _need(k.shape[0] == B and k.shape[2] == L and k.shape[3] == D, "rope: q/k shapes")
    per = L * (D // 2) * 4
    _need(freqs.numel() % per == 0 and freqs.numel() // per in (1, B), "rope: freqs shape")
    qo, ko = torch.empty_like(q), torch.empty_like(k)
    check(lib().k2b_rope(_p(q), _p(k), _p(freqs), _p(qo), _p(ko), B, L, Hq, int(k.shape[1]), D,
                         freqs.numel() // per, _stream()), "k2b_rope")
    return qo, ko


def rotate_quant(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """bf16 [..., K] -> (uint8 [rows, K/2], fp16 [rows, K/128])."""
    _cuda(x)
    _need(x.dtype == torch.bfloat16, "rotate_quant: bf16 expected")
    K = int(x.shape[-1])
    rows = x.numel() // K
    q = torch.empty((rows, K // 2), dtype=torch.uint8, device=x.device)
    s = torch.empty((rows, K // GROUP), dtype=torch.float16, device=x.device)
    if rows == 0:
        return q, s
    check(lib().k2b_rotate_quant(_p(x), _p(q), _p(s), rows, K, _stream()), "k2b_rotate_quant")
    return q, s


# --------------------------------------------------------------------- GEMM

def expand_e4m3(a: torch.Tensor) -> torch.Tensor:
    """Packed INT4 codes uint8 [m, k/2] -> e4m3 bytes uint8 [m, k] (k2b_expand_e4m3)."""
    _cuda(a)
    _need(a.dtype == torch.uint8 and a.dim() == 2 and a.numel() % 16 == 0, "expand_e4m3: packed uint8 [m, k/2]")
    a8 = torch.empty((a.shape[0], 2 * a.shape[1]), dtype=torch.uint8, device=a.device)
    if a.numel():
        check(lib().k2b_expand_e4m3(_p(a), _p(a8), a.numel(), _stream()), "k2b_expand_e4m3")
    return a8


def _a8(a: torch.Tensor, sa: torch.Tensor, k: int):
    """The GEMM's A operand as e4m3 bytes [m, k]: packed codes [m, k/2] are
    expanded first (one pass over 1.5 bytes per code), byte containers are
    used as they are.  The byte-A GEMM takes about 40% less time than the
    in-CTA unpack of packed A."""
    _need(a.dtype == torch.uint8 and sa.dtype == torch.float16 and a.dim() == 2,
          "uint8 activations (packed or e4m3 bytes) + fp16 scales expected")
    m = int(a.shape[0])
    _need(tuple(sa.shape) == (m, k // GROUP) and a.shape[1] in (k // 2, k), "activation / weight K mismatch")
    return (expand_e4m3(a) if a.shape[1] * 2 == k else a), m


def gemm_f32(a: torch.Tensor, sa: torch.Tensor, W: PreparedWeight, out: Optional[torch.Tensor] = None
             ) -> torch.Tensor:
    """fp32 a@W (exact group accumulation); ``out`` may be a preallocated
    [m, n] fp32 buffer (e.g. the first rows of a reduce-scatter input)."""
    _cuda(a, sa, W.w, W.scale, out)
    a8, m = _a8(a, sa, W.k)
    if out is None:
        out = torch.empty((m, W.n), dtype=torch.float32, device=a.device)
    _need(out.dtype == torch.float32 and out.dim() == 2 and tuple(out.shape) == (m, W.n), "gemm_f32: out shape")
    if m == 0:
        return out
    check(lib().k2b_gemm_f32_e4m3(_p(a8), _p(sa), _p(W.w), _p(W.scale), _p(out), m, W.n, W.k, _stream()),
          "k2b_gemm_f32_e4m3")
    return out


def gemm_f32_scatter(a: torch.Tensor, sa: torch.Tensor, W: PreparedWeight, peers, rank: int, chunk: int) -> None:
    """fp32 a@W written into the owners' receive buffers (k2b_gemm_f32_scatter):
    row r to ``peers[r // chunk]`` (device pointers, fp32 [tp, chunk, n] each)
    in slot ``rank``."""
    _cuda(a, sa, W.w, W.scale)
    a8, m = _a8(a, sa, W.k)
    tp = len(peers)
    _need(1 <= tp <= 4 and 0 <= rank < tp and chunk > 0 and chunk * tp >= m, "gemm_f32_scatter: rank layout")
    arr = (ctypes.c_void_p * tp)(*[int(x) for x in peers])
    check(lib().k2b_gemm_f32_scatter_e4m3(_p(a8), _p(sa), _p(W.w), _p(W.scale), arr, tp, rank, chunk, m, W.n, W.k,
                                          _stream()), "k2b_gemm_f32_scatter_e4m3")


def gemm_bf16(a: torch.Tensor, sa: torch.Tensor, W: PreparedWeight) -> torch.Tensor:
    _cuda(a, sa, W.w, W.scale)
    a8, m = _a8(a, sa, W.k)
    out = torch.empty((m, W.n), dtype=torch.bfloat16, device=a.device)
    if m == 0:
        return out
    check(lib().k2b_gemm_bf16_e4m3(_p(a8), _p(sa), _p(W.w), _p(W.scale), _p(out), m, W.n, W.k, _stream()),
          "k2b_gemm_bf16_e4m3")
    return out


def qkv(a: torch.Tensor, sa: torch.Tensor, wq: PreparedWeight, wk: PreparedWeight, wv: PreparedWeight,
        nq: torch.Tensor, nk: torch.Tensor, freqs: torch.Tensor, *, length: int, eps_q: float = 1e-6,
        eps_k: float = 1e-6, wg: Optional[PreparedWeight] = None):
    """Fused Q/K/V(/gate) projection with QK RMSNorm + RoPE (k2_native::qkv_prepared).

    Returns token-major bf16 (q [m, Hq*128], k [m, Hkv*128], v [m, Hkv*128],
    gate [m, Hq*128] or None)."""
    _cuda(a, sa, wq.w, wk.w, wv.w, nq, nk, freqs, None if wg is None else wg.w)
    a8, m = _a8(a, sa, wq.k)
    _need(wk.k == wq.k and wv.k == wq.k and wk.n == wv.n, "qkv weight shapes")
    _need(nq.dtype == torch.float32 and nk.dtype == torch.float32 and nq.numel() == HEAD_DIM and
          nk.numel() == HEAD_DIM, "qkv: fp32 [128] q/k norm weights expected")
    _need(freqs.dtype == torch.float32 and freqs.numel() == length * 64 * 4, "qkv: freqs fp32 [length,64,2,2]")
    _need(m % length == 0, "qkv: rows must be a whole number of latents")
    qo = torch.empty((m, wq.n), dtype=torch.bfloat16, device=a.device)
    ko = torch.empty((m, wk.n), dtype=torch.bfloat16, device=a.device)
    vo = torch.empty((m, wv.n), dtype=torch.bfloat16, device=a.device)
    go = None
    if wg is not None:
        _need(wg.n == wq.n and wg.k == wq.k, "qkv gate weight shape")
        go = torch.empty((m, wg.n), dtype=torch.bfloat16, device=a.device)
    if m == 0:
        return qo, ko, vo, go
    check(lib().k2b_qkv_e4m3(_p(a8), _p(sa), _p(wq.w), _p(wq.scale), _p(wk.w), _p(wk.scale), _p(wv.w),
                             _p(wv.scale), _p(None if wg is None else wg.w), _p(None if wg is None else wg.scale),
                             _p(nq), _p(nk), _p(freqs), _p(qo), _p(ko), _p(vo), _p(go), m, length, wq.n, wk.n, wq.k,
                             ctypes.c_float(eps_q), ctypes.c_float(eps_k), _stream()), "k2b_qkv_e4m3")
    return qo, ko, vo, go


def gated_residual(a: torch.Tensor, sa: torch.Tensor, W: PreparedWeight, gate: torch.Tensor,
                   residual: torch.Tensor, *, length: int) -> torch.Tensor:
    """out = bf16(residual + bf16(bf16(a@W) * gate[row // length]))."""
    _cuda(a, sa, W.w, gate, residual)
    a8, m = _a8(a, sa, W.k)
    _need(gate.dtype == torch.bfloat16 and residual.dtype == torch.bfloat16, "gated_residual: bf16 expected")
    _need(residual.numel() == m * W.n and gate.numel() == (m // length) * W.n and m % length == 0,
          "gated_residual: shapes")
    out = torch.empty((m, W.n), dtype=torch.bfloat16, device=a.device)
    if m == 0:
        return out
    check(lib().k2b_gated_residual_e4m3(_p(a8), _p(sa), _p(W.w), _p(W.scale), _p(gate), _p(residual), _p(out), m,
                                        length, W.n, W.k, _stream()), "k2b_gated_residual_e4m3")
    return out


def swiglu_quant(a: torch.Tensor, sa: torch.Tensor, wg: PreparedWeight, wu: PreparedWeight):
    """Gate/up + SwiGLU + H128 + INT4 -> (hq uint8 [m, F/2], hs fp16 [m, F/128])."""
    _cuda(a, sa, wg.w, wu.w)
    a8, m = _a8(a, sa, wg.k)
    _need(wu.n == wg.n and wu.k == wg.k, "swiglu weight shapes")
    F = wg.n
    hq = torch.empty((m, F // 2), dtype=torch.uint8, device=a.device)
    hs = torch.empty((m, F // GROUP), dtype=torch.float16, device=a.device)
    if m == 0:
        return hq, hs
    check(lib().k2b_swiglu_quant_a8(_p(a8), _p(sa), _p(wg.w), _p(wg.scale), _p(wu.w), _p(wu.scale), _p(hq), _p(hs),
                                    m, F, wg.k, _stream()), "k2b_swiglu_quant_a8")
    return hq, hs


def swiglu_bf16(a: torch.Tensor, sa: torch.Tensor, wg: PreparedWeight, wu: PreparedWeight) -> torch.Tensor:
    _cuda(a, sa, wg.w, wu.w)
    a8, m = _a8(a, sa, wg.k)
    _need(wu.n == wg.n and wu.k == wg.k, "swiglu weight shapes")
    h = torch.empty((m, wg.n), dtype=torch.bfloat16, device=a.device)
    if m == 0:
        return h
    check(lib().k2b_swiglu_bf16_e4m3(_p(a8), _p(sa), _p(wg.w), _p(wg.scale), _p(wu.w), _p(wu.scale), _p(h), m, wg.n,
                                     wg.k, _stream()), "k2b_swiglu_bf16_e4m3")
    return h


# ---------------------------------------------------------------- attention

def _bhld(t: torch.Tensor, name: str):
    _need(t.is_cuda and t.dtype == torch.bfloat16 and t.dim() == 4, f"{name}: bf16 [B,H,L,D] CUDA tensor expected")
    _need(t.shape[-1] == HEAD_DIM and t.stride(-1) == 1, f"{name}: head dim 128, contiguous last dim")
    return int(t.stride(0)), int(t.stride(1)), int(t.stride(2))


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: Optional[torch.Tensor] = None,
              gate: Optional[torch.Tensor] = None, gate_is_sigmoid: bool = True) -> torch.Tensor:
    """GQA flash attention with the Kohaku FA contract
    (KohakuKernelRouter/attention.py:146-193): q [B,Hq,L,D], k/v [B,Hkv,Lk,D]
    (any strides with a contiguous last dim) -> out [B, L, Hq*D]."""
    _need(mask is None, "k2b attention: attention masks are not supported on the B200 path")
    qs, ks, vs = _bhld(q, "q"), _bhld(k, "k"), _bhld(v, "v")
    B, H, L, D = q.shape
    _need(k.shape[0] == B and k.shape[:3] == v.shape[:3] and H % k.shape[1] == 0, "attention: GQA shapes")
    _need(q.device == k.device == v.device, "attention: one device")
    out = torch.empty((B, L, H * D), dtype=q.dtype, device=q.device)
    if L == 0:
        return out
    gate_kind = 0
    if gate is not None:
        _need(tuple(gate.shape) == tuple(out.shape) and gate.dtype == q.dtype and gate.device == q.device,
              "attention: gate must match the output")
        gate = gate.contiguous()
        gate_kind = 2 if gate_is_sigmoid else 1
    check(lib().k2b_attention(_p(q), _p(k), _p(v), _p(gate), _p(out), B, H, int(k.shape[1]), L, int(k.shape[2]), D,
                              *qs, *ks, *vs, gate_kind, _stream()), "k2b_attention")
    return out


def attention_quant(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
    """Attention whose output is stored H128-rotated and INT4-quantised:
    (oq uint8 [B*L, Hq*64], os fp16 [B*L, Hq])."""
    qs, ks, vs = _bhld(q, "q"), _bhld(k, "k"), _bhld(v, "v")
    B, H, L, D = q.shape
    _need(k.shape[0] == B and k.shape[:3] == v.shape[:3] and H % k.shape[1] == 0, "attention: GQA shapes")
    oq = torch.empty((B * L, H * D // 2), dtype=torch.uint8, device=q.device)
    os_ = torch.empty((B * L, H), dtype=torch.float16, device=q.device)
    if B * L == 0:
        return oq, os_
    check(lib().k2b_attention_quant(_p(q), _p(k), _p(v), _p(oq), _p(os_), B, H, int(k.shape[1]), L,
                                    int(k.shape[2]), D, *qs, *ks, *vs, _stream()), "k2b_attention_quant")
    return oq, os_


# ------------------------------------------------------------ LoRA deltas

def _lora_args(t: torch.Tensor, up: torch.Tensor, m: int, n: int):
    _need(t.dtype == torch.bfloat16 and up.dtype == torch.bfloat16, "lora: bf16 factors expected")
    r = int(t.shape[-1])
    _need(tuple(t.shape) == (m, r) and tuple(up.shape) == (n, r) and r % 8 == 0 and 0 < r <= 1024,
          "lora: t [m, r], up [n, r] with r a multiple of 8 (<= 1024)")
    return r


def lora_gemm(a: torch.Tensor, sa: torch.Tensor, W: PreparedWeight, t: torch.Tensor, up: torch.Tensor,
              strength: float, gate: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None, *,
              length: Optional[int] = None) -> torch.Tensor:
    """Group-128 W4A4 projection with one LoRA pair in its epilogue:
    p' = T(T(p) + T(T(t up^T) * s)), t = T(x down^T) bf16 [m, r]; returns p'
    (bf16 [m, n]) or, with gate [batch, n] and residual [m, n],
    T(residual + T(p' * gate[row // length]))."""
    _cuda(a, sa, W.w, W.scale, t, up, gate, residual)
    a8, m = _a8(a, sa, W.k)
    r = _lora_args(t, up, m, W.n)
    _need((gate is None) == (residual is None), "lora_gemm: gate and residual go together")
    length = m if length is None else length
    out = torch.empty((m, W.n), dtype=torch.bfloat16, device=a.device)
    if m == 0:
        return out
    check(lib().k2b_lora_gemm(2, _p(a8), _p(sa), _p(W.w), _p(W.scale), None, _p(gate), _p(residual), length, _p(t),
                              _p(up), r, ctypes.c_float(strength), _p(out), m, W.n, W.k, _stream()), "k2b_lora_gemm")
    return out


def lora_swiglu(a: torch.Tensor, sa: torch.Tensor, wg: PreparedWeight, wu: PreparedWeight, lora_g=None,
                lora_u=None) -> torch.Tensor:
    """SwiGLU h = T(T(silu(g')) * u') with a LoRA pair (t, up, s) on either
    projection (g', u' as in lora_gemm); bf16 h [m, width]."""
    _cuda(a, sa, wg.w, wu.w)
    a8, m = _a8(a, sa, wg.k)
    args = []
    for lo in (lora_g, lora_u):
        if lo is None:
            args += [None, None, 0, ctypes.c_float(0.0)]
        else:
            t, up, st = lo
            _cuda(t, up)
            args += [_p(t), _p(up), _lora_args(t, up, m, wg.n), ctypes.c_float(st)]
    h = torch.empty((m, wg.n), dtype=torch.bfloat16, device=a.device)
    if m == 0:
        return h
    check(lib().k2b_lora_swiglu(2, _p(a8), _p(sa), _p(wg.w), _p(wg.scale), _p(wu.w), _p(wu.scale), *args, _p(h), m,
                                wg.n, wg.k, _stream()), "k2b_lora_swiglu")
    return h


# ------------------------------------------------------- e4m3 byte containers
# The block loop keeps INT4 codes between its kernels as e4m3 bytes [rows, K]
# (one byte per code, column order): its GEMMs then load A with TMA straight
# into the tensor-core layout.  These are the per-op forms of that path.

def norm_quant_e4m3(x: torch.Tensor, w: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor, *,
                    length: Optional[int] = None, cut: int = -1, eps: float = 1e-6
                    ) -> Tuple[torch.Tensor, torch.Tensor]:
    """norm_quant with the codes as e4m3 bytes: (q8 uint8 [rows, K], s fp16 [rows, K/128])."""
    _cuda(x, w, scale, shift)
    _need(x.dtype == torch.bfloat16 and scale.dtype == torch.bfloat16 and shift.dtype == torch.bfloat16 and
          w.dtype == torch.float32, "norm_quant_e4m3: bf16 x/modulation, fp32 w expected")
    K = int(x.shape[-1])
    rows = x.numel() // K
    if length is None:
        length = (int(x.shape[-2]) if x.dim() == 3 else rows) or 1
    batch = max(1, rows // length)
    _need(w.numel() == K and scale.shape[-1] == K and shift.numel() == scale.numel() and
          scale.numel() // K >= (2 * batch if cut >= 0 else batch), "norm_quant_e4m3: modulation shape")
    q = torch.empty((rows, K), dtype=torch.uint8, device=x.device)
    s = torch.empty((rows, K // GROUP), dtype=torch.float16, device=x.device)
    if rows:
        check(lib().k2b_norm_quant_e4m3(_p(x), _p(w), _p(scale), _p(shift), _p(q), _p(s), rows, K, length, cut,
                                        batch, ctypes.c_float(eps), _stream()), "k2b_norm_quant_e4m3")
    return q, s


def _act8(a: torch.Tensor, sa: torch.Tensor, k: int) -> int:
    _need(a.dtype == torch.uint8 and sa.dtype == torch.float16, "e4m3 byte activations + fp16 scales expected")
    _need(a.dim() == 2 and a.shape[1] == k and tuple(sa.shape) == (a.shape[0], k // GROUP),
          "activation / weight K mismatch")
    return int(a.shape[0])


def gemm_f32_e4m3(a8: torch.Tensor, sa: torch.Tensor, W: PreparedWeight) -> torch.Tensor:
    """fp32 a@W with A as e4m3 bytes (exact group accumulation)."""
    _cuda(a8, sa, W.w, W.scale)
    m = _act8(a8, sa, W.k)
    out = torch.empty((m, W.n), dtype=torch.float32, device=a8.device)
    if m:
        check(lib().k2b_gemm_f32_e4m3(_p(a8), _p(sa), _p(W.w), _p(W.scale), _p(out), m, W.n, W.k, _stream()),
              "k2b_gemm_f32_e4m3")
    return out


def qkv_e4m3(a8, sa, wq: PreparedWeight, wk: PreparedWeight, wv: PreparedWeight, nq, nk, freqs, *, length: int,
             eps_q: float = 1e-6, eps_k: float = 1e-6, wg: Optional[PreparedWeight] = None):
    """qkv with A as e4m3 bytes."""
    _cuda(a8, sa, wq.w, wk.w, wv.w, nq, nk, freqs, None if wg is None else wg.w)
    m = _act8(a8, sa, wq.k)
    _need(wk.k == wq.k and wv.k == wq.k and wk.n == wv.n and m % length == 0, "qkv_e4m3: shapes")
    _need(freqs.dtype == torch.float32 and freqs.numel() == length * 64 * 4, "qkv_e4m3: freqs fp32 [length,64,2,2]")
    qo = torch.empty((m, wq.n), dtype=torch.bfloat16, device=a8.device)
    ko = torch.empty((m, wk.n), dtype=torch.bfloat16, device=a8.device)
    vo = torch.empty((m, wv.n), dtype=torch.bfloat16, device=a8.device)
    go = None if wg is None else torch.empty((m, wg.n), dtype=torch.bfloat16, device=a8.device)
    if m:
        check(lib().k2b_qkv_e4m3(_p(a8), _p(sa), _p(wq.w), _p(wq.scale), _p(wk.w), _p(wk.scale), _p(wv.w),
                                 _p(wv.scale), _p(None if wg is None else wg.w),
                                 _p(None if wg is None else wg.scale), _p(nq), _p(nk), _p(freqs), _p(qo), _p(ko),
                                 _p(vo), _p(go), m, length, wq.n, wk.n, wq.k, ctypes.c_float(eps_q),
                                 ctypes.c_float(eps_k), _stream()), "k2b_qkv_e4m3")
    return qo, ko, vo, go


def gated_residual_e4m3(a8, sa, W: PreparedWeight, gate: torch.Tensor, residual: torch.Tensor, *,
                        length: int) -> torch.Tensor:
    """gated_residual with A as e4m3 bytes."""
    _cuda(a8, sa, W.w, gate, residual)
    m = _act8(a8, sa, W.k)
    _need(residual.numel() == m * W.n and gate.numel() == (m // length) * W.n and m % length == 0,
          "gated_residual_e4m3: shapes")
    out = torch.empty((m, W.n), dtype=torch.bfloat16, device=a8.device)
    if m:
        check(lib().k2b_gated_residual_e4m3(_p(a8), _p(sa), _p(W.w), _p(W.scale), _p(gate), _p(residual), _p(out),
                                            m, length, W.n, W.k, _stream()), "k2b_gated_residual_e4m3")
    return out


def swiglu_quant_e4m3(a8, sa, wg: PreparedWeight, wu: PreparedWeight):
    """Gate/up + SwiGLU + H128 + INT4 with A and h as e4m3 bytes:
    (h8 uint8 [m, F], hs fp16 [m, F/128])."""
    _cuda(a8, sa, wg.w, wu.w)
    m = _act8(a8, sa, wg.k)
    _need(wu.n == wg.n and wu.k == wg.k, "swiglu weight shapes")
    F = wg.n
    h8 = torch.empty((m, F), dtype=torch.uint8, device=a8.device)
    hs = torch.empty((m, F // GROUP), dtype=torch.float16, device=a8.device)
    if m:
        check(lib().k2b_swiglu_quant_e4m3(_p(a8), _p(sa), _p(wg.w), _p(wg.scale), _p(wu.w), _p(wu.scale), _p(h8),
                                          _p(hs), m, F, wg.k, _stream()), "k2b_swiglu_quant_e4m3")
    return h8, hs


def attention_quant_e4m3(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
    """attention_quant with the codes as e4m3 bytes: (oq8 uint8 [B*L, Hq*128], os fp16 [B*L, Hq])."""
    qs, ks, vs = _bhld(q, "q"), _bhld(k, "k"), _bhld(v, "v")
    B, H, L, D = q.shape
    _need(k.shape[0] == B and k.shape[:3] == v.shape[:3] and H % k.shape[1] == 0, "attention: GQA shapes")
    oq = torch.empty((B * L, H * D), dtype=torch.uint8, device=q.device)
    os_ = torch.empty((B * L, H), dtype=torch.float16, device=q.device)
    if B * L:
        check(lib().k2b_attention_quant_e4m3(_p(q), _p(k), _p(v), _p(oq), _p(os_), B, H, int(k.shape[1]), L,
                                             int(k.shape[2]), D, *qs, *ks, *vs, _stream()),
              "k2b_attention_quant_e4m3")
    return oq, os_


def device_error(reset: bool = True) -> int:
    return int(lib().k2b_device_error(1 if reset else 0, _stream()))


def selftest_wait(mode: int, limit_ns: int, device=None) -> list:
    """Runs the library's bounded-wait self-test (k2b_selftest_wait) on the
    current stream and returns its int[3] result; mode 1 makes a device wait
    run out after `limit_ns` without faulting the context."""
    res = torch.zeros(3, dtype=torch.int32, device=device or torch.device("cuda"))
    check(lib().k2b_selftest_wait(int(mode), int(limit_ns), _p(res), _stream()), "k2b_selftest_wait")
    torch.cuda.current_stream(res.device).synchronize()
    return [int(v) for v in res.cpu()]


__all__ = [
    "K2BError", "PreparedWeight", "prepare_weight", "norm_quant", "norm_quant_rows", "gated_add", "reduce_gated_add", "norm_mod", "elementwise", "rope", "rotate_quant",
    "gemm_f32", "gemm_f32_scatter", "gemm_bf16", "qkv",
    "gated_residual", "swiglu_quant", "swiglu_bf16", "attention", "attention_quant", "device_error",
    "selftest_wait", "norm_quant_e4m3", "gemm_f32_e4m3", "qkv_e4m3", "gated_residual_e4m3", "swiglu_quant_e4m3",
    "attention_quant_e4m3",
]
