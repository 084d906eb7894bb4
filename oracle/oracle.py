"""CPU oracle for the Krea2 W4A4 DiT block hot path.

TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline / reference legs import this module, always as the checker or as
the timed CPU baseline, never as a product path.

The bit-exact integer/rounding stages live in k2_oracle.c (compiled by
oracle/Makefile into oracle/_build/libk2_oracle.so); this module wraps them
with numpy, parallelises them over row blocks (ctypes releases the GIL), and
adds the two float stages written directly in numpy:

* ``attention`` -- restates the Kohaku GQA flash attention
  (KohakuKernelRouter/attention.py:31-110): non-causal, ``kv = h // (Hq/Hkv)``,
  ``c = log2(e)/sqrt(D)``, exp2 softmax in fp32, P rounded to bf16 before PV,
  ``o = bf16(acc/l)`` (0 where l == 0), optional gate store.
* ``rope_table`` -- restates EmbedND (native_runtime.cpp:509-510): per axis of
  dim d, omega = theta^-(linspace(0,(d-2)/d,d/2)) in float64, angle =
  fp32(pos)*omega, [[cos,-sin],[sin,cos]], concatenated over axes, fp32.

Arrays of bf16 / fp16 values are carried as uint16 bit patterns.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from concurrent.futures import ThreadPoolExecutor

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libk2_oracle.so")
LOG2E = 1.4426950408889634

_lib = None
_lock = threading.Lock()


def build() -> str:
    """Compile k2_oracle.c with the committed Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH) or (
                os.path.getmtime(LIB_PATH) < os.path.getmtime(os.path.join(HERE, "k2_oracle.c"))
            ):
                build()
            _lib = ctypes.CDLL(LIB_PATH)
            _declare(_lib)
    return _lib


def _declare(L):
    P = ctypes.c_void_p
    I = ctypes.c_int
    F = ctypes.c_float
    I64 = ctypes.c_int64
    L.k2o_norm_quant.argtypes = [P, P, P, P, P, P, I, I, I, I, I, F]
    L.k2o_rotate_quant.argtypes = [P, P, P, I, I]
    L.k2o_norm_mod.argtypes = [P, P, P, P, P, I, I, I, I, I, F]
    L.k2o_unpack_weight.argtypes = [P, P, I, I, P, P]
    L.k2o_gemm_w4a4_cols.argtypes = [P, P, P, P, I, I, I, P, I, I, I, P, I, P]
    L.k2o_dequant_group.argtypes = [P, P, P, P, I, I]
    L.k2o_ref_quant.argtypes = [P, P, P, P, P, P, I, I, I, I, I, F, I, I]
    L.k2o_qk_norm_rope.argtypes = [P, I, I, I, P, F, P, I, P, P]
    L.k2o_gated_residual.argtypes = [P, I, I, P, P, I, P, P]
    L.k2o_swiglu_quant.argtypes = [P, P, I, I, P, P, P]
    L.k2o_sigmoid_gate.argtypes = [P, I64, P]
    L.k2o_exp_vec.argtypes = [P, P, I64]
    L.k2o_bf16_round_vec.argtypes = [P, P, I64]
    L.k2o_set_bf16_truncate.argtypes = [I]
    L.k2o_exp.argtypes = [F]
    L.k2o_exp.restype = F
    L.k2o_rsqrt_rn.argtypes = [F]
    L.k2o_rsqrt_rn.restype = F


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def _workers() -> int:
    return max(1, min(32, os.cpu_count() or 1))


def _row_blocks(n: int, parts: int):
    parts = max(1, min(parts, n))
    step = (n + parts - 1) // parts
    return [(s, min(n, s + step)) for s in range(0, n, step)]


# ----------------------------------------------------------------- bf16 helpers

class bf16_truncation:
    """Context manager: bf16 conversions truncate instead of rounding to
    nearest even (only to compare with kernels run under the Triton CPU
    interpreter, which truncates)."""

    def __enter__(self):
        lib().k2o_set_bf16_truncate(1)

    def __exit__(self, *exc):
        lib().k2o_set_bf16_truncate(0)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round to nearest even."""
    x = _c(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().k2o_bf16_round_vec(_p(x), _p(out), x.size)
    return out


def bf16_float(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    return bf16_float(bf16_bits(x))


def f16_float(b: np.ndarray) -> np.ndarray:
    return np.asarray(b, np.uint16).view(np.float16).astype(np.float32)


def exp(x: np.ndarray) -> np.ndarray:
    x = _c(x, np.float32)
    y = np.empty_like(x)
    lib().k2o_exp_vec(_p(x), _p(y), x.size)
    return y


# --------------------------------------------------------------- kernels (C)

def norm_quant(x, w, scale, shift, length=None, cut=-1, batch=None, eps=1e-6):
    """x bf16 bits [rows,K]; w fp32 [K] ("w+1" form); scale/shift bf16 bits
    [nb,K].  Returns (q u8 [rows,K/2], s fp16 bits [rows,K/128])."""
    x = _c(x, np.uint16)
    rows, K = x.shape
    length = rows if length is None else length
    batch = max(1, rows // length) if batch is None else batch
    w = _c(w, np.float32)
    scale = _c(scale, np.uint16)
    shift = _c(shift, np.uint16)
    q = np.empty((rows, K // 2), np.uint8)
    s = np.empty((rows, K // 128), np.uint16)
    L = lib()
    if cut >= 0:
        # the cut split needs the absolute row index: run in one call
        code = L.k2o_norm_quant(_p(x), _p(w), _p(scale), _p(shift), _p(q), _p(s), rows, K,
                                length, cut, batch, ctypes.c_float(eps))
        assert code == 0
        return q, s
    # Row blocks inside one latent share one modulation row: each block is
    # run as its own single-latent call on that row.
    blocks = []
    for b0 in range(0, rows, length):
        b1 = min(rows, b0 + length)
        for a, b in _row_blocks(b1 - b0, _workers()):
            blocks.append((b0 // length, b0 + a, b0 + b))

    def job(t):
        bidx, a, b = t
        code = L.k2o_norm_quant(_p(x[a:b]), _p(w), _p(scale[bidx:bidx + 1]), _p(shift[bidx:bidx + 1]),
                                _p(q[a:b]), _p(s[a:b]), b - a, K, b - a, -1, 1, ctypes.c_float(eps))
        assert code == 0

    with ThreadPoolExecutor(_workers()) as ex:
        list(ex.map(job, blocks))
    return q, s


def norm_mod(x, w, scale, shift, length=None, cut=-1, batch=None, eps=1e-6):
    """RMSNorm + adaLN modulation only (bf16 bits out), the pre-rotation half
    of norm_quant."""
    x = _c(x, np.uint16)
    rows, K = x.shape
    length = rows if length is None else length
    batch = max(1, rows // length) if batch is None else batch
    out = np.empty_like(x)
    assert lib().k2o_norm_mod(_p(x), _p(_c(w, np.float32)), _p(_c(scale, np.uint16)), _p(_c(shift, np.uint16)),
                              _p(out), rows, K, length, cut, batch, ctypes.c_float(eps)) == 0
    return out


def rotate_quant(x):
    """bf16 bits [rows,K] -> (q u8 [rows,K/2], s fp16 bits [rows,K/128])."""
    x = _c(x, np.uint16)
    rows, K = x.shape
    q = np.empty((rows, K // 2), np.uint8)
    s = np.empty((rows, K // 128), np.uint16)
    L = lib()

    def job(ab):
        a, b = ab
        assert L.k2o_rotate_quant(_p(x[a:b]), _p(q[a:b]), _p(s[a:b]), b - a, K) == 0

    with ThreadPoolExecutor(_workers()) as ex:
        list(ex.map(job, _row_blocks(rows, _workers() * 2)))
    return q, s


def unpack_weight(W, sW):
    """Packed INT4 [N,K/2] + fp16 bits [N,K/128] -> (int8 [N,K], fp32 [N,K/128])."""
    W = _c(W, np.uint8)
    sW = _c(sW, np.uint16)
    N, K2 = W.shape
    K = 2 * K2
    wu = np.empty((N, K), np.int8)
    swf = np.empty((N, K // 128), np.float32)
    L = lib()

    def job(ab):
        a, b = ab
        assert L.k2o_unpack_weight(_p(W[a:b]), _p(sW[a:b]), b - a, K, _p(wu[a:b]), _p(swf[a:b])) == 0

    with ThreadPoolExecutor(_workers()) as ex:
        list(ex.map(job, _row_blocks(N, _workers() * 2)))
    return wu, swf


def gemm_w4a4(A, sA, W, sW, rows=None, with_acc=False, unpacked=None):
    """Group-scaled W4A4 GEMM.  A u8 [M,K/2], sA fp16 bits [M,K/128], W u8
    [N,K/2], sW fp16 bits [N,K/128] (or unpacked=(int8 or fp32 codes [N,K],
    fp32 scales [N,K/128])).
    rows: optional row indices.  Returns fp32 [len(rows), N] (and int32
    [len(rows), N, K/128])."""
    A = _c(A, np.uint8)
    sA = _c(sA, np.uint16)
    wu, swf = unpacked if unpacked is not None else unpack_weight(W, sW)
    if not with_acc:
        return _gemm_w4a4_blas(A, sA, wu, swf, rows)
    M, K2 = A.shape
    N = wu.shape[0]
    K = K2 * 2
    rows = np.arange(M, dtype=np.int32) if rows is None else _c(rows, np.int32)
    n = rows.size
    out = np.empty((n, N), np.float32)
    acc = np.empty((n, N, K // 128), np.int32) if with_acc else None
    L = lib()
    w = _workers()
    rb = _row_blocks(n, w)
    cb = _row_blocks(N, max(1, (2 * w) // len(rb)))
    jobs = [(a, b, c0, c1) for a, b in rb for c0, c1 in cb]

    def job(t):
        a, b, c0, c1 = t
        code = L.k2o_gemm_w4a4_cols(_p(A), _p(sA), _p(wu), _p(swf), M, N, K, _p(rows[a:b]), b - a, c0, c1,
                                    _p(out[a:b]), N, _p(acc[a:b]) if with_acc else None)
        assert code == 0

    with ThreadPoolExecutor(w) as ex:
        list(ex.map(job, jobs))
    return (out, acc) if with_acc else out


def _gemm_w4a4_blas(A, sA, wu, swf, rows):
    """gemm_w4a4's result with the group accumulators formed by fp32 BLAS
    matmuls of the integer codes (exact: every partial sum is an integer below
    2^24 in magnitude) and the dequant chain in C (k2o_dequant_group), group by
    group in increasing g -- the same fp32 operations as k2o_gemm_w4a4_cols."""
    if rows is not None:
        rows = _c(rows, np.int64)
        A, sA = A[rows], sA[rows]
    au, saf = unpack_weight(A, sA)
    n, K = au.shape
    N = wu.shape[0]
    G = K // 128
    af = au.astype(np.float32)
    # weights may come pre-converted (fp32 codes), like resident GPU weights
    wf = _c(wu, np.float32) if wu.dtype == np.float32 else _c(wu, np.int8).astype(np.float32)
    saT = np.ascontiguousarray(saf.T)
    swT = np.ascontiguousarray(_c(swf, np.float32).T)
    out = np.zeros((n, N), np.float32)
    L = lib()
    w = _workers()
    rb = max(1, min(n, (1 << 25) // max(1, N)))
    with ThreadPoolExecutor(w) as ex:
        for r0 in range(0, n, rb):
            r1 = min(n, r0 + rb)
            for g in range(G):
                acc = np.ascontiguousarray(af[r0:r1, g * 128:(g + 1) * 128] @ wf[:, g * 128:(g + 1) * 128].T)

                def job(ab, acc=acc, r0=r0, g=g):
                    a, b = ab
                    assert L.k2o_dequant_group(_p(acc[a:b]), _p(saT[g, r0 + a:r0 + b]), _p(swT[g]),
                                               _p(out[r0 + a:r0 + b]), b - a, N) == 0

                list(ex.map(job, _row_blocks(r1 - r0, w)))
    return out


def qk_norm_rope(p, heads, normw, eps, freqs, L, rows=None):
    """p fp32 [n, heads*128]; returns bf16 bits [n, heads*128]."""
    p = _c(p, np.float32)
    n = p.shape[0]
    rows = np.arange(n, dtype=np.int32) if rows is None else _c(rows, np.int32)
    out = np.empty((n, heads * 128), np.uint16)
    normw = _c(normw, np.float32)
    freqs = _c(freqs, np.float32)
    lib().k2o_qk_norm_rope(_p(p), n, p.shape[1], heads, _p(normw), ctypes.c_float(eps), _p(freqs),
                           L, _p(rows), _p(out))
    return out


def gated_residual(p, gate, resid, length, rows=None):
    p = _c(p, np.float32)
    n, N = p.shape
    rows = np.arange(n, dtype=np.int32) if rows is None else _c(rows, np.int32)
    gate = _c(gate, np.uint16).reshape(-1, N)
    resid = _c(resid, np.uint16)
    out = np.empty((n, N), np.uint16)
    lib().k2o_gated_residual(_p(p), n, N, _p(gate), _p(resid), length, _p(rows), _p(out))
    return out


def swiglu_quant(pg, pu, want_h=False):
    pg = _c(pg, np.float32)
    pu = _c(pu, np.float32)
    n, F = pg.shape
    hq = np.empty((n, F // 2), np.uint8)
    hs = np.empty((n, F // 128), np.uint16)
    h = np.empty((n, F), np.uint16) if want_h else None
    L = lib()

    def job(ab):
        a, b = ab
        assert L.k2o_swiglu_quant(_p(pg[a:b]), _p(pu[a:b]), b - a, F, _p(hq[a:b]), _p(hs[a:b]),
                                  _p(h[a:b]) if want_h else None) == 0

    with ThreadPoolExecutor(_workers()) as ex:
        list(ex.map(job, _row_blocks(n, _workers())))
    return (hq, hs, h) if want_h else (hq, hs)


def sigmoid_gate(p):
    p = _c(p, np.float32)
    out = np.empty(p.shape, np.uint16)
    lib().k2o_sigmoid_gate(_p(p), p.size, _p(out))
    return out


def dequant(q, s):
    """Unpacked float view of packed codes: value = code * scale (fp32)."""
    q = np.asarray(q, np.uint8)
    lo = (q & 0xF).astype(np.int8)
    hi = (q >> 4).astype(np.int8)
    lo = np.where(lo >= 8, lo - 16, lo)
    hi = np.where(hi >= 8, hi - 16, hi)
    codes = np.empty(q.shape[:-1] + (q.shape[-1] * 2,), np.float32)
    codes[..., 0::2] = lo
    codes[..., 1::2] = hi
    sc = np.repeat(f16_float(s), 128, axis=-1)
    return codes * sc


# --------------------------------------------------------------- float stages

def attention(q, k, v, gate=None, gate_is_sigmoid=True, rows=None):
    """GQA attention oracle.  q [B,Hq,Lq,D], k/v [B,Hkv,Lk,D] as bf16 bits
    (or float arrays already on the bf16 grid).  Returns bf16 bits
    [B, len(rows), Hq*D] (token-major, KohakuKernelRouter/attention.py:161).
    gate: bf16 bits [B, Lq, Hq*D] applied as bf16(o*gate) (pre-sigmoided when
    gate_is_sigmoid, else sigmoid applied first, attention.py:104-109)."""
    def f(a):
        a = np.asarray(a)
        return bf16_float(a) if a.dtype == np.uint16 else a.astype(np.float32)

    qf, kf, vf = f(q), f(k), f(v)
    B, Hq, Lq, D = qf.shape
    Hkv = kf.shape[1]
    group = Hq // Hkv
    rows = np.arange(Lq) if rows is None else np.asarray(rows)
    c = np.float32(LOG2E / np.sqrt(D))
    out = np.empty((B, rows.size, Hq * D), np.uint16)
    gf = f(gate) if gate is not None else None

    def head(bh):
        b, h = bh
        kh = h // group
        s = (qf[b, h, rows].astype(np.float64) @ kf[b, kh].astype(np.float64).T).astype(np.float32)
        m = s.max(axis=1, keepdims=True)
        p = np.exp2((s - m) * c).astype(np.float32)
        l = p.sum(axis=1, dtype=np.float64)
        pb = bf16_round(p).astype(np.float64)
        acc = pb @ vf[b, kh].astype(np.float64)
        o = np.where(l[:, None] == 0, 0.0, acc / np.where(l == 0, 1.0, l)[:, None]).astype(np.float32)
        ob = bf16_round(o)
        if gf is not None:
            g = gf[b, rows, h * D:(h + 1) * D]
            if not gate_is_sigmoid:
                g = bf16_round(1.0 / (1.0 + np.exp(-g.astype(np.float32))))
            ob = bf16_round(ob * g)
        out[b, :, h * D:(h + 1) * D] = bf16_bits(ob)

    # heads are independent; numpy's matmuls and ufuncs release the GIL
    with ThreadPoolExecutor(max(1, min(8, _workers()))) as ex:
        list(ex.map(head, [(b, h) for b in range(B) for h in range(Hq)]))
    return out


def rope_table(pos: np.ndarray, axes, theta: float) -> np.ndarray:
    """pos fp32 [L, n_axes] -> fp32 [L, sum(axes)/2, 2, 2]."""
    pieces = []
    for i, d in enumerate(axes):
        scale = np.linspace(0.0, (d - 2) / d, d // 2, dtype=np.float64)
        omega = 1.0 / np.power(float(theta), scale)
        angle = pos[:, i].astype(np.float32).astype(np.float64)[:, None] * omega
        cos, sin = np.cos(angle), np.sin(angle)
        pieces.append(np.stack([cos, -sin, sin, cos], axis=-1).reshape(pos.shape[0], d // 2, 2, 2))
    return np.concatenate(pieces, axis=1).astype(np.float32)


# ------------------------------------------------- reference contract (parity)
# The reference's own data contract at its kernel-library symbols
# (native_runtime.cpp:262-311, 399-447): one fp32 scale per activation row and
# per weight channel, ConvRot in groups of 16/64/256, full-K accumulation.

def ref_quant(x, w=None, scale=None, shift=None, length=None, cut=-1, batch=None, eps=1e-6, group=256, bits=4):
    """x bf16 bits [rows, K] -> (q u8 [rows, K/2] packed INT4 or int8 [rows, K],
    s fp32 [rows]); optional RMSNorm + modulation first (w fp32 "w+1" form,
    scale/shift bf16 bits [nb, K]).  k2o_ref_quant."""
    x = _c(x, np.uint16)
    rows, K = x.shape
    length = rows if length is None else length
    batch = max(1, rows // length) if batch is None else batch
    q = np.empty((rows, K // 2 if bits == 4 else K), np.uint8 if bits == 4 else np.int8)
    s = np.empty(rows, np.float32)
    wv = None if w is None else _c(w, np.float32)
    sc = None if scale is None else _c(scale, np.uint16)
    sh = None if shift is None else _c(shift, np.uint16)
    assert lib().k2o_ref_quant(_p(x), _p(wv), _p(sc), _p(sh), _p(q), _p(s), rows, K, length, cut, batch,
                               ctypes.c_float(eps), group, bits) == 0
    return q, s


def int4_codes(packed):
    """packed u8 [rows, K/2] -> int8 codes [rows, K] (low nibble = even column)."""
    p = _c(packed, np.uint8)
    c = np.empty((p.shape[0], p.shape[1] * 2), np.int8)
    lo, hi = (p & 0xF).astype(np.int8), (p >> 4).astype(np.int8)
    c[:, 0::2] = np.where(lo >= 8, lo - 16, lo)
    c[:, 1::2] = np.where(hi >= 8, hi - 16, hi)
    return c


def ref_project(a_codes, xs, w_codes, ws, bias=None):
    """Reference-contract projection before its rounding to T:
    p = fp32(fp32(float(acc) * xs[r]) * ws[c]) (+ bias[c]), acc over all of K
    (kernels/joint_projection.cu:57-59).  a_codes [m, K], w_codes [n, K] integer
    codes (INT4 or int8); the accumulators are exact integers (fp32 BLAS of
    integer codes whose partial sums stay below 2^24 in magnitude)."""
    a = np.asarray(a_codes, np.float32)
    w = np.asarray(w_codes, np.float32)
    acc = a @ w.T
    assert np.abs(acc).max(initial=0) < 2 ** 24
    p = (acc.astype(np.float32) * _c(xs, np.float32).reshape(-1, 1)).astype(np.float32)
    p = (p * _c(ws, np.float32).reshape(1, -1)).astype(np.float32)
    if bias is not None:
        p = (p + _c(bias, np.float32).reshape(1, -1)).astype(np.float32)
    return p
