"""The reference-named exports with the reference's own data contract
(one fp32 scale per activation row and per weight channel, packed INT4 weights
as a ConvRot W4A4 checkpoint stores them, ConvRot groups 16/64/256,
full-K accumulation), through the C ABI:

* bit-exact against the oracle's restatement of that contract;
* against the reference's own kernels/joint_projection.cu, compiled from its
  sources for sm_100a into oracle/_ref (oracle/Makefile `ref`) and run on the
  same device buffers: the plain projection (V) and the gated residual bit for
  bit; the outputs that pass through the reference's rsqrtf/expf (Q/K norm,
  sigmoid gate, SiLU, the row norm) within one bf16 rounding step, because
  this library uses a correctly rounded rsqrt and its own exp.
"""
import ctypes
import os

import numpy as np
import pytest

import oracle as O
from _helpers import TOL_ABS, bf16_x, bits, norm_inputs, t_bf16, t_f32, t_u8

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_JOINT = os.path.join(ROOT, "oracle", "_ref", "libref_joint.so")


_ALIVE = []  # device buffers passed by pointer must outlive the launch


def _p(t):
    """Device pointer of t, keeping t alive until the test ends (a temporary
    freed right after .data_ptr() is recycled by torch's caching allocator,
    and a kernel launched later would read whatever took its place)."""
    if t is None:
        return ctypes.c_void_p(0)
    _ALIVE.append(t)
    return ctypes.c_void_p(t.data_ptr())


@pytest.fixture(autouse=True)
def _release_buffers():
    yield
    import torch

    torch.cuda.synchronize()
    _ALIVE.clear()


def _stream():
    import torch

    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _lib():
    from k2b._native import lib

    return lib()


def _weights(n, k, seed):
    """Per-channel INT4 weight: packed [n, k/2] + fp32 scales [n]."""
    rng = np.random.default_rng(seed)
    w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    ws = (np.abs(w).max(axis=1) / 7.0).astype(np.float32)
    codes = np.clip(np.rint(w / ws[:, None]), -8, 7).astype(np.int8)
    packed = ((codes[:, 0::2] & 0xF) | ((codes[:, 1::2] & 0xF) << 4)).astype(np.uint8)
    return packed, ws, codes


def _act(m, k, seed, group=256):
    x = bf16_x(m, k, seed, outliers=False)
    q, s = O.ref_quant(x, group=group)
    return x, q, s


def test_ref_quantisers_bit_exact(cuda):
    import torch

    L = _lib()
    for rows, K, group in ((37, 1024, 16), (64, 1536, 64), (129, 6144, 256)):
        x = bf16_x(rows, K, 3)
        xg = t_bf16(x, cuda)
        q = torch.empty((rows, K // 2), dtype=torch.uint8, device=cuda)
        s = torch.empty((rows, 1), dtype=torch.float32, device=cuda)
        L.k2b_shim_status(1)
        L.k2_quant4(_p(xg), _p(q), _p(s), rows, K, group, 2, _stream())
        torch.cuda.synchronize()
        assert L.k2b_shim_status(1) == 0
        q_r, s_r = O.ref_quant(x, group=group)
        assert np.array_equal(q.cpu().numpy(), q_r) and np.array_equal(s.cpu().numpy()[:, 0], s_r)
        for g8 in (0, group):
            q8 = torch.empty((rows, K), dtype=torch.int8, device=cuda)
            L.k2_quant8(_p(xg), _p(q8), _p(s), rows, K, g8, 2, _stream())
            torch.cuda.synchronize()
            assert L.k2b_shim_status(1) == 0
            q8_r, s8_r = O.ref_quant(x, group=g8, bits=8)
            assert np.array_equal(q8.cpu().numpy(), q8_r) and np.array_equal(s.cpu().numpy()[:, 0], s8_r)
    # fused norm + modulation + rotation + quant, two latents and a cut
    length, K, nb = 50, 6144, 2
    x = bf16_x(length * nb, K, 4)
    w, sc, sh = norm_inputs(K, 2 * nb, 5)
    q = torch.empty((length * nb, K // 2), dtype=torch.uint8, device=cuda)
    s = torch.empty((length * nb, 1), dtype=torch.float32, device=cuda)
    for cut in (-1, 20):
        rc = L.k2_norm_mod_quant4(_p(t_bf16(x, cuda)), _p(t_f32(w, cuda)), _p(t_bf16(sc, cuda)),
                                  _p(t_bf16(sh, cuda)), _p(q), _p(s), length * nb, K, length, cut, nb,
                                  ctypes.c_float(1e-6), 256, 2, _stream())
        torch.cuda.synchronize()
        assert rc == 0
        q_r, s_r = O.ref_quant(x, w, sc, sh, length=length, cut=cut, batch=nb, group=256)
        assert np.array_equal(q.cpu().numpy(), q_r) and np.array_equal(s.cpu().numpy()[:, 0], s_r)
    # the e4m3 code-byte outputs hold the same codes
    from _helpers import E4M3
    from k2b import ref_ops

    for cut in (-1, 20):
        q8, s8 = ref_ops.norm_quant4_e4m3(t_bf16(x, cuda), t_f32(w, cuda), t_bf16(sc, cuda), t_bf16(sh, cuda),
                                          length=length, cut=cut, group=256)
        q_r, s_r = O.ref_quant(x, w, sc, sh, length=length, cut=cut, batch=nb, group=256)
        assert np.array_equal(q8.view(torch.uint8).cpu().numpy(), E4M3[O.int4_codes(q_r) + 8])
        assert np.array_equal(s8.cpu().numpy()[:, 0], s_r)
    for group in (16, 64, 256):
        q8, s8 = ref_ops.quant4_e4m3(t_bf16(x, cuda), group)
        q_r, s_r = O.ref_quant(x, group=group)
        assert np.array_equal(q8.view(torch.uint8).cpu().numpy(), E4M3[O.int4_codes(q_r) + 8])
        assert np.array_equal(s8.cpu().numpy()[:, 0], s_r)
    # the reference contract only: group 128 and fp16 are rejected
    assert L.k2_norm_mod_quant4(_p(t_bf16(x, cuda)), _p(t_f32(w, cuda)), _p(t_bf16(sc, cuda)), _p(t_bf16(sh, cuda)),
                                _p(q), _p(s), length * nb, K, length, -1, nb, ctypes.c_float(1e-6), 128, 2,
                                _stream()) == 1


def test_ref_gemm4_and_joint_kernels_match_oracle(cuda):
    import torch
    from k2b.model import rope_positions, rope_table

    L = _lib()
    m, K = 300, 1536
    _, a, xs = _act(m, K, 11)
    ac = O.int4_codes(a)
    A, XS = t_u8(a, cuda), t_f32(xs, cuda)
    # k2_gemm4 with and without bias
    wq, ws, wc = _weights(384, K, 12)
    bias = np.random.default_rng(13).normal(0, 0.1, 384).astype(np.float32)
    out = torch.empty((m, 384), dtype=torch.bfloat16, device=cuda)
    for b in (None, bias):
        L.k2_gemm4(_p(A), _p(t_u8(wq, cuda)), _p(XS), _p(t_f32(ws, cuda)), _p(None if b is None else t_f32(b, cuda)),
                   _p(out), m, 384, K, 2, _stream())
        torch.cuda.synchronize()
        assert L.k2b_shim_status(1) == 0
        ref = O.bf16_bits(O.ref_project(ac, xs, wc, ws, b))
        assert np.array_equal(bits(out), ref)
    # joint QKV with the attention gate (heads 4 / kv 2), RoPE over m tokens
    W = {name: _weights(n, K, 20 + i) for i, (name, n) in enumerate((("q", 512), ("k", 256), ("v", 256),
                                                                        ("g", 512)))}
    rng = np.random.default_rng(30)
    nq, nk = (rng.uniform(-0.1, 0.1, 128).astype(np.float32) for _ in range(2))
    freqs = rope_table(rope_positions(m - 16 * 18, 16, 18), (64, 64), 10000.0)
    fn = freqs.numpy()
    outs = {n: torch.empty((m, W[n][0].shape[0]), dtype=torch.bfloat16, device=cuda) for n in W}
    Wd = {n: (t_u8(W[n][0], cuda), t_f32(W[n][1], cuda)) for n in W}
    rc = L.k2_int4_qkv(_p(A), _p(Wd["q"][0]), _p(Wd["k"][0]), _p(Wd["v"][0]), _p(Wd["g"][0]), _p(XS),
                       _p(Wd["q"][1]), _p(Wd["k"][1]), _p(Wd["v"][1]), _p(Wd["g"][1]), _p(t_f32(nq, cuda)),
                       _p(t_f32(nk, cuda)), _p(freqs.to(cuda)), _p(outs["q"]), _p(outs["k"]), _p(outs["v"]),
                       _p(outs["g"]), m, 512, 256, K, 0, ctypes.c_float(1e-6), ctypes.c_float(1e-6), _stream())
    torch.cuda.synchronize()
    assert rc == 0
    P = {n: O.ref_project(ac, xs, W[n][2], W[n][1]) for n in W}
    assert np.array_equal(bits(outs["q"]), O.qk_norm_rope(P["q"], 4, nq, 1e-6, fn, m))
    assert np.array_equal(bits(outs["k"]), O.qk_norm_rope(P["k"], 2, nk, 1e-6, fn, m))
    assert np.array_equal(bits(outs["v"]), O.bf16_bits(P["v"]))
    assert np.array_equal(bits(outs["g"]), O.sigmoid_gate(P["g"]))
    # SwiGLU (bf16 h)
    wg, sg, gc = _weights(256, K, 40)
    wu, su, uc = _weights(256, K, 41)
    h = torch.empty((m, 256), dtype=torch.bfloat16, device=cuda)
    rc = L.k2_int4_swiglu(_p(A), _p(t_u8(wg, cuda)), _p(t_u8(wu, cuda)), _p(XS), _p(t_f32(sg, cuda)),
                          _p(t_f32(su, cuda)), _p(h), m, 256, K, 0, _stream())
    torch.cuda.synchronize()
    assert rc == 0
    pg, pu = O.ref_project(ac, xs, gc, sg), O.ref_project(ac, xs, uc, su)
    assert np.array_equal(bits(h), O.swiglu_quant(pg, pu, want_h=True)[2])
    # gated residual + the row norm of k2_int4_residual_norm
    wo, so, oc = _weights(1024, K, 50)
    gate = O.bf16_bits(rng.normal(0, 0.1, 1024).astype(np.float32))
    resid = O.bf16_bits(rng.standard_normal((m, 1024)).astype(np.float32))
    nw, nsc, nsh = norm_inputs(1024, 1, 51)
    o = torch.empty((m, 1024), dtype=torch.bfloat16, device=cuda)
    nrm = torch.empty_like(o)
    counters = torch.zeros(8, dtype=torch.int32, device=cuda)
    rc = L.k2_int4_residual_norm(_p(A), _p(t_u8(wo, cuda)), _p(XS), _p(t_f32(so, cuda)), _p(t_bf16(gate, cuda)),
                                 _p(t_bf16(resid, cuda)), _p(t_f32(nw, cuda)), _p(t_bf16(nsc, cuda)),
                                 _p(t_bf16(nsh, cuda)), _p(o), _p(nrm), _p(counters), m, 1024, K, 0,
                                 ctypes.c_float(1e-6), _stream())
    torch.cuda.synchronize()
    assert rc == 0
    o_r = O.gated_residual(O.ref_project(ac, xs, oc, so), gate.reshape(1, -1), resid, m)
    assert np.array_equal(bits(o), o_r)
    assert np.array_equal(bits(nrm), O.norm_mod(o_r, nw, nsc, nsh, eps=1e-6))


def test_ref_dequant8_and_fp8(cuda):
    import torch

    L = _lib()
    rng = np.random.default_rng(60)
    m, n = 77, 384
    acc = rng.integers(-2 ** 20, 2 ** 20, (m, n), dtype=np.int32)
    xs = rng.uniform(1e-3, 1e-2, m).astype(np.float32)
    for ns in (n, 1):
        ws = rng.uniform(1e-3, 1e-2, ns).astype(np.float32)
        bias = O.bf16_bits(rng.normal(0, 0.1, n).astype(np.float32))
        out = torch.empty((m, n), dtype=torch.bfloat16, device=cuda)
        L.k2_dequant8(_p(torch.from_numpy(acc).to(cuda)), _p(t_f32(xs, cuda)), _p(t_f32(ws, cuda)),
                      _p(t_bf16(bias, cuda)), _p(out), m, n, ns, 2, _stream())
        torch.cuda.synchronize()
        assert L.k2b_shim_status(1) == 0
        p = (acc.astype(np.float32) * xs[:, None]).astype(np.float32) * ws.reshape(1, -1)
        p = (p.astype(np.float32) + O.bf16_float(bias)[None, :]).astype(np.float32)
        assert np.array_equal(bits(out), O.bf16_bits(p))
    # fp8 round trip through one scale: quantise (x / s) then dequantise (x * s)
    x = torch.randn(4096, device=cuda).to(torch.bfloat16) * 3
    s = torch.tensor([0.05], dtype=torch.float32, device=cuda)
    for code, dt in ((5, torch.float8_e4m3fn), (6, torch.float8_e5m2)):
        q = torch.empty(4096, dtype=torch.uint8, device=cuda)
        L.k2_fp8(_p(x), _p(q), _p(s), 4096, 2, code, True, _stream())
        y = torch.empty(4096, dtype=torch.bfloat16, device=cuda)
        L.k2_fp8(_p(q), _p(y), _p(s), 4096, code, 2, False, _stream())
        torch.cuda.synchronize()
        assert L.k2b_shim_status(1) == 0
        ref_q = (x.float() / 0.05).clamp(-torch.finfo(dt).max, torch.finfo(dt).max).to(dt)
        assert torch.equal(q, ref_q.view(torch.uint8))
        assert torch.equal(y, (ref_q.float() * 0.05).to(torch.bfloat16))


@pytest.mark.skipif(not os.path.exists(REF_JOINT), reason="oracle/_ref not built (needs the reference's sources)")
def test_ref_joint_kernels_agree_with_the_references_own(cuda):
    """The reference's own joint projection kernels (its kernels/joint_projection.cu
    compiled for sm_100a) and this library's reference-named exports on the
    same device buffers."""
    import torch
    from k2b.model import rope_positions, rope_table

    L = _lib()
    R = ctypes.CDLL(REF_JOINT, mode=os.RTLD_NOW | os.RTLD_LOCAL)
    m, K = 262, 1536
    _, a, xs = _act(m, K, 71)
    A, XS = t_u8(a, cuda), t_f32(xs, cuda)
    W = {name: _weights(n, K, 72 + i) for i, (name, n) in enumerate((("q", 512), ("k", 256), ("v", 256),
                                                                        ("g", 512)))}
    Wd = {n: (t_u8(W[n][0], cuda), t_f32(W[n][1], cuda)) for n in W}
    rng = np.random.default_rng(80)
    nq, nk = (t_f32(rng.uniform(-0.1, 0.1, 128).astype(np.float32), cuda) for _ in range(2))
    freqs = rope_table(rope_positions(m - 12 * 18, 12, 18), (64, 64), 10000.0).to(cuda)

    def qkv(fn):
        o = {n: torch.empty((m, W[n][0].shape[0]), dtype=torch.bfloat16, device=cuda) for n in W}
        rc = fn(_p(A), _p(Wd["q"][0]), _p(Wd["k"][0]), _p(Wd["v"][0]), _p(Wd["g"][0]), _p(XS), _p(Wd["q"][1]),
                _p(Wd["k"][1]), _p(Wd["v"][1]), _p(Wd["g"][1]), _p(nq), _p(nk), _p(freqs), _p(o["q"]), _p(o["k"]),
                _p(o["v"]), _p(o["g"]), m, 512, 256, K, 0, ctypes.c_float(1e-6), ctypes.c_float(1e-6), _stream())
        torch.cuda.synchronize()
        assert rc == 0
        return o

    R.k2_int4_qkv.restype = ctypes.c_int
    mine, theirs = qkv(L.k2_int4_qkv), qkv(R.k2_int4_qkv)
    assert torch.equal(mine["v"], theirs["v"])  # T(acc * xs * ws): bit for bit
    for n in ("q", "k", "g"):  # rsqrtf / expf in the reference
        d = (mine[n].float() - theirs[n].float()).abs()
        assert float(d.max()) <= TOL_ABS, (n, float(d.max()))
        assert float((d == 0).float().mean()) > 0.95, n

    # SwiGLU
    wg, sg, _ = _weights(256, K, 90)
    wu, su, _ = _weights(256, K, 91)
    hs = []
    for fn in (L.k2_int4_swiglu, R.k2_int4_swiglu):
        h = torch.empty((m, 256), dtype=torch.bfloat16, device=cuda)
        assert fn(_p(A), _p(t_u8(wg, cuda)), _p(t_u8(wu, cuda)), _p(XS), _p(t_f32(sg, cuda)), _p(t_f32(su, cuda)),
                  _p(h), m, 256, K, 0, _stream()) == 0
        torch.cuda.synchronize()
        hs.append(h)
    d = (hs[0].float() - hs[1].float()).abs()
    assert float(d.max()) <= TOL_ABS and float((d == 0).float().mean()) > 0.95

    # gated residual + row norm (the reference's fused last-CTA kernel)
    wo, so, _ = _weights(1024, K, 92)
    gate = t_bf16(O.bf16_bits(rng.normal(0, 0.1, 1024).astype(np.float32)), cuda)
    resid = t_bf16(O.bf16_bits(rng.standard_normal((m, 1024)).astype(np.float32)), cuda)
    nw, nsc, nsh = (t_f32(v, cuda) if i == 0 else t_bf16(v, cuda)
                    for i, v in enumerate(norm_inputs(1024, 1, 93)))
    res = []
    for fn in (L.k2_int4_residual_norm, R.k2_int4_residual_norm):
        o = torch.empty((m, 1024), dtype=torch.bfloat16, device=cuda)
        nrm = torch.empty_like(o)
        counters = torch.zeros((m + 127) // 128, dtype=torch.int32, device=cuda)
        assert fn(_p(A), _p(t_u8(wo, cuda)), _p(XS), _p(t_f32(so, cuda)), _p(gate), _p(resid), _p(nw), _p(nsc),
                  _p(nsh), _p(o), _p(nrm), _p(counters), m, 1024, K, 0, ctypes.c_float(1e-6), _stream()) == 0
        torch.cuda.synchronize()
        res.append((o, nrm))
    assert torch.equal(res[0][0], res[1][0])  # T(resid + T(T(p) * gate)): bit for bit
    d = (res[0][1].float() - res[1][1].float()).abs()
    assert float(d.max()) <= TOL_ABS and float((d == 0).float().mean()) > 0.95


def test_byte_operand_forms_equal_the_packed_forms(cuda):
    """The byte-operand forms (A and W as e4m3 code bytes: k2b_ref_qkv8,
    k2b_ref_swiglu8, k2b_ref_gated_residual8, k2b_gemm_f8 with per-row /
    per-channel scales) give the bits of the packed forms the reference-named
    exports run, bias included."""
    import torch
    from k2b import ref_ops
    from k2b.model import rope_positions, rope_table

    m, K, L = 256, 1536, 128
    _, a, xs = _act(m, K, 101, group=64)
    A, XS = t_u8(a, cuda).view(torch.int8), t_f32(xs, cuda)
    A8 = ref_ops.codes_e4m3(A)
    W = {n: _weights(w, K, 110 + i) for i, (n, w) in enumerate((("q", 512), ("k", 256), ("v", 256), ("g", 512),
                                                                 ("o", 384)))}
    Wp = {n: t_u8(W[n][0], cuda).view(torch.int8) for n in W}
    Ws = {n: t_f32(W[n][1], cuda) for n in W}
    W8 = {n: ref_ops.codes_e4m3(Wp[n]) for n in W}
    bias = t_f32(np.random.default_rng(120).normal(0, 0.1, 384).astype(np.float32), cuda)
    assert torch.equal(ref_ops.gemm4(A, XS, Wp["o"], Ws["o"], bias), ref_ops.gemm_f8(A8, XS, W8["o"], Ws["o"], bias))
    rng = np.random.default_rng(121)
    nq, nk = (t_f32(rng.uniform(-0.1, 0.1, 128).astype(np.float32), cuda) for _ in range(2))
    freqs = rope_table(rope_positions(2 * 8, 8, 14), (64, 64), 10000.0).to(cuda)  # [128, 64, 2, 2]
    ks = ("q", "k", "v", "g")
    got = ref_ops.qkv8(A8, XS, [W8[n] for n in ks], [Ws[n] for n in ks], nq, nk, freqs, length=L)
    ref = ref_ops.qkv(A, XS, [Wp[n] for n in ks], [Ws[n] for n in ks], nq, nk, freqs, length=L)
    assert all(torch.equal(x, y) for x, y in zip(got, ref))
    assert torch.equal(ref_ops.swiglu8(A8, XS, W8["q"], Ws["q"], W8["g"], Ws["g"]),
                       ref_ops.swiglu(A, XS, Wp["q"], Ws["q"], Wp["g"], Ws["g"]))
    gate = t_bf16(O.bf16_bits(rng.normal(0, 0.5, (2, 384)).astype(np.float32)), cuda)
    resid = t_bf16(O.bf16_bits(rng.normal(0, 1, (m, 384)).astype(np.float32)), cuda)
    assert torch.equal(ref_ops.gated_residual8(A8, XS, W8["o"], Ws["o"], gate, resid, length=L),
                       ref_ops.gated_residual(A, XS, Wp["o"], Ws["o"], gate, resid, length=L))
