"""tcgen05 W4A4 GEMM and its fused epilogues vs the CPU oracle (bit-exact)."""
import ctypes

import numpy as np
import pytest

import oracle as O
from _helpers import bits, packed_act, packed_weight, t_bf16, t_f16, t_f32, t_u8

pytestmark = pytest.mark.gpu


def _prep(cuda, wq, ws):
    from k2b import ops

    return ops.prepare_weight(t_u8(wq, cuda), t_f16(ws, cuda))


@pytest.mark.parametrize("M,N,K", [(1, 256, 128), (129, 512, 512), (300, 768, 1024), (257, 256, 6144)])
def test_gemm_f32_bitexact(cuda, M, N, K):
    import torch
    from k2b import ops

    a, sa = packed_act(M, K, M + N)
    w, sw = packed_weight(N, K, K + 1)
    out = ops.gemm_f32(t_u8(a, cuda), t_f16(sa, cuda), _prep(cuda, w, sw))
    torch.cuda.synchronize()
    ref = O.gemm_w4a4(a, sa, w, sw)
    got = out.cpu().numpy()
    bad = np.argwhere(got != ref)
    assert bad.size == 0, f"{len(bad)} mismatches, first {bad[:4]} got {got[tuple(bad[0])]} ref {ref[tuple(bad[0])]}"


def test_gemm_int32_accumulators_exact(cuda):
    """Unit scales: p = sum_g acc_g exactly, i.e. the full int32 accumulator."""
    import torch
    from k2b import ops

    M, N, K = 200, 512, 2048
    a, _ = packed_act(M, K, 1)
    w, _ = packed_weight(N, K, 2)
    one_a = np.full((M, K // 128), 0x3C00, np.uint16)  # fp16 1.0
    one_w = np.full((N, K // 128), 0x3C00, np.uint16)
    out = ops.gemm_f32(t_u8(a, cuda), t_f16(one_a, cuda), _prep(cuda, w, one_w))
    torch.cuda.synchronize()
    _, acc = O.gemm_w4a4(a, one_a, w, one_w, with_acc=True)
    expect = acc.sum(axis=2).astype(np.int64)
    assert np.array_equal(out.cpu().numpy().astype(np.int64), expect)


def test_gemm_config1_sampled_rows(cuda):
    """Config 1 shape (M=4050, N=9216, K=6144), rows sampled for the oracle."""
    import torch
    from k2b import ops

    M, N, K = 4050, 9216, 6144
    a, sa = packed_act(M, K, 7)
    w, sw = packed_weight(N, K, 8)
    out = ops.gemm_f32(t_u8(a, cuda), t_f16(sa, cuda), _prep(cuda, w, sw))
    torch.cuda.synchronize()
    rows = np.unique(np.concatenate([np.arange(0, 4), np.arange(M - 84, M - 80),
                                     np.random.default_rng(0).choice(M, 40, replace=False)])).astype(np.int32)
    ref = O.gemm_w4a4(a, sa, w, sw, rows=rows)
    assert np.array_equal(out.cpu().numpy()[rows], ref)


def test_gemm_bf16(cuda):
    import torch
    from k2b import ops

    a, sa = packed_act(130, 512, 3)
    w, sw = packed_weight(512, 512, 4)
    out = ops.gemm_bf16(t_u8(a, cuda), t_f16(sa, cuda), _prep(cuda, w, sw))
    torch.cuda.synchronize()
    assert np.array_equal(bits(out), O.bf16_bits(O.gemm_w4a4(a, sa, w, sw)))


def _qkv_case(cuda, M, length, heads, kvheads, K, gate=False, seed=0):
    import torch
    from k2b import ops
    from k2b.model import rope_positions, rope_table

    a, sa = packed_act(M, K, seed)
    ws = {n: packed_weight(r * 128, K, seed + i + 1) for i, (n, r) in
          enumerate([("q", heads), ("k", kvheads), ("v", kvheads), ("g", heads)])}
    rng = np.random.default_rng(seed + 9)
    nq = (O.bf16_round(rng.uniform(0.9, 1.1, 128).astype(np.float32)) - 1).astype(np.float32)
    nk = (O.bf16_round(rng.uniform(0.9, 1.1, 128).astype(np.float32)) - 1).astype(np.float32)
    side = int(np.ceil(np.sqrt(length)))
    text = length - (length // side) * side
    pos = rope_positions(text, length // side, side).numpy()
    freqs = rope_table(torch.from_numpy(pos), (64, 64), 10000.0).numpy()
    P = {n: _prep(cuda, *v) for n, v in ws.items()}
    q, k, v, g = ops.qkv(t_u8(a, cuda), t_f16(sa, cuda), P["q"], P["k"], P["v"], t_f32(nq, cuda), t_f32(nk, cuda),
                         t_f32(freqs, cuda), length=length, eps_q=1e-6, eps_k=1e-5,
                         wg=P["g"] if gate else None)
    torch.cuda.synchronize()
    return a, sa, ws, nq, nk, freqs, q, k, v, g


@pytest.mark.parametrize("M,length,heads,kvheads,K,gate", [(300, 300, 4, 2, 512, False), (260, 130, 4, 2, 1024, True)])
def test_qkv_epilogue_bitexact(cuda, M, length, heads, kvheads, K, gate):
    a, sa, ws, nq, nk, freqs, q, k, v, g = _qkv_case(cuda, M, length, heads, kvheads, K, gate)
    pq = O.gemm_w4a4(a, sa, *ws["q"])
    pk = O.gemm_w4a4(a, sa, *ws["k"])
    pv = O.gemm_w4a4(a, sa, *ws["v"])
    assert np.array_equal(bits(q), O.qk_norm_rope(pq, heads, nq, 1e-6, freqs, length))
    assert np.array_equal(bits(k), O.qk_norm_rope(pk, kvheads, nk, 1e-5, freqs, length))
    assert np.array_equal(bits(v), O.bf16_bits(pv))
    if gate:
        pg = O.gemm_w4a4(a, sa, *ws["g"])
        assert np.array_equal(bits(g), O.sigmoid_gate(pg))


def test_qkv_config1_sampled_rows(cuda):
    """Config 1: M = 4050 (98 text + 76x52 image), N = 6144 + 1536 + 1536, K = 6144."""
    import torch
    from k2b.model import rope_positions, rope_table

    M, K = 4050, 6144
    a, sa, ws, nq, nk, freqs, q, k, v, _ = _qkv_case(cuda, M, M, 48, 12, K, seed=3)
    freqs = rope_table(rope_positions(98, 76, 52), (64, 64), 10000.0).numpy()
    import k2b.ops as ops

    P = {n: _prep(cuda, *ws[n]) for n in ("q", "k", "v")}
    q, k, v, _ = ops.qkv(t_u8(a, cuda), t_f16(sa, cuda), P["q"], P["k"], P["v"], t_f32(nq, cuda), t_f32(nk, cuda),
                         t_f32(freqs, cuda), length=M, eps_q=1e-6, eps_k=1e-5)
    torch.cuda.synchronize()
    rows = np.array([0, 1, 97, 98, 99, 2000, 3967, 4049], np.int32)
    pq = O.gemm_w4a4(a, sa, *ws["q"], rows=rows)
    pk = O.gemm_w4a4(a, sa, *ws["k"], rows=rows)
    pv = O.gemm_w4a4(a, sa, *ws["v"], rows=rows)
    assert np.array_equal(bits(q)[rows], O.qk_norm_rope(pq, 48, nq, 1e-6, freqs, M, rows=rows))
    assert np.array_equal(bits(k)[rows], O.qk_norm_rope(pk, 12, nk, 1e-5, freqs, M, rows=rows))
    assert np.array_equal(bits(v)[rows], O.bf16_bits(pv))


@pytest.mark.parametrize("M,length,N,K", [(300, 150, 512, 512), (129, 129, 256, 1024)])
def test_gated_residual_bitexact(cuda, M, length, N, K):
    import torch
    from k2b import ops

    a, sa = packed_act(M, K, 5)
    w, sw = packed_weight(N, K, 6)
    rng = np.random.default_rng(7)
    gate = O.bf16_bits(rng.normal(0, 0.1, (M // length, N)).astype(np.float32))
    resid = O.bf16_bits(rng.normal(0, 1, (M, N)).astype(np.float32))
    out = ops.gated_residual(t_u8(a, cuda), t_f16(sa, cuda), _prep(cuda, w, sw), t_bf16(gate, cuda),
                             t_bf16(resid, cuda), length=length)
    torch.cuda.synchronize()
    ref = O.gated_residual(O.gemm_w4a4(a, sa, w, sw), gate, resid, length)
    assert np.array_equal(bits(out), ref)


@pytest.mark.parametrize("M,F,K", [(130, 256, 512), (300, 512, 1024)])
def test_swiglu_quant_bitexact(cuda, M, F, K):
    import torch
    from k2b import ops

    a, sa = packed_act(M, K, 12)
    wg, sg = packed_weight(F, K, 13)
    wu, su = packed_weight(F, K, 14)
    Pg, Pu = _prep(cuda, wg, sg), _prep(cuda, wu, su)
    hq, hs = ops.swiglu_quant(t_u8(a, cuda), t_f16(sa, cuda), Pg, Pu)
    h = ops.swiglu_bf16(t_u8(a, cuda), t_f16(sa, cuda), Pg, Pu)
    torch.cuda.synchronize()
    pg = O.gemm_w4a4(a, sa, wg, sg)
    pu = O.gemm_w4a4(a, sa, wu, su)
    rq, rs, rh = O.swiglu_quant(pg, pu, want_h=True)
    assert np.array_equal(bits(h), rh)
    assert np.array_equal(bits(hs), rs)
    assert np.array_equal(hq.cpu().numpy(), rq)


def test_packed_exports_equal_the_byte_path(cuda):
    """The packed-A C exports (A unpacked inside the CTA) and the route the op
    wrappers take for packed codes (k2b_expand_e4m3, then the byte-A GEMM)
    give identical bits; the expansion is the e4m3 table of the codes."""
    import ctypes

    import torch
    from _helpers import e4m3_bytes
    from k2b import ops
    from k2b._native import lib

    M, K, N = 300, 1024, 512
    a, sa = packed_act(M, K, 91)
    wq, ws = packed_weight(N, K, 92)
    uq, us = packed_weight(N, K, 93)
    A, SA = t_u8(a, cuda), t_f16(sa, cuda)
    W = ops.prepare_weight(t_u8(wq, cuda), t_f16(ws, cuda))
    U = ops.prepare_weight(t_u8(uq, cuda), t_f16(us, cuda))
    a8 = ops.expand_e4m3(A)
    assert np.array_equal(a8.cpu().numpy(), e4m3_bytes(a))
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    out = torch.empty((M, N), dtype=torch.float32, device=cuda)
    assert lib().k2b_gemm_f32(p(A), p(SA), p(W.w), p(W.scale), p(out), M, N, K, st) == 0
    assert torch.equal(out, ops.gemm_f32(A, SA, W)) and torch.equal(out, ops.gemm_f32(a8, SA, W))
    hq = torch.empty((M, N // 2), dtype=torch.uint8, device=cuda)
    hs = torch.empty((M, N // 128), dtype=torch.float16, device=cuda)
    assert lib().k2b_swiglu_quant(p(A), p(SA), p(W.w), p(W.scale), p(U.w), p(U.scale), p(hq), p(hs), M, N, K, st) == 0
    hq2, hs2 = ops.swiglu_quant(A, SA, W, U)
    torch.cuda.synchronize()
    assert torch.equal(hq, hq2) and torch.equal(hs, hs2)
