"""The e4m3 byte containers of the block loop: the same INT4 codes, one e4m3
byte per code, and GEMMs whose fp32 group sums (formed on the tensor cores from
e4m3 operands) are the exact integer sums.

* every producer writes the codes its packed twin writes (decoded bytes ==
  unpacked nibbles) and the same scales;
* every consumer gives the packed twin's output bit for bit;
* the fp32 GEMM equals the oracle bit for bit, including worst-case groups
  (all codes -8: group sums of +8192, and sums that climb to 4096 and cancel).
"""
import numpy as np
import pytest

import oracle as O
from _helpers import E4M3, bf16_x, bits, e4m3_bytes, norm_inputs, packed_act, packed_weight, t_bf16, t_f16, t_f32, t_u8

pytestmark = pytest.mark.gpu


def test_gemm_f32_e4m3_bit_exact(cuda):
    from k2b import ops

    for M, N, K, seed in ((130, 256, 512, 1), (300, 384, 6144, 2), (1, 128, 128, 3)):
        a, sa = packed_act(M, K, seed)
        wq, sw = packed_weight(N, K, seed + 10)
        W = ops.prepare_weight(t_u8(wq, cuda), t_f16(sw, cuda))
        got = ops.gemm_f32_e4m3(t_u8(e4m3_bytes(a), cuda), t_f16(sa, cuda), W)
        ref = O.gemm_w4a4(a, sa, wq, sw)
        packed = ops.gemm_f32(t_u8(a, cuda), t_f16(sa, cuda), W)
        assert np.array_equal(got.cpu().numpy().view(np.uint32), ref.view(np.uint32))
        assert np.array_equal(packed.cpu().numpy().view(np.uint32), ref.view(np.uint32))


def test_gemm_extreme_group_sums_exact(cuda):
    """Groups whose exact sums reach the extremes of the container: every code
    -8 (each product +64, each group sum +8192) and groups that climb to 4096
    before cancelling; scales 1 so the fp32 result is the sum over groups."""
    from k2b import ops

    M, N, K = 256, 256, 512
    one = np.full((M, K // 128), 0x3C00, np.uint16)  # fp16 1.0
    onew = np.full((N, K // 128), 0x3C00, np.uint16)
    a_codes = np.full((M, K), -8, np.int16)
    a_codes[1::2, 64:128] = 7      # odd rows: +7 in the second half of group 0
    a_codes[2::4, :] = 7
    w_codes = np.full((N, K), -8, np.int16)
    w_codes[1::3, :] = 7
    pack = lambda c: ((c[:, 0::2] & 0xF) | ((c[:, 1::2] & 0xF) << 4)).astype(np.uint8)
    a, wq = pack(a_codes), pack(w_codes)
    W = ops.prepare_weight(t_u8(wq, cuda), t_f16(onew, cuda))
    exact = (a_codes.astype(np.int64) @ w_codes.astype(np.int64).T).astype(np.float32)
    got8 = ops.gemm_f32_e4m3(t_u8(E4M3[a_codes + 8], cuda), t_f16(one, cuda), W).cpu().numpy()
    got4 = ops.gemm_f32(t_u8(a, cuda), t_f16(one, cuda), W).cpu().numpy()
    assert np.array_equal(got8, exact) and np.array_equal(got4, exact)
    assert exact.max() == 4 * 8192


def test_norm_quant_e4m3_same_codes(cuda):
    from k2b import ops

    for length, K, nb in ((4050, 6144, 1), (43, 1024, 3)):
        xb = bf16_x(length * nb, K, 5)
        w, sc, sh = norm_inputs(K, nb, 6)
        args = (t_bf16(xb, cuda), t_f32(w, cuda), t_bf16(sc, cuda), t_bf16(sh, cuda))
        q8, s8 = ops.norm_quant_e4m3(*args, length=length)
        q4, s4 = ops.norm_quant(*args, length=length)
        assert np.array_equal(q8.cpu().numpy(), e4m3_bytes(q4.cpu().numpy()))
        assert np.array_equal(bits(s8), bits(s4))


def test_swiglu_and_residual_e4m3_equal_packed(cuda):
    from k2b import ops

    M, K, F = 300, 1024, 768
    a, sa = packed_act(M, K, 21)
    wg, swg = packed_weight(F, K, 22)
    wu, swu = packed_weight(F, K, 23)
    Wg = ops.prepare_weight(t_u8(wg, cuda), t_f16(swg, cuda))
    Wu = ops.prepare_weight(t_u8(wu, cuda), t_f16(swu, cuda))
    a8 = t_u8(e4m3_bytes(a), cuda)
    h8, hs8 = ops.swiglu_quant_e4m3(a8, t_f16(sa, cuda), Wg, Wu)
    h4, hs4 = ops.swiglu_quant(t_u8(a, cuda), t_f16(sa, cuda), Wg, Wu)
    assert np.array_equal(h8.cpu().numpy(), e4m3_bytes(h4.cpu().numpy())) and np.array_equal(bits(hs8), bits(hs4))
    wd, swd = packed_weight(K, F, 24)
    Wd = ops.prepare_weight(t_u8(wd, cuda), t_f16(swd, cuda))
    rng = np.random.default_rng(25)
    gate = t_bf16(O.bf16_bits(rng.normal(0, 0.1, (2, K)).astype(np.float32)), cuda)
    resid = t_bf16(O.bf16_bits(rng.standard_normal((M, K)).astype(np.float32)), cuda)
    r8 = ops.gated_residual_e4m3(h8, hs8, Wd, gate, resid, length=M // 2)
    r4 = ops.gated_residual(h4, hs4, Wd, gate, resid, length=M // 2)
    assert np.array_equal(bits(r8), bits(r4))


def test_qkv_e4m3_equals_packed(cuda):
    from k2b import ops
    from k2b.model import rope_positions, rope_table

    M, K = 2 * 150, 512
    a, sa = packed_act(M, K, 31)
    W = {}
    for i, (name, n) in enumerate((("q", 512), ("k", 256), ("v", 256), ("g", 512))):
        wq, ws = packed_weight(n, K, 32 + i)
        W[name] = ops.prepare_weight(t_u8(wq, cuda), t_f16(ws, cuda))
    rng = np.random.default_rng(33)
    nq = t_f32(rng.uniform(-0.1, 0.1, 128).astype(np.float32), cuda)
    nk = t_f32(rng.uniform(-0.1, 0.1, 128).astype(np.float32), cuda)
    freqs = rope_table(rope_positions(6, 12, 12), (64, 64), 10000.0).to(cuda)
    o8 = ops.qkv_e4m3(t_u8(e4m3_bytes(a), cuda), t_f16(sa, cuda), W["q"], W["k"], W["v"], nq, nk, freqs, length=150,
                      wg=W["g"])
    o4 = ops.qkv(t_u8(a, cuda), t_f16(sa, cuda), W["q"], W["k"], W["v"], nq, nk, freqs, length=150, wg=W["g"])
    for x8, x4 in zip(o8, o4):
        assert np.array_equal(bits(x8), bits(x4))


def test_attention_quant_e4m3_same_codes(cuda):
    from k2b import ops

    rng = np.random.default_rng(41)
    q = t_bf16(O.bf16_bits(rng.standard_normal((2, 4, 333, 128)).astype(np.float32)), cuda)
    k = t_bf16(O.bf16_bits(rng.standard_normal((2, 2, 333, 128)).astype(np.float32)), cuda)
    v = t_bf16(O.bf16_bits(rng.standard_normal((2, 2, 333, 128)).astype(np.float32)), cuda)
    q8, s8 = ops.attention_quant_e4m3(q, k, v)
    q4, s4 = ops.attention_quant(q, k, v)
    assert np.array_equal(q8.cpu().numpy(), e4m3_bytes(q4.cpu().numpy())) and np.array_equal(bits(s8), bits(s4))
