"""torch.ops.k2_native over bindings registered in the reference's own data
contract: INT4 ConvRot checkpoints (packed [N, K/2] weights, fp32 per-channel
scales, groups 16/64/256), INT8 and FP8 e4m3/e5m2 projections.

The INT4 / INT8 routes are checked bit for bit against the oracle's
restatement of the reference's quantisers and projection
(native_runtime.cpp:262-311); the FP8 routes against the calls the reference
itself makes for them (torch._scaled_mm for e4m3, a bf16 linear of the
dequantised operands for e5m2, native_runtime.cpp:306-311) within the
north_star tolerance, since the fp32 accumulation order of those library
GEMMs is their own."""
import numpy as np
import pytest

import oracle as O
from _helpers import TOL_ABS, TOL_COS, bf16_x, bits, norm_inputs, t_bf16, t_f32

pytestmark = pytest.mark.gpu

B, L, K, H, HK, F = 2, 40, 1024, 4, 2, 512
GROUP = 64


def _int4_weight(n, k, seed):
    """Per-channel INT4 checkpoint weight: packed int8 [n, k/2], fp32 [n],
    integer codes [n, k]."""
    rng = np.random.default_rng(seed)
    w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    ws = (np.abs(w).max(axis=1) / 7.0).astype(np.float32)
    codes = np.clip(np.rint(w / ws[:, None]), -8, 7).astype(np.int8)
    packed = ((codes[:, 0::2] & 0xF) | ((codes[:, 1::2] & 0xF) << 4)).astype(np.uint8)
    return packed.view(np.int8), ws, codes


def _add(N, key, fmt, tensors, group=0, input_scale=None):
    import torch

    N.add_binding(key, 0, fmt, [], tensors, [], group, True, 1e-6, [], 10000.0,
                  torch.empty(0) if input_scale is None else input_scale, True)


@pytest.fixture(scope="module")
def reg(cuda):
    import torch
    from k2b import native_ops as N

    keys = {}
    for i, (name, n, k) in enumerate([("wq", H * 128, K), ("wk", HK * 128, K), ("wv", HK * 128, K),
                                       ("wg", H * 128, K), ("wo", K, H * 128), ("gate", F, K), ("up", F, K)]):
        packed, ws, codes = _int4_weight(n, k, 200 + i)
        _add(N, 200 + i, 1, [torch.from_numpy(packed).to(cuda), t_f32(ws, cuda)], group=GROUP)
        keys[name] = (200 + i, ws, codes)
    w, _, _ = norm_inputs(K, 1, 5)
    rng = np.random.default_rng(11)
    qn = (O.bf16_round(rng.uniform(0.9, 1.1, 128).astype(np.float32)) - 1).astype(np.float32)
    kn = (O.bf16_round(rng.uniform(0.9, 1.1, 128).astype(np.float32)) - 1).astype(np.float32)
    for key, vec in ((220, w), (221, qn), (222, kn)):
        N.add_binding(key, 1, 0, [], [t_f32(vec, cuda)], [], 0, False, 1e-6, [], 10000.0, torch.empty(0), True)
    keys.update(norm=(220, w), qnorm=(221, qn), knorm=(222, kn))
    yield keys
    N.release_bindings([v[0] for v in keys.values()])


def _freqs(cuda):
    from k2b.model import rope_positions, rope_table

    f = rope_table(rope_positions(4, 4, 9), (64, 64), 10000.0)  # [40, 64, 2, 2]
    return f, f.to(cuda).view(1, 1, L, 64, 2, 2)


def _proj(reg, name, codes, xs):
    return O.ref_project(codes, xs, reg[name][2], reg[name][1])


def test_norm_quant_then_prepared_qkv_and_swiglu(cuda, reg):
    import torch

    xb = bf16_x(B * L, K, 1)
    w = reg["norm"][1]
    _, sc, sh = norm_inputs(K, B, 2)
    q, s = torch.ops.k2_native.norm_quant(t_bf16(xb, cuda).view(B, L, K), t_bf16(sc, cuda), t_bf16(sh, cuda),
                                          reg["norm"][0], reg["wq"][0], -1)
    qo, so = O.ref_quant(xb, w, sc, sh, length=L, batch=B, group=GROUP)
    assert q.dtype == torch.int8 and q.shape == (B * L, K // 2) and s.shape == (B * L, 1)
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), qo)
    assert np.array_equal(s.cpu().numpy()[:, 0], so)

    f_np, f = _freqs(cuda)
    x = torch.empty(B, L, K, dtype=torch.bfloat16, device=cuda)
    keys = [reg[n][0] for n in ("wq", "wk", "wv", "wg")]
    oq, ok, ov, og = torch.ops.k2_native.qkv_prepared(x, q, s, f, keys, [reg["qnorm"][0], reg["knorm"][0]], H, HK)
    assert oq.shape == (B, H, L, 128) and ok.shape == (B, HK, L, 128)
    assert ov.shape == (B, L, HK * 128) and og.shape == (B, L, H * 128)
    codes = O.int4_codes(qo)
    P = {n: _proj(reg, n, codes, so) for n in ("wq", "wk", "wv", "wg")}
    fn = f_np.numpy()
    assert np.array_equal(bits(oq.transpose(1, 2).reshape(B * L, -1)),
                          O.qk_norm_rope(P["wq"], H, reg["qnorm"][1], 1e-6, fn, L))
    assert np.array_equal(bits(ok.transpose(1, 2).reshape(B * L, -1)),
                          O.qk_norm_rope(P["wk"], HK, reg["knorm"][1], 1e-6, fn, L))
    assert np.array_equal(bits(ov).reshape(B * L, -1), O.bf16_bits(P["wv"]))
    assert np.array_equal(bits(og).reshape(B * L, -1), O.sigmoid_gate(P["wg"]))
    h = torch.ops.k2_native.swiglu_prepared(x, q, s, [reg["gate"][0], reg["up"][0]], F)
    pg, pu = _proj(reg, "gate", codes, so), _proj(reg, "up", codes, so)
    assert np.array_equal(bits(h).reshape(B * L, F), O.swiglu_quant(pg, pu, want_h=True)[2])


def test_joint_ops_quantise_like_the_reference(cuda, reg):
    import torch

    xb = bf16_x(B * L, K, 3, outliers=False)
    x = t_bf16(xb, cuda).view(B, L, K)
    qo, so = O.ref_quant(xb, group=GROUP)
    codes = O.int4_codes(qo)
    f_np, f = _freqs(cuda)
    keys = [reg[n][0] for n in ("wq", "wk", "wv", "wg")]
    oq, ok, ov, og = torch.ops.k2_native.joint_qkv(x, f, keys, [reg["qnorm"][0], reg["knorm"][0]], H, HK)
    P = {n: _proj(reg, n, codes, so) for n in ("wq", "wk", "wv", "wg")}
    assert np.array_equal(bits(ov).reshape(B * L, -1), O.bf16_bits(P["wv"]))
    assert np.array_equal(bits(og).reshape(B * L, -1), O.sigmoid_gate(P["wg"]))
    assert np.array_equal(bits(oq.transpose(1, 2).reshape(B * L, -1)),
                          O.qk_norm_rope(P["wq"], H, reg["qnorm"][1], 1e-6, f_np.numpy(), L))
    # attention_inputs: the same Q/K/V, the gate as the plain projection T(p)
    # (graph_model.py:42-44 passes gate_is_sigmoid=False for this route)
    aq, ak, av, ag = torch.ops.k2_native.attention_inputs(x, f, keys, [H * 128, HK * 128, HK * 128, H * 128],
                                                          [reg["qnorm"][0], reg["knorm"][0]], H, HK)
    assert torch.equal(aq, oq) and torch.equal(ak, ok) and torch.equal(av, ov)
    assert np.array_equal(bits(ag).reshape(B * L, -1), O.bf16_bits(P["wg"]))
    h = torch.ops.k2_native.joint_swiglu(x, [reg["gate"][0], reg["up"][0]], F)
    pg, pu = _proj(reg, "gate", codes, so), _proj(reg, "up", codes, so)
    assert np.array_equal(bits(h).reshape(B * L, F), O.swiglu_quant(pg, pu, want_h=True)[2])
    outs = torch.ops.k2_native.project_many(x, [reg["wv"][0], reg["wq"][0]], [HK * 128, H * 128])
    assert np.array_equal(bits(outs[0]).reshape(B * L, -1), O.bf16_bits(P["wv"]))
    assert np.array_equal(bits(outs[1]).reshape(B * L, -1), O.bf16_bits(P["wq"]))


def test_gated_residual_per_latent_gate(cuda, reg):
    import torch

    xb = bf16_x(B * L, H * 128, 4, outliers=False)
    rng = np.random.default_rng(5)
    gate = O.bf16_bits(rng.normal(0, 0.5, (B, K)).astype(np.float32))
    resid = bf16_x(B * L, K, 6)
    out = torch.ops.k2_native.gated(t_bf16(xb, cuda).view(B, L, -1), t_bf16(gate, cuda).view(B, 1, K),
                                    t_bf16(resid, cuda).view(B, L, K), reg["wo"][0])
    qo, so = O.ref_quant(xb, group=GROUP)
    p = _proj(reg, "wo", O.int4_codes(qo), so)
    assert np.array_equal(bits(out).reshape(B * L, K), O.gated_residual(p, gate, resid, L))


def test_padded_int4_with_bias(cuda):
    """n and k that are not multiples of 128: zero-padded at registration."""
    import torch
    from k2b import native_ops as N

    n, k = 200, 960
    packed, ws, codes = _int4_weight(n, k, 300)
    bias = np.random.default_rng(301).normal(0, 0.1, n).astype(np.float32)
    _add(N, 310, 1, [torch.from_numpy(packed).to(cuda), t_f32(ws, cuda), t_f32(bias, cuda)], group=GROUP)
    try:
        xb = bf16_x(33, k, 302)
        y = torch.ops.k2_native.managed(t_bf16(xb, cuda).view(1, 33, k), 310, 0, n)
        qo, so = O.ref_quant(xb, group=GROUP)
        assert y.shape == (1, 33, n)
        assert np.array_equal(bits(y).reshape(33, n), O.bf16_bits(O.ref_project(O.int4_codes(qo), so, codes, ws,
                                                                                  bias)))
    finally:
        N.release_bindings([310])


@pytest.mark.parametrize("group,per_channel", [(0, True), (GROUP, False)])
def test_int8_projection_bitexact(cuda, group, per_channel):
    import torch
    from k2b import native_ops as N

    n, k, m = 384, 1024, 150
    rng = np.random.default_rng(400 + group)
    w8 = rng.integers(-127, 128, (n, k), dtype=np.int8)
    ws = rng.uniform(1e-4, 1e-3, n if per_channel else 1).astype(np.float32)
    bias = rng.normal(0, 0.1, n).astype(np.float32)
    _add(N, 410, 2, [torch.from_numpy(w8).to(cuda), t_f32(ws, cuda), t_f32(bias, cuda)], group=group)
    try:
        xb = bf16_x(m, k, 402, outliers=False)
        y = torch.ops.k2_native.managed(t_bf16(xb, cuda).view(1, m, k), 410, 0, n)
        q8, s8 = O.ref_quant(xb, group=group, bits=8)
        bias_x = O.bf16_float(O.bf16_bits(bias))  # the reference hands bias.to(x dtype) to k2_dequant8
        ref = O.ref_project(q8, s8, w8, np.broadcast_to(ws, (n,)), bias_x)
        assert np.array_equal(bits(y).reshape(m, n), O.bf16_bits(ref))
    finally:
        N.release_bindings([410])


@pytest.mark.parametrize("fmt", [3, 4])
def test_fp8_projection_matches_the_references_library_route(cuda, fmt):
    import torch
    from k2b import native_ops as N

    n, k, m = 256, 1024, 200
    dt = torch.float8_e4m3fn if fmt == 3 else torch.float8_e5m2
    g = torch.Generator(device="cpu").manual_seed(500 + fmt)
    w = (torch.randn(n, k, generator=g) * 4).to(dt).to(cuda)
    ws = torch.tensor([0.01], device=cuda)
    bias = (torch.randn(n, generator=g) * 0.1).to(cuda)
    _add(N, 510, fmt, [w, ws, bias])
    try:
        x = (torch.randn(1, m, k, generator=g) * 2).to(torch.bfloat16).to(cuda)
        y = torch.ops.k2_native.managed(x, 510, 0, n)
        x2 = x.reshape(m, k)
        fmax = 448.0 if fmt == 3 else 57344.0
        s = (x2.abs().amax() / fmax).to(torch.float32).clamp_min(torch.finfo(torch.float32).tiny).reshape(1)
        qa = (x2.float() / s).clamp(-fmax, fmax).to(dt)
        if fmt == 3:  # native_runtime.cpp:306
            ref = torch._scaled_mm(qa, w.t(), s.reshape(()), ws.reshape(()), bias.to(torch.bfloat16),
                                   out_dtype=torch.bfloat16)
        else:  # native_runtime.cpp:307-311: both operands dequantised to bf16, then a linear
            ref = torch.nn.functional.linear((qa.float() * s).to(torch.bfloat16), (w.float() * ws).to(torch.bfloat16),
                                             bias.to(torch.bfloat16))
        d = (y.reshape(m, n).float() - ref.float()).abs()
        scale = float(ref.float().abs().max())
        assert float(d.max()) <= TOL_ABS * max(1.0, scale), float(d.max())
        cos = torch.nn.functional.cosine_similarity(y.reshape(1, -1).float(), ref.reshape(1, -1).float())
        assert float(cos) >= TOL_COS
        # exact against the fp32 restatement of the fused route itself
        acc = qa.float() @ w.float().t()
        own = ((acc * s) * ws + bias.to(torch.bfloat16).float()).to(torch.bfloat16)
        assert float((y.reshape(m, n).float() - own.float()).abs().max()) <= 2 ** -6 * max(1.0, scale)
    finally:
        N.release_bindings([510])
