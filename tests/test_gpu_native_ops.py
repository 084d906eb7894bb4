"""torch.ops.k2_native / k2_fullgraph on the B200: the reference's operator
surface over registered bindings, checked against the CPU oracle (bit-exact
where the contract is exact) and against the direct libk2b ops."""
import ctypes

import numpy as np
import pytest

import oracle as O
from _helpers import TOL_ABS, bf16_x, bits, norm_inputs, packed_act, packed_weight, t_bf16, t_f16, t_f32, t_u8

pytestmark = pytest.mark.gpu

B, L, K, H, HK, F = 2, 40, 1024, 4, 2, 1024


@pytest.fixture(scope="module")
def reg(cuda):
    import torch
    from k2b import native_ops as N

    keys = {}
    rng = np.random.default_rng(11)
    for i, (name, n, k) in enumerate([("wq", H * 128, K), ("wk", HK * 128, K), ("wv", HK * 128, K), ("wg", H * 128, K),
                                       ("wo", K, H * 128), ("gate", F, K), ("up", F, K), ("down", K, F)]):
        q, s = packed_weight(n, k, 100 + i)
        N.add_binding(i + 1, 0, 1, [], [t_u8(q, cuda).view(torch.int8), t_f16(s, cuda)], [], 128, True, 1e-6, [],
                      10000.0, torch.empty(0), True)
        keys[name] = (i + 1, q, s)
    w, _, _ = norm_inputs(K, 1, 5)
    N.add_binding(20, 1, 0, [], [t_f32(w, cuda)], [], 128, False, 1e-6, [], 10000.0, torch.empty(0), True)
    qn = (O.bf16_round(rng.uniform(0.9, 1.1, 128).astype(np.float32)) - 1).astype(np.float32)
    kn = (O.bf16_round(rng.uniform(0.9, 1.1, 128).astype(np.float32)) - 1).astype(np.float32)
    N.add_binding(21, 1, 0, [], [t_f32(qn, cuda)], [], 128, False, 1e-6, [], 10000.0, torch.empty(0), True)
    N.add_binding(22, 1, 0, [], [t_f32(kn, cuda)], [], 128, False, 1e-6, [], 10000.0, torch.empty(0), True)
    keys.update(norm=(20, w), qnorm=(21, qn), knorm=(22, kn))
    yield keys
    N.release_bindings([v[0] for v in keys.values()])


def _mod(cuda, seed):
    _, sc, sh = norm_inputs(K, B, seed)
    return sc, sh


def test_norm_quant_op_bitexact(cuda, reg):
    import torch

    xb = bf16_x(B * L, K, 1)
    sc, sh = _mod(cuda, 2)
    q, s = torch.ops.k2_native.norm_quant(t_bf16(xb, cuda).view(B, L, K), t_bf16(sc, cuda), t_bf16(sh, cuda),
                                          reg["norm"][0], reg["wq"][0], -1)
    qo, so = O.norm_quant(xb, reg["norm"][1], sc, sh, length=L, batch=B)
    assert q.dtype == torch.int8 and np.array_equal(q.view(torch.uint8).cpu().numpy(), qo)
    assert np.array_equal(bits(s), so)


def test_norm_mod_op_bitexact(cuda, reg):
    import torch

    xb = bf16_x(B * L, K, 3)
    sc, sh = _mod(cuda, 4)
    y = torch.ops.k2_native.norm_mod(t_bf16(xb, cuda).view(B, L, K), t_bf16(sc, cuda), t_bf16(sh, cuda),
                                     reg["norm"][0], -1)
    assert y.shape == (B, L, K)
    assert np.array_equal(bits(y).reshape(B * L, K), O.norm_mod(xb, reg["norm"][1], sc, sh, length=L, batch=B))


def test_qkv_prepared_layout_and_parity(cuda, reg):
    import torch
    from k2b import ops
    from k2b.model import rope_positions, rope_table

    a, sa = packed_act(B * L, K, 6)
    x = torch.empty(B, L, K, dtype=torch.bfloat16, device=cuda)
    freqs = rope_table(rope_positions(4, 4, 9), (64, 64), 10000.0).to(cuda)
    keys = [reg[n][0] for n in ("wq", "wk", "wv", "wg")]
    q, k, v, g = torch.ops.k2_native.qkv_prepared(x, t_u8(a, cuda).view(torch.int8), t_f16(sa, cuda),
                                                  freqs.view(1, 1, L, 64, 2, 2), keys,
                                                  [reg["qnorm"][0], reg["knorm"][0]], H, HK)
    assert q.shape == (B, H, L, 128) and k.shape == (B, HK, L, 128)
    assert v.shape == (B, L, HK * 128) and g.shape == (B, L, H * 128)
    from k2b import native_ops as N

    ref = ops.qkv(t_u8(a, cuda), t_f16(sa, cuda), *(N._get(kk).weight for kk in keys[:3]),
                  t_f32(reg["qnorm"][1], cuda), t_f32(reg["knorm"][1], cuda), freqs, length=L,
                  wg=N._get(keys[3]).weight)
    assert torch.equal(q.transpose(1, 2).reshape(B * L, -1), ref[0])
    assert torch.equal(k.transpose(1, 2).reshape(B * L, -1), ref[1])
    assert torch.equal(v.reshape(B * L, -1), ref[2]) and torch.equal(g.reshape(B * L, -1), ref[3])


def test_attention_inputs_returns_the_raw_gate(cuda, reg):
    """attention_inputs (native_runtime.cpp:601) normalises Q/K and RoPEs them
    but leaves the gate as the plain projection: the graph passes
    gate_is_sigmoid=False for this route (graph_model.py:42-44)."""
    import torch
    from k2b import native_ops as N
    from k2b import ops
    from k2b.model import rope_positions, rope_table

    x = t_bf16(bf16_x(B * L, K, 16, outliers=False), cuda).view(B, L, K)
    freqs = rope_table(rope_positions(4, 4, 9), (64, 64), 10000.0).to(cuda).view(1, 1, L, 64, 2, 2)
    keys = [reg[n][0] for n in ("wq", "wk", "wv", "wg")]
    norms = [reg["qnorm"][0], reg["knorm"][0]]
    q, k, v, g = torch.ops.k2_native.attention_inputs(x, freqs, keys, [H * 128, HK * 128, HK * 128, H * 128], norms,
                                                      H, HK)
    jq, jk, jv, jg = torch.ops.k2_native.joint_qkv(x, freqs, keys, norms, H, HK)
    assert torch.equal(q, jq) and torch.equal(k, jk) and torch.equal(v, jv)
    a, sa = ops.rotate_quant(x.reshape(B * L, K))
    raw = ops.gemm_bf16(a, sa, N._get(keys[3]).weight)
    assert torch.equal(g.reshape(B * L, -1), raw)
    # joint_qkv's gate is sigmoid(p) of the same projection
    assert float((jg.reshape(B * L, -1).float() - torch.sigmoid(raw.float())).abs().max()) <= 8e-3


def test_swiglu_prepared_bitexact(cuda, reg):
    import torch

    a, sa = packed_act(B * L, K, 7)
    x = torch.empty(B, L, K, dtype=torch.bfloat16, device=cuda)
    h = torch.ops.k2_native.swiglu_prepared(x, t_u8(a, cuda).view(torch.int8), t_f16(sa, cuda),
                                            [reg["gate"][0], reg["up"][0]], F)
    assert h.shape == (B, L, F)
    pg = O.gemm_w4a4(a, sa, reg["gate"][1], reg["gate"][2])
    pu = O.gemm_w4a4(a, sa, reg["up"][1], reg["up"][2])
    _, _, ho = O.swiglu_quant(pg, pu, want_h=True)
    assert np.array_equal(bits(h).reshape(B * L, F), ho)


def test_gated_norm_quant_and_residual_norm(cuda, reg):
    import torch
    from k2b import ops

    xb = bf16_x(B * L, H * 128, 8, outliers=False)
    resid = t_bf16(bf16_x(B * L, K, 9), cuda).view(B, L, K)
    rng = np.random.default_rng(10)
    gate = t_bf16(O.bf16_bits(rng.normal(0, 0.5, (B, 1, K)).astype(np.float32)), cuda)
    sc, sh = _mod(cuda, 12)
    x = t_bf16(xb, cuda).view(B, L, H * 128)
    out, q, s = torch.ops.k2_native.gated_norm_quant(x, gate, resid, t_bf16(sc, cuda), t_bf16(sh, cuda),
                                                     reg["wo"][0], reg["norm"][0], reg["wq"][0], -1)
    from k2b import native_ops as N

    xq, xs = ops.rotate_quant(x.reshape(B * L, -1))
    ref = ops.gated_residual(xq, xs, N._get(reg["wo"][0]).weight, gate.reshape(B, K), resid.reshape(B * L, K),
                             length=L)
    assert torch.equal(out.reshape(B * L, K), ref)
    qo, so = O.norm_quant(bits(ref), reg["norm"][1], sc, sh, length=L, batch=B)
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), qo) and np.array_equal(bits(s), so)
    out2, nrm = torch.ops.k2_native.residual_norm(x, gate, resid, t_bf16(sc, cuda), t_bf16(sh, cuda),
                                                  reg["wo"][0], reg["norm"][0])
    assert torch.equal(out2, out)
    assert np.array_equal(bits(nrm).reshape(B * L, K), O.norm_mod(bits(ref), reg["norm"][1], sc, sh, length=L,
                                                                  batch=B))


def test_kohaku_fa_op(cuda):
    import torch
    from k2b import ops

    rng = np.random.default_rng(13)
    q = t_bf16(O.bf16_bits(rng.standard_normal((1, 4, 70, 128)).astype(np.float32)), cuda)
    k = t_bf16(O.bf16_bits(rng.standard_normal((1, 2, 70, 128)).astype(np.float32)), cuda)
    g = torch.sigmoid(torch.randn(1, 70, 512, device=cuda)).to(torch.bfloat16)
    o = torch.ops.k2_fullgraph.kohaku_fa(q, k, k, None, g, True)
    assert torch.equal(o, ops.attention(q, k, k, gate=g, gate_is_sigmoid=True))
    ref = O.bf16_float(O.attention(bits(q), bits(k), bits(k), gate=bits(g)))
    assert np.abs(O.bf16_float(bits(o)) - ref).max() <= TOL_ABS


def test_elementwise_and_rope_ops(cuda):
    import torch

    a = torch.randn(3, 257, device=cuda).to(torch.bfloat16)
    b = torch.randn(3, 257, device=cuda).to(torch.bfloat16)
    silu = torch.ops.k2_native.activate_mul(a, b, "silu")
    ref = (torch.nn.functional.silu(a.float()).to(torch.bfloat16).float() * b.float())
    assert (silu.float() - ref).abs().max() <= 0.02 * ref.abs().max()
    sig = torch.ops.k2_native.activation(a, "sigmoid")
    assert (sig.float() - torch.sigmoid(a.float())).abs().max() <= 8e-3
    gate = torch.randn(257, device=cuda).to(torch.bfloat16)
    res = torch.ops.k2_native.residual(b, gate, a)
    ref = b.float() + (a.float() * gate.float()).to(torch.bfloat16).float()
    assert (res.float() - ref).abs().max() <= 0.02 * ref.abs().max()
    from k2b.model import rope_positions, rope_table

    f = rope_table(rope_positions(2, 3, 4), (64, 64), 10000.0).to(cuda)  # [14, 64, 2, 2]
    q = torch.randn(2, 3, 14, 128, device=cuda).to(torch.bfloat16)
    k = torch.randn(2, 1, 14, 128, device=cuda).to(torch.bfloat16)
    qo, ko = torch.ops.k2_native.rope(q, k, f.view(1, 1, 14, 64, 2, 2))
    for x, o in ((q, qo), (k, ko)):
        xp = x.float().view(*x.shape[:3], 64, 2)
        r = torch.stack([f[..., 0, 0] * xp[..., 0] + f[..., 0, 1] * xp[..., 1],
                         f[..., 1, 0] * xp[..., 0] + f[..., 1, 1] * xp[..., 1]], -1).view(x.shape)
        assert (o.float() - r).abs().max() <= 0.02 * r.abs().max()


def test_reference_void_shims(cuda):
    import torch
    from k2b import ops
    from k2b._native import lib

    Lb = lib()
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    xb = bf16_x(16, 512, 14)
    x = t_bf16(xb, cuda)
    q = torch.empty(16, 256, dtype=torch.uint8, device=cuda)
    s = torch.empty(16, 1, dtype=torch.float32, device=cuda)
    Lb.k2b_shim_status(1)
    Lb.k2_quant4(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(s.data_ptr()), 16, 512,
                 64, 2, st)
    torch.cuda.synchronize()
    assert Lb.k2b_shim_status(1) == 0
    qo, so = O.ref_quant(xb, group=64)
    assert np.array_equal(q.cpu().numpy(), qo) and np.array_equal(s.cpu().numpy()[:, 0], so)
    w, _, _ = norm_inputs(512, 1, 15)
    y = torch.empty_like(x)
    wt = t_f32(w, cuda)  # held across the launch
    Lb.k2_norm(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(wt.data_ptr()), None, None,
               ctypes.c_void_p(y.data_ptr()), 16, 512, 16, -1, 1, ctypes.c_float(1e-6), 2, st)
    torch.cuda.synchronize()
    assert Lb.k2b_shim_status(1) == 0
    assert torch.equal(y, ops.norm_mod(x, wt))
