"""LoRA bypass deltas fused into the projection epilogue.

The reference composes value + T(T(x down^T) up^T) * s after its native
projection (graph_ops.py:246-249).  Here t = T(x down^T) is the same library
GEMM and the up-projection runs in the W4A4 GEMM's epilogue in fp32, so the
fused result equals the composition except where the two fp32 summation
orders of t up^T round T(d) differently (a last-bit difference on a small
fraction of elements), which the tests bound explicitly."""
import numpy as np
import pytest

import oracle as O
from _helpers import bits, packed_act, packed_weight, t_bf16, t_f16, t_u8

pytestmark = pytest.mark.gpu

M, K, N, R = 300, 1024, 384, 24


def _bf(a):
    return O.bf16_float(O.bf16_bits(np.asarray(a, np.float32)))


def _factors(n, k, r, seed, scale=0.05):
    rng = np.random.default_rng(seed)
    up = O.bf16_bits(rng.normal(0, scale, (n, r)).astype(np.float32))
    t = O.bf16_bits(rng.normal(0, 1, (M, r)).astype(np.float32))
    return t, up


def _lora_ref(p, t, up, s):
    """T(T(p) + T(T(t up^T) * s)) in the oracle's arithmetic."""
    d = O.bf16_float(t).astype(np.float64) @ O.bf16_float(up).astype(np.float64).T
    dt = _bf(d.astype(np.float32))
    return O.bf16_bits((_bf(p) + _bf((dt * np.float32(s)).astype(np.float32))).astype(np.float32))


def _agree(got, ref, frac=0.99):
    g, r = O.bf16_float(got), O.bf16_float(ref)
    same = float((got == ref).mean())
    assert same >= frac, same
    # a differing T(d) moves the sum by at most one bf16 step of d * s plus the final rounding
    assert float(np.abs(g - r).max()) <= 2e-2 * max(1.0, float(np.abs(r).max()))


def test_lora_gemm_group128_and_gated(cuda):
    import torch
    from k2b import ops

    a, sa = packed_act(M, K, 1)
    wq, ws = packed_weight(N, K, 2)
    W = ops.prepare_weight(t_u8(wq, cuda), t_f16(ws, cuda))
    t, up = _factors(N, K, R + 8, 3)  # r = 32
    p = O.gemm_w4a4(a, sa, wq, ws)
    out = ops.lora_gemm(t_u8(a, cuda), t_f16(sa, cuda), W, t_bf16(t, cuda), t_bf16(up, cuda), 0.75)
    torch.cuda.synchronize()
    ref = _lora_ref(p, t, up, 0.75)
    _agree(bits(out), ref)
    # gated residual over 3 latents of 100 rows
    rng = np.random.default_rng(4)
    gate = O.bf16_bits(rng.normal(0, 0.5, (3, N)).astype(np.float32))
    resid = O.bf16_bits(rng.normal(0, 1, (M, N)).astype(np.float32))
    o2 = ops.lora_gemm(t_u8(a, cuda), t_f16(sa, cuda), W, t_bf16(t, cuda), t_bf16(up, cuda), 0.75,
                       t_bf16(gate, cuda), t_bf16(resid, cuda), length=100)
    torch.cuda.synchronize()
    _agree(bits(o2), O.gated_residual(O.bf16_float(ref), gate, resid, 100))


def test_lora_swiglu_group128(cuda):
    import torch
    from k2b import ops

    a, sa = packed_act(M, K, 5)
    gq, gs = packed_weight(N, K, 6)
    uq, us = packed_weight(N, K, 7)
    Wg = ops.prepare_weight(t_u8(gq, cuda), t_f16(gs, cuda))
    Wu = ops.prepare_weight(t_u8(uq, cuda), t_f16(us, cuda))
    tg, upg = _factors(N, K, 16, 8)
    tu, upu = _factors(N, K, 8, 9)
    pg, pu = O.gemm_w4a4(a, sa, gq, gs), O.gemm_w4a4(a, sa, uq, us)
    for lg, lu in (((tg, upg, 0.5), (tu, upu, 1.25)), ((tg, upg, 0.5), None), (None, (tu, upu, 1.25))):
        dev = lambda lo: None if lo is None else (t_bf16(lo[0], cuda), t_bf16(lo[1], cuda), lo[2])
        h = ops.lora_swiglu(t_u8(a, cuda), t_f16(sa, cuda), Wg, Wu, dev(lg), dev(lu))
        torch.cuda.synchronize()
        g2 = pg if lg is None else O.bf16_float(_lora_ref(pg, *lg))
        u2 = pu if lu is None else O.bf16_float(_lora_ref(pu, *lu))
        _agree(bits(h), O.swiglu_quant(g2, u2, want_h=True)[2])


def test_lora_gemm_reference_contract_with_bias(cuda):
    import torch
    from k2b import ref_ops

    rng = np.random.default_rng(10)
    x = O.bf16_bits(rng.standard_normal((M, K)).astype(np.float32))
    q, xs = O.ref_quant(x, group=64)
    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    ws = (np.abs(w).max(axis=1) / 7.0).astype(np.float32)
    codes = np.clip(np.rint(w / ws[:, None]), -8, 7).astype(np.int8)
    packed = ((codes[:, 0::2] & 0xF) | ((codes[:, 1::2] & 0xF) << 4)).astype(np.uint8)
    bias = rng.normal(0, 0.1, N).astype(np.float32)
    t, up = _factors(N, K, 16, 11)
    out = ref_ops.lora_gemm4(t_u8(q, cuda).view(torch.int8), torch.from_numpy(xs).to(cuda),
                             t_u8(packed, cuda).view(torch.int8), torch.from_numpy(ws).to(cuda), t_bf16(t, cuda),
                             t_bf16(up, cuda), 0.3, torch.from_numpy(bias).to(cuda))
    torch.cuda.synchronize()
    p = O.ref_project(O.int4_codes(q), xs, codes, ws, bias)
    _agree(bits(out), _lora_ref(p, t, up, 0.3))


def test_native_ops_apply_loras_like_the_reference(cuda):
    """torch.ops.k2_native over a binding with LoRA factors equals the
    reference's composition around the plain op (graph_ops.py:246-249):
    value + T(T(x down^T) up^T) * s per factor, then residual + gate * value."""
    import torch
    import torch.nn.functional as F
    from k2b import native_ops as Nops
    from k2b import ops

    B, L = 2, 60
    q, s = packed_weight(N, K, 12)
    Nops.add_binding(701, 0, 1, [], [t_u8(q, cuda).view(torch.int8), t_f16(s, cuda)], [], 128, True, 1e-6, [],
                     1.0, torch.empty(0), True)
    g = torch.Generator(device="cpu").manual_seed(13)
    fac = [((torch.randn(N, r, generator=g) * 0.05).to(torch.bfloat16).to(cuda),
            (torch.randn(r, K, generator=g) * 0.05).to(torch.bfloat16).to(cuda), st) for r, st in ((12, 0.5), (8, 2.0))]
    x = (torch.randn(B, L, K, generator=g)).to(torch.bfloat16).to(cuda)
    gate = (torch.randn(B, 1, N, generator=g) * 0.5).to(torch.bfloat16).to(cuda)
    resid = torch.randn(B, L, N, generator=g).to(torch.bfloat16).to(cuda)
    try:
        base = torch.ops.k2_native.managed(x, 701, 0, N)
        for nf in (1, 2):
            Nops.set_loras(701, fac[:nf])
            value = torch.ops.k2_native.managed(x, 701, 0, N)
            gated = torch.ops.k2_native.gated(x, gate, resid, 701)
            ref = base
            for up, down, st in fac[:nf]:
                ref = ref + F.linear(F.linear(x, down), up) * st
            _agree(bits(value), bits(ref))
            _agree(bits(gated), bits(resid + gate * ref))
        # prepared-input ops refuse bindings with factors (x is metadata there)
        a, sa = ops.rotate_quant(x.reshape(B * L, K))
        with pytest.raises(RuntimeError, match="LoRA"):
            torch.ops.k2_native.swiglu_prepared(x, a.view(torch.int8), sa, [701, 701], N)
        Nops.set_loras(701, [])
        assert torch.equal(torch.ops.k2_native.managed(x, 701, 0, N), base)
    finally:
        Nops.release_bindings([701])
