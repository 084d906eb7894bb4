"""tcgen05 GQA flash attention vs the CPU oracle (tolerance: max abs <= 2e-2, cosine >= 0.999)."""
import numpy as np
import pytest

import oracle as O
from _helpers import TOL_ABS, TOL_COS, bits, cosine, t_bf16

pytestmark = pytest.mark.gpu


def _qkv_bits(B, Hq, Hkv, L, Lk, seed, rms=True):
    rng = np.random.default_rng(seed)

    def mk(shape):
        x = rng.standard_normal(shape).astype(np.float32)
        if rms:  # config 2: Q/K pre-RMS-normalised
            x = x / np.sqrt((x * x).mean(-1, keepdims=True))
        return O.bf16_bits(x)

    return mk((B, Hq, L, 128)), mk((B, Hkv, Lk, 128)), O.bf16_bits(rng.standard_normal((B, Hkv, Lk, 128)).astype(np.float32))


def _check(got_bits, ref_bits):
    g = O.bf16_float(got_bits).astype(np.float64)
    r = O.bf16_float(ref_bits).astype(np.float64)
    err = np.abs(g - r).max()
    cos = cosine(g, r)
    assert err <= TOL_ABS, f"max abs err {err}"
    assert cos >= TOL_COS, f"cosine {cos}"


@pytest.mark.parametrize("B,Hq,Hkv,L", [(1, 2, 1, 128), (1, 4, 2, 300), (2, 4, 1, 257), (1, 8, 2, 1000)])
def test_attention_small(cuda, B, Hq, Hkv, L):
    import torch
    from k2b import ops

    q, k, v = _qkv_bits(B, Hq, Hkv, L, L, B * 100 + L)
    out = ops.attention(t_bf16(q, cuda), t_bf16(k, cuda), t_bf16(v, cuda))
    torch.cuda.synchronize()
    _check(bits(out), O.attention(q, k, v))


@pytest.mark.parametrize("B,Hq,Hkv,L,Lk", [(1, 4, 4, 300, 300), (2, 3, 1, 129, 129), (7, 2, 2, 40, 40),
                                          (1, 20, 20, 98, 98), (1, 6, 2, 257, 500)])
def test_attention_odd_group(cuda, B, Hq, Hkv, L, Lk):
    """Odd GQA groups (group 1 is the text-fusion blocks' H20/KV20): each CTA
    pairs two Q tiles of one head on every K/V tile."""
    import torch
    from k2b import ops

    q, k, v = _qkv_bits(B, Hq, Hkv, L, Lk, 40 + Hq + L)
    rng = np.random.default_rng(41)
    gate = O.bf16_bits(rng.normal(0, 1, (B, L, Hq * 128)).astype(np.float32))
    out = ops.attention(t_bf16(q, cuda), t_bf16(k, cuda), t_bf16(v, cuda), gate=t_bf16(gate, cuda),
                        gate_is_sigmoid=False)
    torch.cuda.synchronize()
    _check(bits(out), O.attention(q, k, v, gate=gate, gate_is_sigmoid=False))


def test_attention_cross_length_and_gate(cuda):
    import torch
    from k2b import ops

    B, Hq, Hkv, L, Lk = 1, 4, 2, 200, 333
    q, k, v = _qkv_bits(B, Hq, Hkv, L, Lk, 5)
    rng = np.random.default_rng(6)
    gate = O.bf16_bits(rng.normal(0, 1, (B, L, Hq * 128)).astype(np.float32))
    for sig in (True, False):
        out = ops.attention(t_bf16(q, cuda), t_bf16(k, cuda), t_bf16(v, cuda), gate=t_bf16(gate, cuda),
                            gate_is_sigmoid=sig)
        torch.cuda.synchronize()
        _check(bits(out), O.attention(q, k, v, gate=gate, gate_is_sigmoid=sig))


def test_attention_token_major_strides(cuda):
    """Q/K/V as views of token-major [B, L, H*D] buffers (the QKV GEMM's output layout)."""
    import torch
    from k2b import ops

    B, Hq, Hkv, L = 2, 4, 2, 190
    q, k, v = _qkv_bits(B, Hq, Hkv, L, L, 8)
    tm = lambda a: np.ascontiguousarray(a.transpose(0, 2, 1, 3)).reshape(B, L, -1)
    qt = t_bf16(tm(q), cuda).view(B, L, Hq, 128).transpose(1, 2)
    kt = t_bf16(tm(k), cuda).view(B, L, Hkv, 128).transpose(1, 2)
    vt = t_bf16(tm(v), cuda).view(B, L, Hkv, 128).transpose(1, 2)
    out = ops.attention(qt, kt, vt)
    torch.cuda.synchronize()
    _check(bits(out), O.attention(q, k, v))


def test_attention_quant_matches_rotate_quant(cuda):
    """The fused INT4 store equals rotate_quant of the bf16 output bit for bit."""
    import torch
    from k2b import ops

    B, Hq, Hkv, L = 1, 4, 2, 260
    q, k, v = _qkv_bits(B, Hq, Hkv, L, L, 12)
    qt, kt, vt = t_bf16(q, cuda), t_bf16(k, cuda), t_bf16(v, cuda)
    out = ops.attention(qt, kt, vt)
    oq, os_ = ops.attention_quant(qt, kt, vt)
    torch.cuda.synchronize()
    rq, rs = O.rotate_quant(bits(out).reshape(B * L, Hq * 128))
    assert np.array_equal(bits(os_), rs)
    assert np.array_equal(oq.cpu().numpy(), rq)


def test_attention_config2_sampled_rows(cuda):
    """Config 2: Q [1,48,4050,128], K/V [1,12,4050,128]; oracle on 48 sampled query rows."""
    import torch
    from k2b import ops

    q, k, v = _qkv_bits(1, 48, 12, 4050, 4050, 2)
    out = ops.attention(t_bf16(q, cuda), t_bf16(k, cuda), t_bf16(v, cuda))
    torch.cuda.synchronize()
    rows = np.unique(np.concatenate([[0, 127, 128, 3967, 3968, 4049],
                                     np.random.default_rng(1).choice(4050, 42, replace=False)]))
    ref = O.attention(q, k, v, rows=rows)
    _check(bits(out)[:, rows], ref)
