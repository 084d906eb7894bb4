"""CPU oracle: pinned against the reference's own Triton kernels (golden
fixtures from tests/golden/make_golden.py) and checked for the properties
its contract promises.  No GPU."""
import os

import numpy as np
import pytest

import oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_triton.npz")


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLDEN)


# The Triton CPU interpreter converts fp32 -> bf16 by truncation (the GPU
# rounds to nearest even), so the oracle is switched to truncation for these
# comparisons: equality then shows that every operation and rounding point of
# the oracle is the reference kernel's.

def test_norm_mod_matches_reference_triton(gold):
    """RMSNorm + adaLN (forward_kernels.py:13-45): bit-exact."""
    x, y = gold["nm_x"], gold["nm_y"]
    L = int(gold["nm_L"])
    with O.bf16_truncation():
        ours = O.norm_mod(x, gold["nm_w"], gold["nm_scale"], gold["nm_shift"], length=L, batch=x.shape[0] // L,
                          eps=float(gold["nm_eps"]))
    assert np.array_equal(ours, y)


def test_qk_norm_rope_matches_reference_triton(gold):
    """Per-head RMSNorm + adjacent-pair RoPE (forward_kernels.py:64-98): bit-exact
    except where the interpreter's rsqrt and the oracle's correctly rounded
    rsqrt differ in the last fp32 bit."""
    L = gold["qk_q"].shape[1]
    freqs = gold["qk_freqs"].reshape(L, 64, 2, 2)
    for key, w, heads in (("q", gold["qk_qw"], 2), ("k", gold["qk_kw"], 1)):
        p = O.bf16_float(gold[f"qk_{key}"].reshape(L, -1))
        with O.bf16_truncation():
            ours = O.qk_norm_rope(p, heads, w, 1e-6, freqs, L)
        ref = gold[f"qk_{key}o"].reshape(L, -1)
        assert (ours == ref).mean() > 0.99
        assert np.abs(O.bf16_float(ours) - O.bf16_float(ref)).max() <= 2 ** -6


def test_silu_product_matches_reference_triton(gold):
    """SiLU(a) rounded to bf16, times b (forward_kernels.py:48-61)."""
    a = O.bf16_float(gold["am_a"])
    b = O.bf16_float(gold["am_b"])
    with O.bf16_truncation():
        act = O.bf16_round(a / (1.0 + O.exp(-a)))
        ours = O.bf16_bits(act * b)
    assert (ours == gold["am_y"]).mean() > 0.99


@pytest.mark.parametrize("tag", ["plain", "gated"])
def test_attention_matches_reference_triton(gold, tag):
    """Kohaku GQA flash attention (KohakuKernelRouter/attention.py:63-110)."""
    gate = gold["fa_gate"] if tag == "gated" else None
    ours = O.bf16_float(O.attention(gold["fa_q"], gold["fa_k"], gold["fa_v"], gate=gate))
    ref = gold[f"fa_{tag}"]  # fp32 run of the reference kernel (see make_golden.py)
    assert np.abs(ours - ref).max() <= 2e-2
    c = float((ours.ravel().astype(np.float64) @ ref.ravel()) / (np.linalg.norm(ours) * np.linalg.norm(ref)))
    assert c > 0.9999


# --------------------------------------------------------- oracle properties

def test_exp_accuracy():
    x = np.linspace(-87.0, 88.0, 400001, dtype=np.float32)
    y = O.exp(x).astype(np.float64)
    ref = np.exp(x.astype(np.float64))
    ulp = np.abs(y - ref) / np.spacing(ref.astype(np.float32)).astype(np.float64)
    assert ulp.max() <= 2.0
    assert O.exp(np.array([-200.0, 100.0], np.float32)).tolist() == [0.0, float("inf")]


def test_hadamard_is_orthonormal():
    # rotate_quant of a tiny-valued basis would quantise; check the rotation
    # through the norm it preserves: |H x| == |x| and the dequantised codes
    # reconstruct H x within the quantisation step.
    rng = np.random.default_rng(0)
    x = O.bf16_bits(rng.standard_normal((16, 256)).astype(np.float32))
    q, s = O.rotate_quant(x)
    deq = O.dequant(q, s).astype(np.float64)
    xf = O.bf16_float(x).astype(np.float64)
    H = np.array([[1.0]])
    while H.shape[0] < 128:
        H = np.block([[H, H], [H, -H]])
    H /= np.sqrt(128.0)
    rot = np.concatenate([xf[:, i:i + 128] @ H.T for i in (0, 128)], axis=1)
    step = np.repeat(O.f16_float(s), 128, axis=1)
    assert np.all(np.abs(deq - rot) <= 0.5 * step + 1e-6 + np.maximum(0, np.abs(rot) - 7.5 * step))
    np.testing.assert_allclose(np.linalg.norm(rot, axis=1), np.linalg.norm(xf, axis=1), rtol=1e-5)


def test_quant_codes_and_scale_rule():
    rng = np.random.default_rng(1)
    x = O.bf16_bits(rng.standard_normal((8, 128)).astype(np.float32))
    q, s = O.rotate_quant(x)
    lo = (q & 0xF).astype(np.int16)
    hi = (q >> 4).astype(np.int16)
    codes = np.where(np.concatenate([lo, hi], 1) >= 8, np.concatenate([lo, hi], 1) - 16, np.concatenate([lo, hi], 1))
    assert codes.min() >= -8 and codes.max() <= 7
    # the group absmax maps to +-7 (or -8 after fp16 rounding of the scale)
    assert np.all(np.abs(codes).max(axis=1) >= 7)


def test_gemm_matches_float_dequant_product():
    a, sa = O.rotate_quant(O.bf16_bits(np.random.default_rng(2).standard_normal((20, 512)).astype(np.float32)))
    w, sw = O.rotate_quant(O.bf16_bits(np.random.default_rng(3).normal(0, 0.02, (64, 512)).astype(np.float32)))
    p, acc = O.gemm_w4a4(a, sa, w, sw, with_acc=True)
    ref = O.dequant(a, sa).astype(np.float64) @ O.dequant(w, sw).astype(np.float64).T
    np.testing.assert_allclose(p, ref, rtol=1e-5, atol=1e-5 * np.abs(ref).max())
    assert np.abs(acc).max() <= 128 * 64


def test_norm_quant_matches_norm_mod_then_rotate_quant():
    """norm_quant == rotate_quant(norm_mod(x)) (the fused op is the composition)."""
    rng = np.random.default_rng(4)
    x = O.bf16_bits(rng.standard_normal((9, 1024)).astype(np.float32) * 3)
    w = (O.bf16_round(rng.uniform(0.9, 1.1, 1024).astype(np.float32)) - 1).astype(np.float32)
    sc = O.bf16_bits(rng.normal(0, 0.1, (3, 1024)).astype(np.float32))
    sh = O.bf16_bits(rng.normal(0, 0.1, (3, 1024)).astype(np.float32))
    q, s = O.norm_quant(x, w, sc, sh, length=3, batch=3)
    q2, s2 = O.rotate_quant(O.norm_mod(x, w, sc, sh, length=3, batch=3))
    assert np.array_equal(q, q2) and np.array_equal(s, s2)


def test_edge_cases_zero_rows_and_single_row():
    x = np.zeros((1, 512), np.uint16)
    q, s = O.rotate_quant(x)
    assert np.all(q == 0) and np.all(s == 0)
    w = np.zeros(512, np.float32)
    z = np.zeros((1, 512), np.uint16)
    q, s = O.norm_quant(x, w, z, z)
    assert np.all(q == 0)
