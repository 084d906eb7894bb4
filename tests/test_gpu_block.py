"""Block chain on the B200: native block loop == per-op loop (bit-exact), and
both within tolerance of the CPU oracle chain (max abs <= 2e-2 relative to the
stream's scale is not meaningful for a residual stream, so the check is
cosine >= 0.999 per block output plus a bounded max abs error)."""
import numpy as np
import pytest

import oracle as O
from _helpers import TOL_COS, bits, cosine, oracle_block, t_bf16

pytestmark = pytest.mark.gpu


def _small_model(cuda, batch, length, blocks=2):
    from k2b.model import Krea2Blocks, ModelConfig, rope_positions, rope_table, synthetic_blocks

    cfg = ModelConfig(hidden=512, heads=4, kvheads=2, mlp=1024, blocks=blocks)
    bw = synthetic_blocks(cfg, batch, seed=3, device=cuda, keep_packed=True)
    side = 12
    text = length - (length // side) * side
    freqs = rope_table(rope_positions(text, length // side, side), (64, 64), cfg.theta).to(cuda)
    return cfg, bw, freqs, Krea2Blocks(cfg, bw, batch, length, device=cuda)


def _np_block(b):
    from _helpers import bits as tb

    d = {"prenorm": b.prenorm.cpu().numpy(), "postnorm": b.postnorm.cpu().numpy(),
         "qnorm": b.qnorm.cpu().numpy(), "knorm": b.knorm.cpu().numpy(), "mod": tb(b.mod)}
    for n, (q, s) in b.packed.items():
        d[n] = (q.cpu().numpy(), tb(s))
    return d


def test_block_loop_matches_per_op_loop(cuda):
    import torch
    from k2b.model import block_python

    batch, length = 2, 150
    cfg, bw, freqs, model = _small_model(cuda, batch, length)
    rng = np.random.default_rng(0)
    x0 = t_bf16(O.bf16_bits(rng.standard_normal((batch * length, cfg.hidden)).astype(np.float32)), cuda)
    x_native = model.forward_(x0.clone(), freqs)
    x_py = x0.clone()
    for b in bw:
        x_py = block_python(cfg, b, x_py, freqs, batch, length)
    torch.cuda.synchronize()
    assert torch.equal(x_native, x_py)


def test_block_chain_vs_oracle(cuda):
    import torch
    from k2b.model import block_python

    batch, length = 1, 200
    cfg, bw, freqs, _ = _small_model(cuda, batch, length, blocks=2)
    rng = np.random.default_rng(1)
    xb = O.bf16_bits(rng.standard_normal((batch * length, cfg.hidden)).astype(np.float32))
    x = t_bf16(xb, cuda)
    f_np = freqs.cpu().numpy()
    ref = xb
    for b in bw:
        x = block_python(cfg, b, x, freqs, batch, length)
        torch.cuda.synchronize()
        ref = oracle_block(ref, _np_block(b), f_np, batch, length, cfg.heads, cfg.kvheads)
        g = O.bf16_float(bits(x)).astype(np.float64)
        r = O.bf16_float(ref).astype(np.float64)
        cos = cosine(g, r)
        rel = np.abs(g - r).max() / np.abs(r).max()
        assert cos >= TOL_COS, f"cosine {cos}"
        assert rel <= 2e-2, f"max abs err relative to stream max {rel}"


def test_krea2_width_block_vs_oracle(cuda):
    """One block at the Krea2 widths (hidden 6144, 48/12 heads, MLP 16384),
    two latents of 32 tokens (batch modulation rows), stage by stage against the
    oracle on the same inputs: every INT4 / GEMM stage bit-exact, attention within
    2e-2, and the block output (native loop vs the independent oracle chain)
    at cosine >= 0.999.  Over a whole chain one attention rounding difference can
    flip an INT4 code and move single elements by more than 2e-2, so the block
    output is held to the cosine bound (the north_star's per-block criterion)."""
    import torch
    from k2b import ops
    from k2b.model import Krea2Blocks, ModelConfig, rope_positions, rope_table, synthetic_blocks

    batch, length = 2, 32
    cfg = ModelConfig(blocks=1)
    bw = synthetic_blocks(cfg, batch, seed=11, device=cuda, keep_packed=True)
    b = bw[0]
    nb = _np_block(b)
    freqs = rope_table(rope_positions(8, 4, 6), (64, 64), cfg.theta).to(cuda)
    f_np = freqs.cpu().numpy()
    rng = np.random.default_rng(12)
    xb = O.bf16_bits(rng.standard_normal((batch * length, cfg.hidden)).astype(np.float32))
    x = t_bf16(xb, cuda)
    mod = nb["mod"]
    ps, ph, pg, ss, sh, sg = b.mod.unbind(0)

    xq, xs = ops.norm_quant(x, b.prenorm, ps, ph, length=length)
    xq_r, xs_r = O.norm_quant(xb, nb["prenorm"], mod[0], mod[1], length=length)
    assert np.array_equal(xq.cpu().numpy(), xq_r) and np.array_equal(bits(xs), xs_r)
    q, k, v, _ = ops.qkv(xq, xs, b.wq, b.wk, b.wv, b.qnorm, b.knorm, freqs, length=length)
    q_r = O.qk_norm_rope(O.gemm_w4a4(xq_r, xs_r, *nb["wq"]), cfg.heads, nb["qnorm"], 1e-6, f_np, length)
    k_r = O.qk_norm_rope(O.gemm_w4a4(xq_r, xs_r, *nb["wk"]), cfg.kvheads, nb["knorm"], 1e-6, f_np, length)
    v_r = O.bf16_bits(O.gemm_w4a4(xq_r, xs_r, *nb["wv"]))
    assert np.array_equal(bits(q), q_r) and np.array_equal(bits(k), k_r) and np.array_equal(bits(v), v_r)
    shp = lambda t, h: t.view(batch, length, h, 128).transpose(1, 2)
    o = ops.attention(shp(q, cfg.heads), shp(k, cfg.kvheads), shp(v, cfg.kvheads))
    t4 = lambda a, h: a.reshape(batch, length, h, 128).transpose(0, 2, 1, 3)
    o_r = O.attention(t4(q_r, cfg.heads), t4(k_r, cfg.kvheads), t4(v_r, cfg.kvheads)).reshape(batch * length, -1)
    o_g = bits(o).reshape(batch * length, -1)
    assert np.abs(O.bf16_float(o_g) - O.bf16_float(o_r)).max() <= 2e-2
    oq, os_ = ops.attention_quant(shp(q, cfg.heads), shp(k, cfg.kvheads), shp(v, cfg.kvheads))
    oq_r, os_r = O.rotate_quant(o_g)
    assert np.array_equal(oq.cpu().numpy(), oq_r) and np.array_equal(bits(os_), os_r)
    x1 = ops.gated_residual(oq, os_, b.wo, pg.contiguous(), x, length=length)
    x1_r = O.gated_residual(O.gemm_w4a4(oq_r, os_r, *nb["wo"]), mod[2], xb, length)
    assert np.array_equal(bits(x1), x1_r)
    hq_in, hs_in = ops.norm_quant(x1, b.postnorm, ss, sh, length=length)
    hqi_r, hsi_r = O.norm_quant(x1_r, nb["postnorm"], mod[3], mod[4], length=length)
    assert np.array_equal(hq_in.cpu().numpy(), hqi_r) and np.array_equal(bits(hs_in), hsi_r)
    hq, hs = ops.swiglu_quant(hq_in, hs_in, b.wg, b.wu)
    hq_r, hs_r = O.swiglu_quant(O.gemm_w4a4(hqi_r, hsi_r, *nb["wg"]), O.gemm_w4a4(hqi_r, hsi_r, *nb["wu"]))
    assert np.array_equal(hq.cpu().numpy(), hq_r) and np.array_equal(bits(hs), hs_r)
    out = ops.gated_residual(hq, hs, b.wd, sg.contiguous(), x1, length=length)
    out_r = O.gated_residual(O.gemm_w4a4(hq_r, hs_r, *nb["wd"]), mod[5], x1_r, length)
    assert np.array_equal(bits(out), out_r)

    model = Krea2Blocks(cfg, bw, batch, length, device=cuda)
    native = model.forward_(t_bf16(xb, cuda), freqs)
    torch.cuda.synchronize()
    assert torch.equal(native, out)  # the native loop is the per-op chain
    ref = oracle_block(xb, nb, f_np, batch, length, cfg.heads, cfg.kvheads)
    assert cosine(O.bf16_float(bits(native)), O.bf16_float(ref)) >= TOL_COS


def test_config4_shapes_native_loop_equals_per_op(cuda):
    """Two latents of 4224 tokens (128 text + 64x64 image) at the Krea2 widths:
    the native block loop and the per-op chain agree bit for bit."""
    import torch
    from k2b.model import Krea2Blocks, ModelConfig, block_python, rope_positions, rope_table, synthetic_blocks

    batch, length = 2, 4224
    cfg = ModelConfig(blocks=2)
    bw = synthetic_blocks(cfg, batch, seed=13, device=cuda)
    freqs = rope_table(rope_positions(128, 64, 64), (64, 64), cfg.theta).to(cuda)
    model = Krea2Blocks(cfg, bw, batch, length, device=cuda)
    x0 = torch.randn((batch * length, cfg.hidden), device=cuda, generator=torch.Generator(device=cuda).manual_seed(14))
    x0 = x0.to(torch.bfloat16)
    native = model.forward_(x0.clone(), freqs)
    py = x0.clone()
    for b in bw:
        py = block_python(cfg, b, py, freqs, batch, length)
    torch.cuda.synchronize()
    assert torch.equal(native, py)
    assert bool(torch.isfinite(native.float()).all())
