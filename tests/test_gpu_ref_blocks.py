"""A Krea2 block in the reference's own contract (k2b.ref_blocks) against the
oracle's restatement, stage by stage: the quantisers, the projections and
their epilogues bit for bit; attention within the north_star tolerance (each
oracle stage after it starts from the GPU's attention output)."""
import numpy as np
import pytest

import oracle as O
from _helpers import TOL_ABS, bits

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("group", [64, 256])
def test_ref_block_stagewise(cuda, group):
    import torch
    from k2b import ops, ref_ops
    from k2b.model import ModelConfig, rope_positions, rope_table
    from k2b.ref_blocks import ref_block, synthetic_ref_blocks

    cfg = ModelConfig(hidden=512, heads=4, kvheads=2, mlp=1024, blocks=1)
    B, L = 2, 100
    rows = B * L
    blk = synthetic_ref_blocks(cfg, B, seed=3, device=cuda)[0]
    freqs = rope_table(rope_positions(20, 8, 10), (64, 64), 10000.0).to(cuda)
    rng = np.random.default_rng(5)
    xb = O.bf16_bits(rng.standard_normal((rows, cfg.hidden)).astype(np.float32))
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).to(cuda)
    out = ref_block(cfg, blk, x, freqs, B, L, group=group)

    m = {k: bits(v) for k, v in zip(("ps", "ph", "pg", "ss", "sh", "sg"), blk.mod.unbind(0))}
    W = {n: (O.int4_codes(v[0].view(torch.uint8).cpu().numpy()), v[1].cpu().numpy()) for n, v in blk.w.items()}
    fn = freqs.cpu().numpy()
    # stage 1: norm + modulation + ConvRot + per-row INT4 (GPU result checked bit for bit)
    q, s = ref_ops.norm_quant4(x, blk.prenorm, blk.mod[0], blk.mod[1], length=L, group=group)
    q_r, s_r = O.ref_quant(xb, blk.prenorm.cpu().numpy(), m["ps"], m["ph"], length=L, batch=B, group=group)
    assert np.array_equal(q.view(torch.uint8).cpu().numpy(), q_r) and np.array_equal(s.cpu().numpy()[:, 0], s_r)
    codes = O.int4_codes(q_r)
    P = {n: O.ref_project(codes, s_r, *W[n]) for n in ("wq", "wk", "wv", "wg_attn")}
    Q = O.qk_norm_rope(P["wq"], cfg.heads, blk.qnorm.cpu().numpy(), cfg.qk_eps, fn, L)
    K = O.qk_norm_rope(P["wk"], cfg.kvheads, blk.knorm.cpu().numpy(), cfg.qk_eps, fn, L)
    V = O.bf16_bits(P["wv"])
    G = O.sigmoid_gate(P["wg_attn"])
    names = ("wq", "wk", "wv", "wg_attn")
    got = ref_ops.qkv8(ref_ops.codes_e4m3(q), s.reshape(-1), [blk.w[n][2] for n in names],
                       [blk.w[n][1] for n in names], blk.qnorm, blk.knorm, freqs, length=L)
    for g, r in zip(got, (Q, K, V, G)):
        assert np.array_equal(bits(g), r)
    t4 = lambda a, h: a.reshape(B, L, h, 128).transpose(0, 2, 1, 3)
    o_r = O.attention(t4(Q, cfg.heads), t4(K, cfg.kvheads), t4(V, cfg.kvheads),
                      gate=G.reshape(B, L, -1)).reshape(rows, -1)
    view = lambda t, h: t.view(B, L, h, 128).transpose(1, 2)
    o = ops.attention(view(got[0], cfg.heads), view(got[1], cfg.kvheads), view(got[2], cfg.kvheads),
                      gate=got[3].view(B, L, -1), gate_is_sigmoid=True)
    o_g = bits(o).reshape(rows, -1)
    assert float(np.abs(O.bf16_float(o_g) - O.bf16_float(o_r)).max()) <= TOL_ABS
    # the rest from the GPU's attention output
    qo, so = O.ref_quant(o_g, group=group)
    x1 = O.gated_residual(O.ref_project(O.int4_codes(qo), so, *W["wo"]), m["pg"], xb, L)
    q2, s2 = O.ref_quant(x1, blk.postnorm.cpu().numpy(), m["ss"], m["sh"], length=L, batch=B, group=group)
    c2 = O.int4_codes(q2)
    h = O.swiglu_quant(O.ref_project(c2, s2, *W["wg"]), O.ref_project(c2, s2, *W["wu"]), want_h=True)[2]
    qh, sh = O.ref_quant(h, group=group)
    out_r = O.gated_residual(O.ref_project(O.int4_codes(qh), sh, *W["wd"]), m["sg"], x1, L)
    assert np.array_equal(bits(out), out_r)
