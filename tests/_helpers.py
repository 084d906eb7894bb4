"""Seeded inputs and oracle chains shared by the parity tests."""
from __future__ import annotations

import numpy as np

import oracle as O

TOL_ABS = 2e-2   # north_star: max abs error <= 2e-2 on bf16 outputs
TOL_COS = 0.999  # north_star: cosine >= 0.999 per block output


def bf16_x(rows, K, seed, outliers=True, scale=1.0):
    """bf16 bits of N(0,1)*scale with 1% of channels x20 (config 0)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, K)).astype(np.float32) * scale
    if outliers:
        ch = rng.choice(K, max(1, K // 100), replace=False)
        x[:, ch] *= 20.0
    return O.bf16_bits(x)


def norm_inputs(K, nb, seed):
    rng = np.random.default_rng(seed)
    w_eff = O.bf16_round(rng.uniform(0.9, 1.1, K).astype(np.float32))
    w = (w_eff - np.float32(1.0)).astype(np.float32)
    scale = O.bf16_bits(rng.normal(0, 0.1, (nb, K)).astype(np.float32))
    shift = O.bf16_bits(rng.normal(0, 0.1, (nb, K)).astype(np.float32))
    return w, scale, shift


def packed_act(M, K, seed):
    return O.rotate_quant(bf16_x(M, K, seed, outliers=False))


def packed_weight(N, K, seed, std=0.02):
    rng = np.random.default_rng(seed)
    return O.rotate_quant(O.bf16_bits(rng.normal(0, std, (N, K)).astype(np.float32)))


def cosine(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30))


# ---------------------------------------------------------------- torch glue

def t_bf16(bits, device):
    import torch

    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(device)


def t_f16(bits, device):
    import torch

    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.float16).to(device)


def t_u8(a, device):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def t_f32(a, device):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(device)


def bits(t):
    """CUDA bf16/fp16 tensor -> uint16 numpy bits."""
    import torch

    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


# ------------------------------------------------------ oracle block chain

def oracle_block(x_bits, blk, freqs, batch, length, heads, kvheads, eps=1e-6, qk_eps=1e-6):
    """One block of graph_model.block's quant chain on the CPU oracle.
    blk: dict of numpy arrays {prenorm, postnorm, qnorm, knorm, mod [6,B,H],
    wq/wk/wv/wo/wg/wu/wd: (packed, scales)}."""
    H = x_bits.shape[1]
    rows = x_bits.shape[0]
    mod = blk["mod"]
    xq, xs = O.norm_quant(x_bits, blk["prenorm"], mod[0], mod[1], length=length, eps=eps)
    pq = O.gemm_w4a4(xq, xs, *blk["wq"])
    pk = O.gemm_w4a4(xq, xs, *blk["wk"])
    pv = O.gemm_w4a4(xq, xs, *blk["wv"])
    q = O.qk_norm_rope(pq, heads, blk["qnorm"], qk_eps, freqs, length)
    k = O.qk_norm_rope(pk, kvheads, blk["knorm"], qk_eps, freqs, length)
    v = O.bf16_bits(pv)
    q4 = q.reshape(batch, length, heads, 128).transpose(0, 2, 1, 3)
    k4 = k.reshape(batch, length, kvheads, 128).transpose(0, 2, 1, 3)
    v4 = v.reshape(batch, length, kvheads, 128).transpose(0, 2, 1, 3)
    o = O.attention(q4, k4, v4).reshape(rows, heads * 128)
    oq, os_ = O.rotate_quant(o)
    po = O.gemm_w4a4(oq, os_, *blk["wo"])
    x1 = O.gated_residual(po, mod[2], x_bits, length)
    hq_in, hs_in = O.norm_quant(x1, blk["postnorm"], mod[3], mod[4], length=length, eps=eps)
    pg = O.gemm_w4a4(hq_in, hs_in, *blk["wg"])
    pu = O.gemm_w4a4(hq_in, hs_in, *blk["wu"])
    hq, hs = O.swiglu_quant(pg, pu)
    pd = O.gemm_w4a4(hq, hs, *blk["wd"])
    return O.gated_residual(pd, mod[5], x1, length)


def np_block(b):
    """A model.BlockWeights (keep_packed=True) as the numpy dict oracle_block takes."""
    d = {"prenorm": b.prenorm.cpu().numpy(), "postnorm": b.postnorm.cpu().numpy(),
         "qnorm": b.qnorm.cpu().numpy(), "knorm": b.knorm.cpu().numpy(), "mod": bits(b.mod)}
    for n, (q, s) in b.packed.items():
        d[n] = (q.cpu().numpy(), bits(s))
    return d


def stagewise_block(cfg, b, xb, freqs, batch, length, device):
    """Runs one block stage by stage on the GPU (per-op wrappers) and on the CPU
    oracle with the same inputs, asserting every integer stage bit-exact and the
    attention output within TOL_ABS.  Each GPU stage takes the GPU output of the
    stage before it; after attention the oracle continues from the GPU's
    attention output (the only stage with a tolerance), so the later integer
    stages are still compared bit for bit.  Returns (gpu block output bits,
    stats dict)."""
    from k2b import ops

    nb = np_block(b)
    f_np = freqs.cpu().numpy()
    x = t_bf16(xb, device)
    mod = nb["mod"]
    ps, ph, pg, ss, sh, sg = b.mod.unbind(0)
    rows = batch * length
    stats = {}

    xq, xs = ops.norm_quant(x, b.prenorm, ps, ph, length=length)
    xq_r, xs_r = O.norm_quant(xb, nb["prenorm"], mod[0], mod[1], length=length)
    assert np.array_equal(xq.cpu().numpy(), xq_r) and np.array_equal(bits(xs), xs_r), "norm_quant (pre)"
    q, k, v, _ = ops.qkv(xq, xs, b.wq, b.wk, b.wv, b.qnorm, b.knorm, freqs, length=length)
    q_r = O.qk_norm_rope(O.gemm_w4a4(xq_r, xs_r, *nb["wq"]), cfg.heads, nb["qnorm"], cfg.qk_eps, f_np, length)
    assert np.array_equal(bits(q), q_r), "q projection + QK-norm + RoPE"
    k_r = O.qk_norm_rope(O.gemm_w4a4(xq_r, xs_r, *nb["wk"]), cfg.kvheads, nb["knorm"], cfg.qk_eps, f_np, length)
    assert np.array_equal(bits(k), k_r), "k projection + QK-norm + RoPE"
    v_r = O.bf16_bits(O.gemm_w4a4(xq_r, xs_r, *nb["wv"]))
    assert np.array_equal(bits(v), v_r), "v projection"
    shp = lambda t, h: t.view(batch, length, h, 128).transpose(1, 2)
    o = ops.attention(shp(q, cfg.heads), shp(k, cfg.kvheads), shp(v, cfg.kvheads))
    t4 = lambda a, h: a.reshape(batch, length, h, 128).transpose(0, 2, 1, 3)
    o_r = O.attention(t4(q_r, cfg.heads), t4(k_r, cfg.kvheads), t4(v_r, cfg.kvheads)).reshape(rows, -1)
    o_g = bits(o).reshape(rows, -1)
    err = float(np.abs(O.bf16_float(o_g) - O.bf16_float(o_r)).max())
    stats["attention_max_abs"] = err
    stats["attention_cos"] = cosine(O.bf16_float(o_g), O.bf16_float(o_r))
    assert err <= TOL_ABS, f"attention max abs {err}"
    oq, os_ = ops.attention_quant(shp(q, cfg.heads), shp(k, cfg.kvheads), shp(v, cfg.kvheads))
    oq_r, os_r = O.rotate_quant(o_g)
    assert np.array_equal(oq.cpu().numpy(), oq_r) and np.array_equal(bits(os_), os_r), "attention INT4 store"
    x1 = ops.gated_residual(oq, os_, b.wo, pg.contiguous(), x, length=length)
    x1_r = O.gated_residual(O.gemm_w4a4(oq_r, os_r, *nb["wo"]), mod[2], xb, length)
    assert np.array_equal(bits(x1), x1_r), "out projection + gated residual"
    hq_in, hs_in = ops.norm_quant(x1, b.postnorm, ss, sh, length=length)
    hqi_r, hsi_r = O.norm_quant(x1_r, nb["postnorm"], mod[3], mod[4], length=length)
    assert np.array_equal(hq_in.cpu().numpy(), hqi_r) and np.array_equal(bits(hs_in), hsi_r), "norm_quant (post)"
    hq, hs = ops.swiglu_quant(hq_in, hs_in, b.wg, b.wu)
    hq_r, hs_r = O.swiglu_quant(O.gemm_w4a4(hqi_r, hsi_r, *nb["wg"]), O.gemm_w4a4(hqi_r, hsi_r, *nb["wu"]))
    assert np.array_equal(hq.cpu().numpy(), hq_r) and np.array_equal(bits(hs), hs_r), "gate/up + SwiGLU + requant"
    out = ops.gated_residual(hq, hs, b.wd, sg.contiguous(), x1, length=length)
    out_r = O.gated_residual(O.gemm_w4a4(hq_r, hs_r, *nb["wd"]), mod[5], x1_r, length)
    assert np.array_equal(bits(out), out_r), "down projection + gated residual"
    return bits(out), stats


# e4m3 encodings of the INT4 codes -8..7 (index code + 8): the byte container
# of the block loop and of the prepared weights
E4M3 = np.array([0xD0, 0xCE, 0xCC, 0xCA, 0xC8, 0xC4, 0xC0, 0xB8,
                 0x00, 0x38, 0x40, 0x44, 0x48, 0x4A, 0x4C, 0x4E], np.uint8)


def unpack_codes(packed):
    """packed u8 [rows, K/2] -> int codes [rows, K] (low nibble = even column)."""
    p = np.asarray(packed, np.uint8)
    c = np.empty((p.shape[0], p.shape[1] * 2), np.int16)
    c[:, 0::2], c[:, 1::2] = p & 0xF, p >> 4
    return np.where(c >= 8, c - 16, c)


def e4m3_bytes(packed):
    return E4M3[unpack_codes(packed) + 8]
