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
