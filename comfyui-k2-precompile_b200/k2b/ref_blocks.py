"""Krea2 blocks in the reference's own data contract (a ConvRot W4A4
checkpoint's arithmetic), on libk2b's byte-operand kernels.

The per-block dataflow is graph_model.block's input-quant chain
(graph_model.py:108-114) as the reference's runtime serves it
(native_runtime.cpp:262-311, 399-475):

    q, s   = norm_quant4(x; ps, ph)               ConvRot group, one fp32 scale per row (codes as e4m3 bytes)
    Q,K,V,G = joint QKV (Q/K RMSNorm + RoPE, V, sigmoid gate)   N = 6144+1536+1536+6144
    o      = GQA attention(Q, K, V) * G            (gate pre-sigmoided)
    x1     = T(x + T(T(proj_o(quant4(o))) * pg))
    q, s   = norm_quant4(x1; ss, sh)
    h      = SwiGLU(gate/up(q))                    bf16 h, as the reference's joint kernel
    out    = T(x1 + T(T(proj_d(quant4(h))) * sg))

Every projection is T(fp32(fp32(acc * xs) * ws)) over all of K with INT4
codes as e4m3 bytes on both sides (exact integer sums), so the results are
those of the packed reference-named exports.  Weights are packed [n, k/2]
checkpoint rows with fp32 per-channel scales, expanded once to code bytes.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List

import torch

from . import ops, ref_ops
from .model import ModelConfig


@dataclass
class RefBlockWeights:
    prenorm: torch.Tensor   # fp32 [hidden] ("w+1" form)
    postnorm: torch.Tensor
    qnorm: torch.Tensor     # fp32 [128]
    knorm: torch.Tensor
    w: dict                 # name -> (packed int8 [n, k/2], fp32 [n], e4m3 codes [n, k])
    mod: torch.Tensor       # bf16 [6, batch, hidden]: ps, ph, pg, ss, sh, sg


def synthetic_ref_blocks(cfg: ModelConfig, batch: int, seed: int = 0, device="cuda") -> List[RefBlockWeights]:
    """Seeded checkpoint-like blocks: uniform INT4 codes with per-channel
    scales ~U(0.5, 1.5) * 0.02 / 7 (a random N(0, 0.02) weight quantised per
    channel has that scale range), norm multipliers ~U(0.9, 1.1), modulation
    ~N(0, 0.1).  The attention gate projection is included (N = 15360 for
    the joint QKV at Krea2 widths)."""
    gen = torch.Generator(device=device).manual_seed(seed + 4099)
    H, D = cfg.hidden, 128
    shapes = {"wq": (cfg.heads * D, H), "wk": (cfg.kvheads * D, H), "wv": (cfg.kvheads * D, H),
              "wg_attn": (cfg.heads * D, H), "wo": (H, cfg.heads * D), "wg": (cfg.mlp, H), "wu": (cfg.mlp, H),
              "wd": (H, cfg.mlp)}

    def norm_w(n):
        w_eff = (torch.rand(n, generator=gen, device=device) * 0.2 + 0.9).to(torch.bfloat16)
        return (w_eff.to(torch.float32) - 1.0).contiguous()

    blocks = []
    for _ in range(cfg.blocks):
        w = {}
        for name, (n, k) in shapes.items():
            packed = torch.randint(-128, 128, (n, k // 2), generator=gen, device=device, dtype=torch.int8)
            scale = (torch.rand(n, generator=gen, device=device) + 0.5) * (0.02 / 7.0)
            w[name] = (packed, scale, ref_ops.codes_e4m3(packed))
        mod = (torch.randn((6, batch, H), generator=gen, device=device) * 0.1).to(torch.bfloat16).contiguous()
        blocks.append(RefBlockWeights(norm_w(H), norm_w(H), norm_w(D), norm_w(D), w, mod))
    return blocks


def ref_block(cfg: ModelConfig, b: RefBlockWeights, x: torch.Tensor, freqs: torch.Tensor, batch: int, length: int,
              group: int = 256) -> torch.Tensor:
    """One block of the reference contract; x bf16 [batch*length, hidden]."""
    ps, ph, pg, ss, sh, sg = b.mod.unbind(0)
    rows = batch * length
    q, s = ref_ops.norm_quant4_e4m3(x, b.prenorm, ps, ph, length=length, eps=cfg.eps, group=group)
    names = ("wq", "wk", "wv", "wg_attn")
    Q, K, V, G = ref_ops.qkv8(q, s.reshape(-1), [b.w[n][2] for n in names],
                              [b.w[n][1] for n in names], b.qnorm, b.knorm, freqs, length=length,
                              eps_q=cfg.qk_eps, eps_k=cfg.qk_eps)
    view = lambda t, h: t.view(batch, length, h, 128).transpose(1, 2)
    o = ops.attention(view(Q, cfg.heads), view(K, cfg.kvheads), view(V, cfg.kvheads),
                      gate=G.view(batch, length, -1), gate_is_sigmoid=True)
    qo, so = ref_ops.quant4_e4m3(o.view(rows, -1), group)
    x1 = ref_ops.gated_residual8(qo, so.reshape(-1), b.w["wo"][2], b.w["wo"][1], pg.contiguous(), x, length=length)
    q, s = ref_ops.norm_quant4_e4m3(x1, b.postnorm, ss, sh, length=length, eps=cfg.eps, group=group)
    h = ref_ops.swiglu8(q, s.reshape(-1), b.w["wg"][2], b.w["wg"][1], b.w["wu"][2], b.w["wu"][1])
    qh, sh_ = ref_ops.quant4_e4m3(h, group)
    return ref_ops.gated_residual8(qh, sh_.reshape(-1), b.w["wd"][2], b.w["wd"][1], sg.contiguous(), x1,
                                   length=length)


def ref_forward(cfg: ModelConfig, blocks: List[RefBlockWeights], x: torch.Tensor, freqs: torch.Tensor, batch: int,
                length: int, group: int = 256) -> torch.Tensor:
    for b in blocks:
        x = ref_block(cfg, b, x, freqs, batch, length, group)
    return x
