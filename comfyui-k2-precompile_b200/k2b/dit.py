"""The whole Krea2 DiT forward around the W4A4 block stack.

The call order is graph_model.dit (graph_model.py:202-305) with its norm
chain:

    img   = first(patchify(x))                              (:212, 233)
    t     = tmlp(timestep(timesteps, tdim))                 (:234; native_runtime.cpp:513)
    tvec  = tproj(t)                                        (:235)
    ctx   = txtmlp(txtfusion(context))                      (:239-240)
    x     = cat(ctx, img); freqs = EmbedND(pos)             (:242-254; txt positions 0)
    x     = blocks(x), block i modulated by tvec + lin_i    (:259-295; DoubleSharedModulation,
                                                             native_runtime.cpp:506, 6 chunks)
    out   = last.linear(norm_mod(x; t + last_lin))          (:159-163; SimpleModulation,
                                                             native_runtime.cpp:505, 2 chunks)
    image = unpatchify(out[:, txt:txt + img])               (:299-302)

Everything that holds the arithmetic is this library's kernels: the 28 W4A4
blocks run the native block loop, the text-fusion blocks run the same W4A4
ops (norm_quant, the joint QKV with QK-norm and the sigmoid gate, GQA
attention at group 1, the gated residuals, SwiGLU + requant), the final
RMSNorm + modulation is k2b_norm_mod.  The small plain linears around them
(``first``, the timestep MLP, ``tproj``, ``txtmlp``, ``last.linear``) are
format-0 projections, which the reference also runs as plain linears
(native_runtime.cpp:288), here cuBLAS through torch.  The final norm + modulation
is applied to the whole stream and the text rows are dropped afterwards, as
graph_model.py:296-299 does.

ComfyUI's krea2 module (comfy.ldm.krea2.model) is not part of the reference
and is not restated: the inner layout of its text-fusion stage, the timestep
MLP and the patch embedding are not visible there.  This module fixes them
as follows, and the parity tests check this composition, not ComfyUI's:
text-fusion block = x + attn(rmsnorm(x)), then x + swiglu(rmsnorm(x)), the
attention being graph_model.attention's (QK RMSNorm, sigmoid gate, no RoPE);
tmlp = Linear, GELU(tanh) (managed kind 5), Linear; tproj = Linear to 6
modulation chunks; patches are 'b c (h ph) (w pw) -> b (h w) (c ph pw)', the
inverse of graph_model.py:300-301.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn.functional as F

from . import ops
from .model import BlockWeights, Krea2Blocks, ModelConfig, quantize_weight, rope_table, synthetic_blocks
from .ops import PreparedWeight


@dataclass
class DiTConfig:
    """Widths of the W4A4 text-fusion stage (txtdim, txt_heads * 128,
    txt_mlp) are multiples of 512, as for the block stack: the rotation +
    quantisation kernels tile a row in 512-column steps."""

    core: ModelConfig = field(default_factory=ModelConfig)
    channels: int = 16
    patch: int = 2
    tdim: int = 256
    txtdim: int = 2560
    txt_heads: int = 20
    txt_kvheads: int = 20
    txt_mlp: int = 7168
    txt_layers: int = 4
    axes: Tuple[int, int] = (64, 64)

    @property
    def patch_dim(self) -> int:
        return self.channels * self.patch * self.patch


@dataclass
class TextBlockWeights:
    norm1: torch.Tensor  # fp32 [txtdim] ("w+1" form)
    norm2: torch.Tensor
    qnorm: torch.Tensor  # fp32 [128]
    knorm: torch.Tensor
    wq: PreparedWeight
    wk: PreparedWeight
    wv: PreparedWeight
    wgate: PreparedWeight  # attention gate projection
    wo: PreparedWeight
    wg: PreparedWeight     # SwiGLU gate / up / down
    wu: PreparedWeight
    wd: PreparedWeight
    packed: dict = field(default_factory=dict)


@dataclass
class DiTWeights:
    first: Tuple[torch.Tensor, torch.Tensor]     # bf16 [hidden, patch_dim], [hidden]
    tmlp1: Tuple[torch.Tensor, torch.Tensor]     # [hidden, tdim]
    tmlp2: Tuple[torch.Tensor, torch.Tensor]     # [hidden, hidden]
    tproj: Tuple[torch.Tensor, torch.Tensor]     # [6*hidden, hidden]
    txt: List[TextBlockWeights]
    txtmlp: Tuple[torch.Tensor, torch.Tensor]    # [hidden, txtdim]
    mod_lin: torch.Tensor                        # bf16 [blocks, 6*hidden]
    last_lin: torch.Tensor                       # bf16 [2, hidden]
    last_norm: torch.Tensor                      # fp32 [hidden]
    last: Tuple[torch.Tensor, torch.Tensor]      # [patch_dim, hidden]
    blocks: List[BlockWeights]


def patchify(x: torch.Tensor, p: int) -> Tuple[torch.Tensor, int, int]:
    """[B, C, H, W] -> [B, (H/p)(W/p), C p p]."""
    B, C, H, W = x.shape
    h, w = H // p, W // p
    t = x.reshape(B, C, h, p, w, p).permute(0, 2, 4, 1, 3, 5)
    return t.reshape(B, h * w, C * p * p).contiguous(), h, w


def unpatchify(t: torch.Tensor, h: int, w: int, p: int, c: int) -> torch.Tensor:
    """[B, h w, C p p] -> [B, C, h p, w p] (graph_model.py:300-301)."""
    B = t.shape[0]
    return t.reshape(B, h, w, c, p, p).permute(0, 3, 1, 4, 2, 5).reshape(B, c, h * p, w * p)


def positions(text_tokens: int, h: int, w: int, device=None) -> torch.Tensor:
    """fp32 [text + h w, 2]: text tokens at 0 (graph_model.py:242), image
    token (y, x) at (y, x)."""
    txt = torch.zeros(text_tokens, 2, dtype=torch.float32, device=device)
    y = torch.arange(h, dtype=torch.float32, device=device).repeat_interleave(w)
    x = torch.arange(w, dtype=torch.float32, device=device).repeat(h)
    return torch.cat([txt, torch.stack([y, x], 1)], 0)


def timestep_embedding(t: torch.Tensor, dim: int) -> torch.Tensor:
    """native_runtime.cpp:513: args = fp32(1000 t) * exp(-ln(10^4) i / (dim/2)),
    [cos, sin] (+ a zero column for odd dim), in t's dtype."""
    t = t * 1000.0
    freq = torch.exp(-math.log(10000.0) * torch.arange(dim // 2, dtype=torch.float32, device=t.device) / (dim // 2))
    args = t.to(torch.float32).unsqueeze(-1) * freq.unsqueeze(0)
    out = torch.cat([args.cos(), args.sin()], -1)
    if dim % 2:
        out = torch.cat([out, torch.zeros_like(out[..., :1])], -1)
    return out.to(t.dtype) if t.is_floating_point() else out


def identity_rope(length: int, device) -> torch.Tensor:
    """A RoPE table that leaves every pair unchanged ([[1,-0],[0,1]]): the
    joint QKV epilogue with it is QK RMSNorm alone, bit for bit."""
    f = torch.zeros(length, 64, 2, 2, dtype=torch.float32, device=device)
    f[..., 0, 0] = 1.0
    f[..., 1, 1] = 1.0
    return f


def text_block(cfg: DiTConfig, b: TextBlockWeights, x: torch.Tensor, batch: int, length: int,
               rope: torch.Tensor, zero_mod: torch.Tensor, ones_gate: torch.Tensor) -> torch.Tensor:
    """One text-fusion block on the W4A4 ops, x bf16 [batch*length, txtdim].
    RMSNorm is norm_quant with zero modulation (y*(0+1)+0 is exact); the
    residual adds are gated residuals with a gate of ones (T(T(p)*1) = T(p))."""
    eps = cfg.core.eps
    xq, xs = ops.norm_quant(x, b.norm1, zero_mod, zero_mod, length=length, eps=eps)
    q, k, v, g = ops.qkv(xq, xs, b.wq, b.wk, b.wv, b.qnorm, b.knorm, rope, length=length, eps_q=cfg.core.qk_eps,
                         eps_k=cfg.core.qk_eps, wg=b.wgate)
    H, Hk = cfg.txt_heads, cfg.txt_kvheads
    view = lambda t, h: t.view(batch, length, h, 128).transpose(1, 2)
    o = ops.attention(view(q, H), view(k, Hk), view(v, Hk), gate=g.view(batch, length, H * 128),
                      gate_is_sigmoid=True)
    oq, os_ = ops.rotate_quant(o.view(batch * length, H * 128))
    x1 = ops.gated_residual(oq, os_, b.wo, ones_gate, x, length=length)
    hq_in, hs_in = ops.norm_quant(x1, b.norm2, zero_mod, zero_mod, length=length, eps=eps)
    hq, hs = ops.swiglu_quant(hq_in, hs_in, b.wg, b.wu)
    return ops.gated_residual(hq, hs, b.wd, ones_gate, x1, length=length)


class Krea2DiT:
    """Resident weights of the whole model and its forward."""

    def __init__(self, cfg: DiTConfig, weights: DiTWeights):
        self.cfg, self.w = cfg, weights
        self._stacks: Dict[Tuple[int, int], Krea2Blocks] = {}

    def _stack(self, batch: int, length: int, device) -> Krea2Blocks:
        key = (batch, length)
        if key not in self._stacks:
            for b in self.w.blocks:
                if b.mod.shape[1] != batch:
                    b.mod = torch.empty((6, batch, self.cfg.core.hidden), dtype=torch.bfloat16, device=device)
            self._stacks = {key: Krea2Blocks(self.cfg.core, self.w.blocks, batch, length, device=device)}
        return self._stacks[key]

    def forward(self, x: torch.Tensor, timesteps: torch.Tensor, context: torch.Tensor,
                trace: Optional[dict] = None) -> torch.Tensor:
        """x bf16 [B, C, H, W] (H, W multiples of the patch), timesteps [B],
        context bf16 [B, Lt, txtdim] -> bf16 [B, C, H, W].  ``trace``: a dict
        that receives a copy of each stage's output (for stagewise checks)."""
        keep = (lambda k, v: trace.__setitem__(k, v.clone())) if trace is not None else (lambda k, v: None)
        cfg, w = self.cfg, self.w
        hidden = cfg.core.hidden
        B = int(x.shape[0])
        dev = x.device
        img, h, wd = patchify(x, cfg.patch)
        img = F.linear(img, *w.first)
        keep("img", img)
        t = timestep_embedding(timesteps, cfg.tdim).unsqueeze(1).to(img.dtype)
        t = F.linear(F.gelu(F.linear(t, *w.tmlp1), approximate="tanh"), *w.tmlp2)   # [B, 1, hidden]
        tvec = F.linear(t, *w.tproj)                                                # [B, 1, 6*hidden]
        keep("t", t)
        keep("tvec", tvec)
        # text fusion on the W4A4 ops (group-1 attention)
        Lt = int(context.shape[1])
        ctx = context.reshape(B * Lt, cfg.txtdim).contiguous()
        if w.txt:
            zero_mod = torch.zeros((B, cfg.txtdim), dtype=torch.bfloat16, device=dev)
            ones_gate = torch.ones((B, cfg.txtdim), dtype=torch.bfloat16, device=dev)
            rope = identity_rope(Lt, dev)
            for i, tb in enumerate(w.txt):
                ctx = text_block(cfg, tb, ctx, B, Lt, rope, zero_mod, ones_gate)
                keep(f"txt{i}", ctx)
        ctx = F.linear(ctx.view(B, Lt, cfg.txtdim), *w.txtmlp)
        combined = torch.cat([ctx, img], 1).contiguous()                             # [B, L, hidden]
        keep("combined", combined)
        L = int(combined.shape[1])
        freqs = rope_table(positions(Lt, h, wd, dev), cfg.axes, cfg.core.theta)
        stack = self._stack(B, L, dev)
        # DoubleSharedModulation per block: (tvec + lin_i).chunk(6), written
        # into the block loop's [6, B, hidden] modulation slots
        nblk = len(w.blocks)
        mods = (tvec.view(1, B, 6 * hidden) + w.mod_lin.view(nblk, 1, 6 * hidden)).view(nblk, B, 6, hidden)
        for i, b in enumerate(w.blocks):
            b.mod.copy_(mods[i].transpose(0, 1))
        stream = combined.view(B * L, hidden)
        stack.forward_(stream, freqs)
        keep("blocks", stream)
        scale, shift = (t + w.last_lin.unsqueeze(0)).chunk(2, dim=1)                # SimpleModulation
        y = ops.norm_mod(stream, w.last_norm, scale.reshape(B, hidden).contiguous(),
                         shift.reshape(B, hidden).contiguous(), length=L, eps=cfg.core.eps)
        keep("normed", y)
        out = F.linear(y.view(B, L, hidden)[:, Lt:], *w.last)
        return unpatchify(out, h, wd, cfg.patch, cfg.channels)


# ------------------------------------------------------------ synthetic init

def _lin(n: int, k: int, gen, device, std=0.02):
    w = (torch.randn((n, k), generator=gen, device=device) * std).to(torch.bfloat16)
    b = (torch.randn((n,), generator=gen, device=device) * std).to(torch.bfloat16)
    return w, b


def _norm_w(n: int, gen, device) -> torch.Tensor:
    w_eff = (torch.rand(n, generator=gen, device=device) * 0.2 + 0.9).to(torch.bfloat16)
    return (w_eff.to(torch.float32) - 1.0).contiguous()


def synthetic_dit(cfg: DiTConfig, batch: int = 1, seed: int = 0, device="cuda", keep_packed: bool = False,
                  blocks: Optional[List[BlockWeights]] = None) -> DiTWeights:
    """Seeded random-init weights of the whole model (no checkpoint): the
    W4A4 projections N(0, 0.02) rotated and INT4-quantised, plain linears
    N(0, 0.02) bf16, norm multipliers ~U(0.9, 1.1), modulation vectors
    N(0, 0.1).  ``blocks``: an existing block stack to reuse."""
    gen = torch.Generator(device=device).manual_seed(seed + 7919)
    hid, T = cfg.core.hidden, cfg.txtdim
    txt = []
    shapes = {"wq": (cfg.txt_heads * 128, T), "wk": (cfg.txt_kvheads * 128, T), "wv": (cfg.txt_kvheads * 128, T),
              "wgate": (cfg.txt_heads * 128, T), "wo": (T, cfg.txt_heads * 128), "wg": (cfg.txt_mlp, T),
              "wu": (cfg.txt_mlp, T), "wd": (T, cfg.txt_mlp)}
    for _ in range(cfg.txt_layers):
        prepared, packed = {}, {}
        for name, (n, k) in shapes.items():
            q, s = quantize_weight((torch.randn((n, k), generator=gen, device=device) * 0.02).to(torch.bfloat16))
            prepared[name] = ops.prepare_weight(q, s)
            if keep_packed:
                packed[name] = (q, s)
        txt.append(TextBlockWeights(norm1=_norm_w(T, gen, device), norm2=_norm_w(T, gen, device),
                                    qnorm=_norm_w(128, gen, device), knorm=_norm_w(128, gen, device),
                                    packed=packed, **prepared))
    return DiTWeights(
        first=_lin(hid, cfg.patch_dim, gen, device), tmlp1=_lin(hid, cfg.tdim, gen, device),
        tmlp2=_lin(hid, hid, gen, device), tproj=_lin(6 * hid, hid, gen, device), txt=txt,
        txtmlp=_lin(hid, T, gen, device),
        mod_lin=(torch.randn((cfg.core.blocks, 6 * hid), generator=gen, device=device) * 0.1).to(torch.bfloat16),
        last_lin=(torch.randn((2, hid), generator=gen, device=device) * 0.1).to(torch.bfloat16),
        last_norm=_norm_w(hid, gen, device), last=_lin(cfg.patch_dim, hid, gen, device),
        blocks=blocks if blocks is not None else synthetic_blocks(cfg.core, batch, seed=seed, device=device,
                                                                  keep_packed=keep_packed))
