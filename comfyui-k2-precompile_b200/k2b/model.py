"""Krea2-shaped W4A4 DiT block stack on libk2b.

* ``rope_positions`` / ``rope_table`` -- the EmbedND table the QKV epilogue
  consumes (native_runtime.cpp:509-510: per axis of dim d,
  omega = theta^-(linspace(0,(d-2)/d,d/2)) in float64, angle = fp32(pos)*omega,
  [[cos,-sin],[sin,cos]], concatenated over axes, fp32 [L, 64, 2, 2]).
  Positions: text token i -> (i, i) (1-D), image token (y, x) -> (T+y, T+x)
  on the 2-D axial grid, 64 rotary dims per axis, theta = 10000.
* ``Krea2Blocks`` -- resident prepared weights for N blocks and the forward
  that runs the native block loop (k2b_forward_blocks) -- the replacement of
  graph_model.dit's per-block chain (graph_model.py:259-295).
* ``synthetic_blocks`` -- seeded random-init weights: N(0, 0.02) bf16,
  H128-rotated and INT4-quantised by k2b_rotate_quant; norm multipliers
  ~U(0.9, 1.1); adaLN vectors ~N(0, 0.1) per block.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass, field
from typing import Callable, List, Optional, Tuple

import torch

from . import ops
from ._native import check, lib
from .ops import PreparedWeight


@dataclass
class ModelConfig:
    hidden: int = 6144
    heads: int = 48
    kvheads: int = 12
    mlp: int = 16384
    blocks: int = 28
    eps: float = 1e-6
    qk_eps: float = 1e-6
    theta: float = 10000.0

    @property
    def head_dim(self) -> int:
        return 128


def rope_positions(text_tokens: int, grid_h: int, grid_w: int) -> torch.Tensor:
    """fp32 [text + h*w, 2]: (i, i) for text, (T + y, T + x) for image tokens."""
    t = torch.arange(text_tokens, dtype=torch.float32)
    txt = torch.stack([t, t], dim=1)
    y = torch.arange(grid_h, dtype=torch.float32).repeat_interleave(grid_w)
    x = torch.arange(grid_w, dtype=torch.float32).repeat(grid_h)
    img = torch.stack([y + text_tokens, x + text_tokens], dim=1)
    return torch.cat([txt, img], dim=0)


def rope_table(pos: torch.Tensor, axes=(64, 64), theta: float = 10000.0) -> torch.Tensor:
    """pos [L, n_axes] -> fp32 [L, sum(axes)/2, 2, 2] (EmbedND)."""
    pieces = []
    for i, d in enumerate(axes):
        scale = torch.linspace(0.0, (d - 2) / d, d // 2, dtype=torch.float64, device=pos.device)
        omega = torch.reciprocal(torch.pow(torch.tensor(theta, dtype=torch.float64, device=pos.device), scale))
        angle = pos[:, i].to(torch.float32).to(torch.float64).unsqueeze(-1) * omega
        cos, sin = angle.cos(), angle.sin()
        pieces.append(torch.stack([cos, -sin, sin, cos], dim=-1).reshape(pos.shape[0], d // 2, 2, 2))
    return torch.cat(pieces, dim=1).to(torch.float32).contiguous()


@dataclass
class BlockWeights:
    prenorm: torch.Tensor   # fp32 [hidden] ("w+1" form)
    postnorm: torch.Tensor
    qnorm: torch.Tensor     # fp32 [128]
    knorm: torch.Tensor
    wq: PreparedWeight
    wk: PreparedWeight
    wv: PreparedWeight
    wo: PreparedWeight
    wg: PreparedWeight
    wu: PreparedWeight
    wd: PreparedWeight
    mod: torch.Tensor       # bf16 [6, batch, hidden]: ps, ph, pg, ss, sh, sg
    packed: dict = field(default_factory=dict)  # optional "checkpoint" form {name: (u8, fp16)}

    def slots(self) -> List[int]:
        return [self.prenorm.data_ptr(), self.postnorm.data_ptr(), self.qnorm.data_ptr(), self.knorm.data_ptr(),
                self.wq.w.data_ptr(), self.wq.scale.data_ptr(), self.wk.w.data_ptr(), self.wk.scale.data_ptr(),
                self.wv.w.data_ptr(), self.wv.scale.data_ptr(), self.wo.w.data_ptr(), self.wo.scale.data_ptr(),
                self.wg.w.data_ptr(), self.wg.scale.data_ptr(), self.wu.w.data_ptr(), self.wu.scale.data_ptr(),
                self.wd.w.data_ptr(), self.wd.scale.data_ptr(), self.mod.data_ptr()]


def quantize_weight(w: torch.Tensor):
    """bf16 [n, k] -> packed INT4 (u8 [n, k/2]) + fp16 group scales, with the
    same H128 rotation along k as the activations (ConvRot W4A4)."""
    return ops.rotate_quant(w.to(torch.bfloat16).contiguous())


def _norm_weight(n: int, gen: torch.Generator, device) -> torch.Tensor:
    w_eff = (torch.rand(n, generator=gen, device=device) * 0.2 + 0.9).to(torch.bfloat16)
    # "w+1" form: fp32(w_eff) - 1 is exact (Sterbenz), and w + 1 == w_eff exactly
    return (w_eff.to(torch.float32) - 1.0).contiguous()


def synthetic_blocks(cfg: ModelConfig, batch: int, seed: int = 0, device="cuda", keep_packed: bool = False,
                     shard: Optional[Callable[[str, torch.Tensor, torch.Tensor], Tuple[torch.Tensor, torch.Tensor]]]
                     = None) -> List[BlockWeights]:
    """``shard(name, packed, scales)`` (optional) keeps a slice of each packed
    weight before it is prepared: every rank draws the same full weights from
    the seed and keeps its own shard (k2b.parallel.shard_packed)."""
    gen = torch.Generator(device=device).manual_seed(seed)
    H, D = cfg.hidden, cfg.head_dim
    shapes = {"wq": (cfg.heads * D, H), "wk": (cfg.kvheads * D, H), "wv": (cfg.kvheads * D, H),
              "wo": (H, cfg.heads * D), "wg": (cfg.mlp, H), "wu": (cfg.mlp, H), "wd": (H, cfg.mlp)}
    blocks = []
    for _ in range(cfg.blocks):
        prepared, packed = {}, {}
        for name, (n, k) in shapes.items():
            w = (torch.randn((n, k), generator=gen, device=device) * 0.02).to(torch.bfloat16)
            q, s = quantize_weight(w)
            del w
            if shard is not None:
                q, s = shard(name, q, s)
            prepared[name] = ops.prepare_weight(q, s)
            if keep_packed:
                packed[name] = (q, s)
        mod = (torch.randn((6, batch, H), generator=gen, device=device) * 0.1).to(torch.bfloat16).contiguous()
        blocks.append(BlockWeights(
            prenorm=_norm_weight(H, gen, device), postnorm=_norm_weight(H, gen, device),
            qnorm=_norm_weight(D, gen, device), knorm=_norm_weight(D, gen, device),
            mod=mod, packed=packed, **prepared))
    return blocks


class Krea2Blocks:
    """Resident W4A4 block stack + the native forward."""

    def __init__(self, cfg: ModelConfig, blocks: List[BlockWeights], batch: int, length: int, device="cuda"):
        self.cfg, self.blocks, self.batch, self.length = cfg, blocks, batch, length
        L = lib()
        nslots = L.k2b_block_slots()
        table = []
        for b in blocks:
            s = b.slots()
            assert len(s) == nslots
            table.extend(s)
        self._table = (ctypes.c_void_p * len(table))(*table)
        rows = batch * length
        nbytes = L.k2b_block_workspace_bytes(rows, cfg.hidden, cfg.heads, cfg.kvheads, cfg.mlp)
        check(0 if nbytes > 0 else 1, "k2b_block_workspace_bytes")
        self.workspace = torch.empty(int(nbytes), dtype=torch.uint8, device=device)

    def forward_(self, x: torch.Tensor, freqs: torch.Tensor, events=None) -> torch.Tensor:
        """In-place forward of the residual stream x bf16 [batch*length, hidden].
        events: optional list of nblocks*8 torch.cuda.Event (enable_timing)
        recorded between the native launches (see k2b_forward_blocks)."""
        cfg = self.cfg
        ops._cuda(x, freqs)
        ops._need(x.dtype == torch.bfloat16 and tuple(x.shape) == (self.batch * self.length, cfg.hidden),
                  "forward: x shape")
        ops._need(freqs.dtype == torch.float32 and freqs.numel() == self.length * 256, "forward: freqs shape")
        ev = None
        if events is not None:
            ops._need(len(events) == 8 * len(self.blocks), "forward: need 8 events per block")
            ev = (ctypes.c_void_p * len(events))(*[e.cuda_event for e in events])
        check(lib().k2b_forward_blocks(self._table, len(self.blocks), ops._p(x), ops._p(freqs),
                                       ops._p(self.workspace), self.workspace.numel(), self.batch, self.length,
                                       cfg.hidden, cfg.heads, cfg.kvheads, cfg.mlp, ctypes.c_float(cfg.eps),
                                       ctypes.c_float(cfg.qk_eps), ev, ops._stream()), "k2b_forward_blocks")
        return x


def block_python(cfg: ModelConfig, b: BlockWeights, x: torch.Tensor, freqs: torch.Tensor, batch: int, length: int
                 ) -> torch.Tensor:
    """The same block through the per-op wrappers (one launch per op), for
    debugging and for tensor-parallel variants that insert collectives."""
    H = cfg.hidden
    ps, ph, pg, ss, sh, sg = b.mod.unbind(0)
    xq, xs = ops.norm_quant(x, b.prenorm, ps, ph, length=length, eps=cfg.eps)
    q, k, v, _ = ops.qkv(xq, xs, b.wq, b.wk, b.wv, b.qnorm, b.knorm, freqs, length=length, eps_q=cfg.qk_eps,
                         eps_k=cfg.qk_eps)
    qv = q.view(batch, length, cfg.heads, 128).transpose(1, 2)
    kv = k.view(batch, length, cfg.kvheads, 128).transpose(1, 2)
    vv = v.view(batch, length, cfg.kvheads, 128).transpose(1, 2)
    oq, os_ = ops.attention_quant(qv, kv, vv)
    x1 = ops.gated_residual(oq, os_, b.wo, pg.contiguous(), x, length=length)
    hq_in, hs_in = ops.norm_quant(x1, b.postnorm, ss, sh, length=length, eps=cfg.eps)
    hq, hs = ops.swiglu_quant(hq_in, hs_in, b.wg, b.wu)
    return ops.gated_residual(hq, hs, b.wd, sg.contiguous(), x1, length=length)


def block_flops(cfg: ModelConfig, rows: int, length: int, batch: int) -> dict:
    """Algorithmic work of one block (int ops of the W4A4 GEMMs, bf16 flops of attention)."""
    H, D = cfg.hidden, 128
    qkv = 2 * rows * (cfg.heads + 2 * cfg.kvheads) * D * H
    out = 2 * rows * H * cfg.heads * D
    gu = 2 * rows * 2 * cfg.mlp * H
    down = 2 * rows * H * cfg.mlp
    attn = 4 * batch * cfg.heads * length * length * D
    return {"qkv": qkv, "out": out, "gate_up": gu, "down": down, "int_ops": qkv + out + gu + down, "attn": attn}
