"""The headline configurations against the CPU oracle at their full sizes.

* config 3's block: one latent of 4050 tokens (98 text + 76x52 image) at the
  Krea2 widths, every row, stage by stage: norm_quant, the QKV epilogue, the
  out-projection, SwiGLU + requant and the down-projection bit-exact, attention
  within 2e-2 absolute (4050 = 31*128 + 82 leaves a ragged last tile in every
  kernel);
* 28 blocks x 4050 tokens at a reduced width (hidden 512, 4/2 heads): the native
  block loop and the oracle chain each evolve their own residual stream, and
  after every block the two agree to cosine >= 0.999 (north_star's per-block
  criterion); the max abs error per block is reported;
* config 4's block shape: latents of 4224 tokens (128 text + 64x64 image),
  three of them so that the last 256-row pair tile of the GEMMs is half filled
  (3*4224 = 49.5 * 256) and the modulation rows of three latents are used.

The block outputs are held to the cosine bound rather than 2e-2 absolute: a
residual stream's values grow past 2e-2 resolution (bf16 spacing is 2^-7
relative), and one attention rounding difference can flip an INT4 code.  The
per-stage checks above hold every stage to the absolute bound (or bit-exact).
"""
import json
import os

import numpy as np
import pytest

import oracle as O
from _helpers import TOL_COS, bits, cosine, np_block, oracle_block, stagewise_block, t_bf16

pytestmark = pytest.mark.gpu


def _report(name, payload):
    path = os.environ.get("K2B_PARITY_REPORT")
    if path:
        os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
        data = {}
        if os.path.exists(path):
            with open(path) as f:
                data = json.load(f)
        data[name] = payload
        with open(path, "w") as f:
            json.dump(data, f, indent=1)


def _x(rows, hidden, seed):
    rng = np.random.default_rng(seed)
    return O.bf16_bits(rng.standard_normal((rows, hidden)).astype(np.float32))


def _full_block(cuda, batch, text, gh, gw, seed):
    import torch
    from k2b.model import Krea2Blocks, ModelConfig, rope_positions, rope_table, synthetic_blocks

    length = text + gh * gw
    cfg = ModelConfig(blocks=1)
    bw = synthetic_blocks(cfg, batch, seed=seed, device=cuda, keep_packed=True)
    freqs = rope_table(rope_positions(text, gh, gw), (64, 64), cfg.theta).to(cuda)
    xb = _x(batch * length, cfg.hidden, seed + 1)
    out, stats = stagewise_block(cfg, bw[0], xb, freqs, batch, length, cuda)
    # the native block loop is the per-op chain, and stays within the
    # per-block bound of the independent oracle chain
    model = Krea2Blocks(cfg, bw, batch, length, device=cuda)
    native = model.forward_(t_bf16(xb, cuda), freqs)
    torch.cuda.synchronize()
    assert np.array_equal(bits(native), out), "native loop != per-op chain"
    ref = oracle_block(xb, np_block(bw[0]), freqs.cpu().numpy(), batch, length, cfg.heads, cfg.kvheads)
    g, r = O.bf16_float(bits(native)), O.bf16_float(ref)
    stats["block_cos"] = cosine(g, r)
    stats["block_max_abs"] = float(np.abs(g.astype(np.float64) - r).max())
    stats["block_exact_frac"] = float(np.mean(bits(native) == ref))
    assert stats["block_cos"] >= TOL_COS, stats
    return stats


def test_config3_block_full_size_vs_oracle(cuda):
    stats = _full_block(cuda, 1, 98, 76, 52, seed=31)
    _report("config3_block_4050", stats)


def test_config4_block_shape_vs_oracle(cuda):
    stats = _full_block(cuda, 3, 128, 64, 64, seed=41)
    _report("config4_block_3x4224", stats)


def test_chain_28_blocks_4050_tokens_vs_oracle(cuda):
    import torch
    from k2b.model import Krea2Blocks, ModelConfig, rope_positions, rope_table, synthetic_blocks

    batch, text, gh, gw = 1, 98, 76, 52
    length = text + gh * gw
    cfg = ModelConfig(hidden=512, heads=4, kvheads=2, mlp=1024, blocks=28)
    bw = synthetic_blocks(cfg, batch, seed=51, device=cuda, keep_packed=True)
    freqs = rope_table(rope_positions(text, gh, gw), (64, 64), cfg.theta).to(cuda)
    f_np = freqs.cpu().numpy()
    xb = _x(batch * length, cfg.hidden, 52)
    x = t_bf16(xb, cuda)
    ref = xb
    per_block = []
    for i, b in enumerate(bw):
        x = Krea2Blocks(cfg, [b], batch, length, device=cuda).forward_(x, freqs)
        torch.cuda.synchronize()
        ref = oracle_block(ref, np_block(b), f_np, batch, length, cfg.heads, cfg.kvheads)
        g, r = O.bf16_float(bits(x)).astype(np.float64), O.bf16_float(ref).astype(np.float64)
        per_block.append({"block": i, "cos": cosine(g, r), "max_abs": float(np.abs(g - r).max()),
                          "stream_max": float(np.abs(r).max())})
    _report("chain_28x4050_hidden512", per_block)
    print("\nblock  cosine      max_abs   stream_max")
    for e in per_block:
        print(f"{e['block']:5d}  {e['cos']:.7f}  {e['max_abs']:.4g}  {e['stream_max']:.4g}")
    worst = min(e["cos"] for e in per_block)
    assert worst >= TOL_COS, per_block
