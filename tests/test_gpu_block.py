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
