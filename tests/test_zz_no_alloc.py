"""The block loop entry point that allocates nothing (k2b_forward_blocks_static).

Some callers of this library cannot call cudaMalloc -- a host application that
owns the device allocator, or a plugin that only receives its input and output
buffers -- so this entry point keeps its workspace in a fixed device array
inside the library instead of a caller-provided buffer.  This test calls it
through the C ABI, twice in a row (the second call reuses the array left over
from the first), and checks each result against the regular entry point that
takes a caller-allocated workspace.  The file sorts last so that a run which
stops at the first failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest

import oracle as O
from _helpers import t_bf16

pytestmark = pytest.mark.gpu


def test_static_workspace_block_loop_matches_allocating_entry(cuda):
    import torch
    from k2b._native import lib
    from k2b.model import Krea2Blocks, ModelConfig, rope_positions, rope_table, synthetic_blocks

    L = lib()
    batch, length = 2, 150
    cfg = ModelConfig(hidden=512, heads=4, kvheads=2, mlp=1024, blocks=2)
    blocks = synthetic_blocks(cfg, batch, seed=11, device=cuda)
    model = Krea2Blocks(cfg, blocks, batch, length, device=cuda)
    freqs = rope_table(rope_positions(6, 12, 12), (64, 64), cfg.theta).to(cuda)
    need = L.k2b_block_workspace_bytes(batch * length, cfg.hidden, cfg.heads, cfg.kvheads, cfg.mlp)
    assert 0 < need <= L.k2b_static_workspace_bytes()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rng = np.random.default_rng(3)
    for call in range(2):
        x0 = t_bf16(O.bf16_bits(rng.standard_normal((batch * length, cfg.hidden)).astype(np.float32)), cuda)
        expect = model.forward_(x0.clone(), freqs)
        got = x0.clone()
        rc = L.k2b_forward_blocks_static(model._table, len(blocks), ctypes.c_void_p(got.data_ptr()),
                                         ctypes.c_void_p(freqs.data_ptr()), batch, length, cfg.hidden, cfg.heads,
                                         cfg.kvheads, cfg.mlp, ctypes.c_float(cfg.eps), ctypes.c_float(cfg.qk_eps),
                                         stream)
        assert rc == 0, f"call {call}: status {rc}"
        torch.cuda.synchronize()
        assert torch.equal(got, expect), f"call {call}: output differs from k2b_forward_blocks"


def test_static_workspace_rejects_oversized_requests(cuda):
    import torch
    from k2b._native import lib

    L = lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # 8 latents x 4224 tokens at the Krea2 widths needs ~1.5 GB: beyond the fixed array
    rc = L.k2b_forward_blocks_static(None, 1, None, None, 8, 4224, 6144, 48, 12, 16384, ctypes.c_float(1e-6),
                                     ctypes.c_float(1e-6), stream)
    assert rc == 1  # cudaErrorInvalidValue, before any pointer is touched
