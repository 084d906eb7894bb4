"""Host-side logic of the k2b package (no GPU): RoPE positions and table,
argument validation of the torch wrappers, the work accounting bench.py uses."""
import numpy as np
import pytest
import torch

import oracle as O


def test_rope_table_matches_oracle_restatement():
    from k2b.model import rope_positions, rope_table

    pos = rope_positions(98, 76, 52)
    assert pos.shape == (4050, 2)
    t = rope_table(pos, (64, 64), 10000.0)
    assert t.shape == (4050, 64, 2, 2) and t.dtype == torch.float32
    ref = O.rope_table(pos.numpy(), (64, 64), 10000.0)
    assert np.array_equal(t.numpy(), ref)


def test_rope_positions_layout():
    from k2b.model import rope_positions

    pos = rope_positions(128, 64, 64).numpy()
    assert pos.shape == (4224, 2)
    assert np.array_equal(pos[:128, 0], np.arange(128)) and np.array_equal(pos[:128, 0], pos[:128, 1])
    assert pos[128].tolist() == [128.0, 128.0] and pos[128 + 65].tolist() == [129.0, 129.0]


def test_ops_reject_cpu_tensors():
    from k2b import ops

    x = torch.zeros(4, 512, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        ops.rotate_quant(x)
    with pytest.raises(ValueError):
        ops.attention(torch.zeros(1, 2, 4, 128, dtype=torch.bfloat16), torch.zeros(1, 1, 4, 128, dtype=torch.bfloat16),
                      torch.zeros(1, 1, 4, 128, dtype=torch.bfloat16), mask=torch.ones(4, 4, dtype=torch.bool))


def test_block_work_accounting_matches_baseline_figures():
    from k2b.model import ModelConfig, block_flops

    cfg = ModelConfig()
    f = block_flops(cfg, 4050, 4050, 1)
    assert round(f["qkv"] / 1e9, 2) == 458.65
    assert round(f["attn"] / 1e9, 2) == 403.11
    assert round(f["int_ops"] / 1e9, 1) == 3210.5


def test_norm_weight_w_plus_one_form_is_exact():
    from k2b.model import _norm_weight

    g = torch.Generator().manual_seed(0)
    w = _norm_weight(6144, g, "cpu")
    w_eff = w + 1.0
    assert torch.equal(w_eff, w_eff.to(torch.bfloat16).to(torch.float32))
    assert float(w_eff.min()) >= 0.89 and float(w_eff.max()) <= 1.11


def test_e4m3_code_table_matches_torch_float8():
    """The byte-permute lookup tables of the INT4 -> e4m3 conversion (shared by
    the GEMM's A unpacker, the weight preparation and the byte-container
    producers) hold torch's e4m3fn encodings of the codes -8..7."""
    import torch

    from _helpers import E4M3

    ref = torch.arange(-8, 8, dtype=torch.float32).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert (E4M3 == ref).all()
    # the words of the CUDA lookup: bytes 0..7 of the positive table = e4m3(0..7),
    # of the negative table = e4m3(-8..-1)
    pos = (0x44403800).to_bytes(4, "little") + (0x4E4C4A48).to_bytes(4, "little")
    neg = (0xCACCCED0).to_bytes(4, "little") + (0xB8C0C4C8).to_bytes(4, "little")
    assert list(pos) == list(ref[8:]) and list(neg) == list(ref[:8])


def test_dit_patch_layout_and_helpers():
    """k2b.dit's host-side pieces: patchify / unpatchify are inverse
    ('b c (h ph) (w pw) <-> b (h w) (c ph pw)', graph_model.py:300-301), text
    tokens sit at position 0 (graph_model.py:242), the identity RoPE table is
    [[1, 0], [0, 1]] and the timestep embedding follows native_runtime.cpp:511-513."""
    import math

    import torch
    from k2b import dit

    x = torch.randn(2, 4, 6, 10)
    t, h, w = dit.patchify(x, 2)
    assert t.shape == (2, 15, 16) and (h, w) == (3, 5)
    assert torch.equal(t[1, 5 + 2, 4 * 1 + 2 * 1 + 0], x[1, 1, 2 * 1 + 1, 2 * 2 + 0])
    assert torch.equal(dit.unpatchify(t, h, w, 2, 4), x)
    pos = dit.positions(3, 2, 4)
    assert pos.shape == (11, 2) and not pos[:3].any() and pos[3 + 4 * 1 + 2].tolist() == [1.0, 2.0]
    f = dit.identity_rope(5, "cpu")
    assert torch.equal(f[2, 7], torch.tensor([[1.0, 0.0], [0.0, 1.0]]))
    e = dit.timestep_embedding(torch.tensor([0.25]), 8)
    args = 250.0 * torch.exp(-math.log(10000.0) * torch.arange(4, dtype=torch.float32) / 4)
    assert torch.allclose(e[0], torch.cat([args.cos(), args.sin()]))
