"""norm_quant / rotate_quant on the B200 vs the CPU oracle: bit-exact codes and scales."""
import ctypes

import numpy as np
import pytest

import oracle as O
from _helpers import bf16_x, bits, norm_inputs, t_bf16, t_f32

pytestmark = pytest.mark.gpu


def _run(cuda, rows, K, length, cut, nb, seed):
    import torch
    from k2b import ops

    xb = bf16_x(rows, K, seed)
    w, sc, sh = norm_inputs(K, nb, seed + 1)
    q, s = ops.norm_quant(t_bf16(xb, cuda), t_f32(w, cuda), t_bf16(sc, cuda), t_bf16(sh, cuda), length=length,
                          cut=cut, eps=1e-6)
    torch.cuda.synchronize()
    batch = max(1, rows // length)
    qo, so = O.norm_quant(xb, w, sc, sh, length=length, cut=cut, batch=batch, eps=1e-6)
    return q.cpu().numpy(), bits(s), qo, so


@pytest.mark.parametrize("rows,K", [(1, 512), (129, 1024), (300, 6144), (4050, 6144), (64, 16384)])
def test_norm_quant_bitexact(cuda, rows, K):
    q, s, qo, so = _run(cuda, rows, K, rows, -1, 1, 11 + rows)
    assert np.array_equal(s, so), "fp16 group scales differ"
    assert np.array_equal(q, qo), f"packed codes differ at {np.argwhere(q != qo)[:5]}"


def test_norm_quant_batched_modulation(cuda):
    # 3 latents of 100 tokens, one modulation row each
    q, s, qo, so = _run(cuda, 300, 1024, 100, -1, 3, 5)
    assert np.array_equal(s, so) and np.array_equal(q, qo)


def test_norm_quant_cut_split(cuda):
    # reference-image split: rows >= cut of each latent use modulation row b + batch
    q, s, qo, so = _run(cuda, 200, 512, 100, 60, 4, 9)
    assert np.array_equal(s, so) and np.array_equal(q, qo)


@pytest.mark.parametrize("rows,K", [(7, 512), (4050, 6144)])
def test_rotate_quant_bitexact(cuda, rows, K):
    import torch
    from k2b import ops

    xb = bf16_x(rows, K, 3)
    q, s = ops.rotate_quant(t_bf16(xb, cuda))
    torch.cuda.synchronize()
    qo, so = O.rotate_quant(xb)
    assert np.array_equal(bits(s), so) and np.array_equal(q.cpu().numpy(), qo)


def test_reference_named_export_keeps_the_reference_contract(cuda):
    """k2_norm_mod_quant4 (kernels/norm_quant.cu:89) writes ONE fp32 scale per
    row into the reference's [rows, 1] buffer (group 256 here); group 128, which
    the reference's own kernel rejects, is rejected, so a reference-sized scale
    buffer can never receive group-128 scales.  (Bit-exactness of the contract:
    tests/test_gpu_ref_contract.py.)"""
    import torch
    from k2b._native import lib

    rows, K = 33, 1024
    xb = bf16_x(rows, K, 21)
    w, sc, sh = norm_inputs(K, 1, 22)
    x, wt, sct, sht = t_bf16(xb, cuda), t_f32(w, cuda), t_bf16(sc, cuda), t_bf16(sh, cuda)
    q = torch.empty((rows, K // 2), dtype=torch.uint8, device=cuda)
    s = torch.full((rows + 1, 1), -1.0, dtype=torch.float32, device=cuda)  # one guard row
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    assert lib().k2_norm_mod_quant4(P(x), P(wt), P(sct), P(sht), P(q), P(s), rows, K, rows, -1, 1,
                                    ctypes.c_float(1e-6), 256, 2, st) == 0
    for group, dtype in ((128, 2), (256, 1), (32, 2)):
        assert lib().k2_norm_mod_quant4(P(x), P(wt), P(sct), P(sht), P(q), P(s), rows, K, rows, -1, 1,
                                        ctypes.c_float(1e-6), group, dtype, st) != 0
    torch.cuda.synchronize()
    sv = s.cpu().numpy()[:, 0]
    assert (sv[:rows] > 0).all() and sv[rows] == -1.0  # nothing written past [rows, 1]
    qo, so = O.ref_quant(xb, w, sc, sh, group=256)
    assert np.array_equal(q.cpu().numpy(), qo) and np.array_equal(sv[:rows], so)