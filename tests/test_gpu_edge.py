"""Edge cases of the op layer on the B200: empty batches return empty outputs
without a launch, and single rows / ragged row counts go through every kernel
family (the reference allocates with at::empty and launches per call,
native_runtime.cpp:373,413-414,441)."""
import numpy as np
import pytest

import oracle as O
from _helpers import bf16_x, bits, norm_inputs, packed_act, packed_weight, t_bf16, t_f16, t_f32, t_u8

pytestmark = pytest.mark.gpu


def test_empty_inputs_return_empty_outputs(cuda):
    import torch
    from k2b import ops

    K, N = 512, 256
    x = torch.empty((0, K), dtype=torch.bfloat16, device=cuda)
    w, sc, sh = norm_inputs(K, 1, 0)
    q, s = ops.norm_quant(x, t_f32(w, cuda), t_bf16(sc, cuda), t_bf16(sh, cuda))
    assert q.shape == (0, K // 2) and s.shape == (0, K // 128)
    q2, s2 = ops.rotate_quant(x)
    assert q2.shape == (0, K // 2) and s2.shape == (0, K // 128)
    assert ops.norm_mod(x, t_f32(w, cuda)).shape == (0, K)
    wq, ws = packed_weight(N, K, 1)
    W = ops.prepare_weight(t_u8(wq, cuda), t_f16(ws, cuda))
    a = torch.empty((0, K // 2), dtype=torch.uint8, device=cuda)
    sa = torch.empty((0, K // 128), dtype=torch.float16, device=cuda)
    assert ops.gemm_f32(a, sa, W).shape == (0, N)
    assert ops.gemm_bf16(a, sa, W).shape == (0, N)
    gate = torch.zeros((0, N), dtype=torch.bfloat16, device=cuda)  # [batch = 0 // length, N]
    res = torch.empty((0, N), dtype=torch.bfloat16, device=cuda)
    assert ops.gated_residual(a, sa, W, gate, res, length=1).shape == (0, N)
    hq, hs = ops.swiglu_quant(a, sa, W, W)
    assert hq.shape == (0, N // 2) and hs.shape == (0, N // 128)
    qv = torch.empty((1, 4, 0, 128), dtype=torch.bfloat16, device=cuda)
    kv = torch.empty((1, 2, 0, 128), dtype=torch.bfloat16, device=cuda)
    assert ops.attention(qv, kv, kv).shape == (1, 0, 512)
    oq, os_ = ops.attention_quant(qv, kv, kv)
    assert oq.shape == (0, 256) and os_.shape == (0, 4)
    torch.cuda.synchronize()
    assert ops.device_error() == 0


@pytest.mark.parametrize("rows", [1, 7, 129])
def test_single_and_ragged_rows_bitexact(cuda, rows):
    import torch
    from k2b import ops

    K, N = 512, 256
    xb = bf16_x(rows, K, 30 + rows)
    w, sc, sh = norm_inputs(K, 1, 31)
    q, s = ops.norm_quant(t_bf16(xb, cuda), t_f32(w, cuda), t_bf16(sc, cuda), t_bf16(sh, cuda), length=rows)
    qr, sr = O.norm_quant(xb, w, sc, sh, length=rows)
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), qr) and np.array_equal(bits(s), sr)
    wq, ws = packed_weight(N, K, 32)
    W = ops.prepare_weight(t_u8(wq, cuda), t_f16(ws, cuda))
    out = ops.gemm_f32(q, s, W)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), O.gemm_w4a4(qr, sr, wq, ws))
