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


@pytest.mark.parametrize("rows", [0, 1, 7])
def test_reference_contract_empty_and_ragged_rows(cuda, rows):
    """The reference contract's quantisers and byte-operand projections on
    empty and ragged row counts: empty outputs without a launch, and single /
    odd rows bit-exact (the last 256-row pair of the GEMM mostly empty)."""
    import torch
    from k2b import ref_ops

    K, N = 1024, 256
    xb = bf16_x(rows, K, 40 + rows, outliers=False)
    x = t_bf16(xb, cuda) if rows else torch.empty((0, K), dtype=torch.bfloat16, device=cuda)
    q8, s8 = ref_ops.quant4_e4m3(x, 64)
    q, s = ref_ops.quant4(x, 64)
    assert q8.shape == (rows, K) and q.shape == (rows, K // 2) and s.shape == (rows, 1)
    rng = np.random.default_rng(41)
    codes = rng.integers(-8, 8, (N, K)).astype(np.int8)
    packed = ((codes[:, 0::2] & 0xF) | ((codes[:, 1::2] & 0xF) << 4)).astype(np.uint8)
    ws = rng.uniform(1e-3, 1e-2, N).astype(np.float32)
    Wp, WS = t_u8(packed, cuda).view(torch.int8), t_f32(ws, cuda)
    W8 = ref_ops.codes_e4m3(Wp)
    out = ref_ops.gemm_f8(q8, s8.reshape(-1), W8, WS)
    assert out.shape == (rows, N)
    torch.cuda.synchronize()
    if rows:
        q_r, s_r = O.ref_quant(xb, group=64)
        assert np.array_equal(q.view(torch.uint8).cpu().numpy(), q_r)
        assert np.array_equal(bits(out), O.bf16_bits(O.ref_project(O.int4_codes(q_r), s_r, codes, ws)))
        assert torch.equal(out, ref_ops.gemm4(q, s.reshape(-1), Wp, WS))
