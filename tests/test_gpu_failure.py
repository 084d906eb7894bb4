"""Failure detection on the B200 without a GPU fault: a device-side mbarrier
wait that nothing completes gives up after its limit, records its error bit,
makes the rest of the CTA unwind through the abort flag, and leaves the
context usable (every kernel's waits share this mbar_wait path)."""
import time

import numpy as np
import pytest

import oracle as O
from _helpers import bf16_x, bits, norm_inputs, t_bf16, t_f32

pytestmark = pytest.mark.gpu

ERR_WAIT_SELFTEST = 1 << 6


def test_wait_that_completes_reports_nothing(cuda):
    from k2b import ops

    ops.device_error(reset=True)
    res = ops.selftest_wait(0, 20_000_000, device=cuda)
    assert res[0] == 1
    assert ops.device_error(reset=True) == 0


def test_wait_runs_out_reports_and_context_survives(cuda):
    from k2b import ops

    ops.device_error(reset=True)
    limit_ns = 20_000_000  # 20 ms
    t0 = time.perf_counter()
    res = ops.selftest_wait(1, limit_ns, device=cuda)
    elapsed = time.perf_counter() - t0
    assert res[0] == 0  # warp 0's wait gave up
    assert res[1] == 1  # warp 1 left through the abort flag, before its own 64x limit
    assert res[2] * 1000 < 16 * limit_ns
    assert elapsed < 2.0
    err = ops.device_error(reset=True)
    assert err == ERR_WAIT_SELFTEST
    assert ops.device_error(reset=True) == 0

    # the context still computes: a norm_quant bit-exact against the oracle
    rows, K = 9, 1024
    xb = bf16_x(rows, K, 5)
    w, sc, sh = norm_inputs(K, 1, 6)
    q, s = ops.norm_quant(t_bf16(xb, cuda), t_f32(w, cuda), t_bf16(sc, cuda), t_bf16(sh, cuda), length=rows)
    q_r, s_r = O.norm_quant(xb, w, sc, sh, length=rows)
    assert np.array_equal(q.cpu().numpy(), q_r) and np.array_equal(bits(s), s_r)


def test_selftest_rejects_bad_arguments(cuda):
    from k2b import ops

    for mode, limit in ((2, 1000), (1, 0), (1, 2_000_000_000)):
        with pytest.raises(ops.K2BError):
            ops.selftest_wait(mode, limit, device=cuda)
