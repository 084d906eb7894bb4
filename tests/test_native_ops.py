"""torch.ops.k2_native / k2_fullgraph surface without a GPU: schemas equal the
reference's (native_runtime.cpp:576-591, KohakuKernelRouter/attention.py:189),
fake implementations give the shapes torch.compile traces with, the binding
registry behaves like native_runtime.cpp's, and CPU tensors reach no kernel."""
import ctypes

import pytest
import torch

from k2b import native_ops as N

# The reference's schema strings (native_runtime.cpp:576-591).
REFERENCE_SCHEMAS = [
    "norm_quant(Tensor x, Tensor scale, Tensor shift, int norm_key, int target_key, int cut) -> (Tensor, Tensor)",
    "gated_norm_quant(Tensor x, Tensor gate, Tensor residual, Tensor scale, Tensor shift, int key, int norm_key, "
    "int target_key, int cut) -> (Tensor, Tensor, Tensor)",
    "qkv_prepared(Tensor x, Tensor qa, Tensor qs, Tensor freqs, int[] keys, int[] norms, int heads, int kvheads) "
    "-> (Tensor, Tensor, Tensor, Tensor)",
    "swiglu_prepared(Tensor x, Tensor qa, Tensor qs, int[] keys, int width) -> Tensor",
    "sdpa(Tensor q, Tensor k, Tensor v, bool enable_gqa) -> Tensor",
    "managed(Tensor x, int key, int kind, int width) -> Tensor",
    "gated(Tensor x, Tensor gate, Tensor residual, int key) -> Tensor",
    "norm_mod(Tensor x, Tensor scale, Tensor shift, int key, int cut) -> Tensor",
    "project_many(Tensor x, int[] keys, int[] widths) -> Tensor[]",
    "attention_inputs(Tensor x, Tensor? freqs, int[] keys, int[] widths, int[] norms, int heads, int kvheads) "
    "-> (Tensor, Tensor, Tensor, Tensor)",
    "residual_norm(Tensor x, Tensor gate, Tensor residual, Tensor scale, Tensor shift, int key, int norm_key) "
    "-> (Tensor, Tensor)",
    "joint_swiglu(Tensor x, int[] keys, int width) -> Tensor",
    "joint_qkv(Tensor x, Tensor freqs, int[] keys, int[] norms, int heads, int kvheads) "
    "-> (Tensor, Tensor, Tensor, Tensor)",
    "activation(Tensor x, str kind) -> Tensor",
    "activate_mul(Tensor a, Tensor b, str kind) -> Tensor",
    "modulation(Tensor x, Tensor scale, Tensor shift) -> Tensor",
    "residual(Tensor x, Tensor gate, Tensor value) -> Tensor",
    "rope(Tensor q, Tensor k, Tensor freqs) -> (Tensor, Tensor)",
    "timestep(Tensor t, int dim) -> Tensor",
]


@pytest.mark.parametrize("schema", REFERENCE_SCHEMAS)
def test_schema_matches_reference(schema):
    name = schema.split("(")[0]
    assert str(getattr(torch.ops.k2_native, name).default._schema) == "k2_native::" + schema


def test_kohaku_fa_schema():
    assert str(torch.ops.k2_fullgraph.kohaku_fa.default._schema) == (
        "k2_fullgraph::kohaku_fa(Tensor q, Tensor k, Tensor v, Tensor? mask, Tensor? gate, bool gate_is_sigmoid) "
        "-> Tensor")


def _m(*shape, dtype=torch.bfloat16):
    return torch.empty(shape, device="meta", dtype=dtype)


def test_fakes_give_reference_shapes():
    B, L, K, H, Hk = 2, 5, 1024, 8, 2
    x = _m(B, L, K)
    q, s = torch.ops.k2_native.norm_quant(x, _m(B, K), _m(B, K), 1, 2, -1)
    assert q.shape == (B * L, K // 2) and q.dtype == torch.int8
    assert s.shape == (B * L, K // 128) and s.dtype == torch.float16
    out, q2, s2 = torch.ops.k2_native.gated_norm_quant(x, _m(B, 1, K), x, _m(B, K), _m(B, K), 3, 1, 2, -1)
    assert out.shape == x.shape and q2.shape == q.shape and s2.shape == s.shape
    qq, kk, vv, gg = torch.ops.k2_native.qkv_prepared(x, q, s, _m(1, 1, L, 64, 2, 2, dtype=torch.float32),
                                                      [1, 2, 3, 4], [5, 6], H, Hk)
    assert qq.shape == (B, H, L, 128) and kk.shape == (B, Hk, L, 128)
    assert qq.stride()[1] == 128 and qq.stride()[2] == H * 128  # token-major storage
    assert vv.shape == (B, L, Hk * 128) and gg.shape == (B, L, H * 128)
    assert torch.ops.k2_native.swiglu_prepared(x, q, s, [1, 2], 4096).shape == (B, L, 4096)
    o, n = torch.ops.k2_native.residual_norm(x, _m(B, 1, K), x, _m(B, K), _m(B, K), 3, 1)
    assert o.shape == x.shape and n.shape == x.shape
    a = torch.ops.k2_fullgraph.kohaku_fa(_m(B, H, L, 128), _m(B, Hk, L, 128), _m(B, Hk, L, 128), None, None, True)
    assert a.shape == (B, L, H * 128)


def test_registry_lifecycle():
    w = torch.rand(64)
    N.add_binding(9001, 1, 0, [w], [w], [], 128, False, 1e-6, [], 1000.0, torch.empty(0), True)
    N.add_binding(9002, 4, 0, [w], [w], [], 128, False, 1e-6, [], 1000.0, torch.empty(0), True)
    N.set_lookahead(9001, [9002])
    N.set_route(3, 9001, 4096, 1)
    assert N._get(9001).tensors[0].dtype == torch.float32 and N._get(9001).lookahead == [9002]
    assert N.stats([9001, 9002]) == {}
    N.release_bindings([9001, 9002])
    with pytest.raises(RuntimeError, match="binding released"):
        N._get(9001)
    with pytest.raises(ValueError):
        N.add_binding(9003, 0, 1, [], [w, w], [], 64, True, 1e-6, [], 1000.0, torch.empty(0), True)
    with pytest.raises(ValueError):  # INT8 projection with float weights
        N.add_binding(9004, 0, 2, [], [w, w], [], 128, True, 1e-6, [], 1000.0, torch.empty(0), True)
    with pytest.raises(NotImplementedError):
        N.add_binding(9005, 0, 7, [], [w, w], [], 128, True, 1e-6, [], 1000.0, torch.empty(0), True)


def test_reference_contract_bindings_keep_the_checkpoint_format():
    """Format 1 (ConvRot group 64, per-channel fp32 scales), 2 (INT8) and 3
    (FP8 e4m3) bindings keep the checkpoint's own layout, zero-padded to the
    GEMM's 128 (registration touches no kernel)."""
    g = torch.Generator().manual_seed(3)
    n, k = 200, 1000
    packed = torch.randint(-128, 128, (n, k // 2), generator=g, dtype=torch.int8)
    ws = torch.rand(n, generator=g)
    bias = torch.randn(n, generator=g)
    N.add_binding(9101, 0, 1, [], [packed, ws, bias], [], 64, True, 1e-6, [], 1000.0, torch.empty(0), True)
    r = N._get(9101).ref
    assert N._get(9101).weight is None and r.format == 1 and r.group == 64 and (r.n, r.k) == (n, k)
    assert r.w.shape == (256, 512) and r.w.dtype == torch.int8 and r.padded
    assert torch.equal(r.w[:n, :k // 2], packed) and not r.w[n:].any() and not r.w[:, k // 2:].any()
    assert torch.equal(r.ws[:n], ws) and not r.ws[n:].any()
    assert torch.equal(r.bias[:n], bias)  # fp32 as k2_gemm4 receives it
    w8 = torch.randint(-127, 128, (256, 1024), generator=g, dtype=torch.int8)
    N.add_binding(9102, 0, 2, [], [w8, torch.rand(1), bias[:128].repeat(2)], [], 0, True, 1e-6, [], 1000.0,
                  torch.empty(0), True)
    r = N._get(9102).ref
    assert r.w.shape == (256, 1024) and not r.padded and r.ws.numel() == 1
    assert torch.equal(r.bias, bias[:128].repeat(2).to(torch.bfloat16).float())  # rounded to the x dtype
    w3 = torch.randn(128, 256, generator=g).to(torch.float8_e4m3fn)
    N.add_binding(9103, 0, 3, [], [w3, torch.tensor(0.5)], [], 0, True, 1e-6, [], 1000.0, torch.tensor([0.25]),
                  True)
    r = N._get(9103).ref
    assert r.w.dtype == torch.float8_e4m3fn and float(r.input_scale) == 0.25
    with pytest.raises(ValueError):  # INT4 with a group the ConvRot quantiser does not have
        N.add_binding(9104, 0, 1, [], [packed, ws], [], 32, True, 1e-6, [], 1000.0, torch.empty(0), True)
    x = _m(1, 7, 1024)
    N.add_binding(9105, 1, 0, [], [torch.rand(1024)], [], 0, False, 1e-6, [], 1000.0, torch.empty(0), True)
    N.add_binding(9106, 0, 1, [], [torch.zeros(128, 512, dtype=torch.int8), torch.rand(128)], [], 256, True, 1e-6,
                  [], 1000.0, torch.empty(0), True)
    q, s = torch.ops.k2_native.norm_quant(x, _m(1, 1024), _m(1, 1024), 9105, 9106, -1)
    assert q.shape == (7, 512) and q.dtype == torch.int8 and s.shape == (7, 1) and s.dtype == torch.float32
    N.release_bindings([9101, 9102, 9103, 9105, 9106])


def test_cpu_tensors_reach_no_kernel():
    x = torch.zeros(1, 4, 512, dtype=torch.bfloat16)
    with pytest.raises(NotImplementedError):
        torch.ops.k2_native.norm_quant(x, x[0], x[0], 1, 2, -1)


def test_void_shims_report_unsupported_input():
    """The reference's void exports launch nothing on unsupported input and
    leave a status (no GPU is touched: the check precedes any launch)."""
    from k2b._native import lib

    L = lib()
    L.k2b_shim_status(1)
    L.k2_quant4(None, None, None, 4, 512, 128, 2, None)         # group 128 (not a reference group)
    assert L.k2b_shim_status(1) == 1                               # cudaErrorInvalidValue
    L.k2_norm(None, None, None, None, None, 4, 512, 4, -1, 1, ctypes.c_float(1e-6), 1, None)  # fp16
    assert L.k2b_shim_status(0) == 1 and L.k2b_shim_status(1) == 1 and L.k2b_shim_status(0) == 0
    L.k2_elementwise(None, None, None, None, 16, 0, 0, 0, None)    # fp32
    L.k2_rope(None, None, None, None, None, 1, 4, 1, 1, 128, 1, 1, None)
    assert L.k2b_shim_status(1) == 1
