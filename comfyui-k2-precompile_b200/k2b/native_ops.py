"""The reference's torch operator surface, served by libk2b.

``torch.ops.k2_native.*`` keeps the schemas of native_runtime.cpp:576-591 and
``torch.ops.k2_fullgraph.kohaku_fa`` the one of KohakuKernelRouter/attention.py:
189-197, so graph code written against the reference (input_quant_ops.py:14-31,
graph_ops.py, graph_model.py:63-65) calls into the B200 kernels unchanged.
Every op has a fake (meta) implementation for torch.compile tracing, as the
reference registers in native_schedule.py:70-114 and input_quant_ops.py:34-42.

Weights are referenced by integer keys through the same registry calls the
reference's extension module exposes (``add_binding`` / ``release_bindings``,
native_runtime.cpp:528, 573).  Registration converts an INT4 projection
once into the GEMM's resident layout (weights are never streamed per call).

Data contract (the B200 build's, documented in the C header): packed
activations are uint8 codes viewed as int8 [M, K/2] with fp16 group-128 scales
[M, K/128] (the reference returns one fp32 scale per row); INT4 weights are
registered as packed [N, K/2] + fp16 [N, K/128] group scales (``group`` 128).

Only CUDA implementations are registered: a CPU tensor reaches no kernel and
torch raises, there is no eager fallback.
"""
from __future__ import annotations

import math
import threading
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import torch

from . import ops

HEAD_DIM = 128

# --------------------------------------------------------------- registry


@dataclass
class Binding:
    """One registered module (native_runtime.cpp:74-79)."""

    key: int
    kind: int          # 0 projection, 1 RMSNorm, 2 RoPE table, 3/4 bias / modulation add
    format: int        # 1: INT4 (the only projection format of this build)
    group: int
    fuse: bool
    eps: float
    axes: List[int]
    theta: float
    optimize_io: bool
    weight: Optional[ops.PreparedWeight] = None
    tensors: List[torch.Tensor] = field(default_factory=list)
    lookahead: List[int] = field(default_factory=list)
    routes: Dict[int, int] = field(default_factory=dict)
    stats: Dict[str, int] = field(default_factory=dict)

    def count(self, name: str) -> None:
        self.stats[name] = self.stats.get(name, 0) + 1


_records: Dict[int, Binding] = {}
_lock = threading.RLock()  # one process-wide lock, as native_runtime.cpp:81


def _get(key: int) -> Binding:
    with _lock:
        b = _records.get(int(key))
    if b is None:
        raise RuntimeError(f"Native K2 binding released: {key}")
    return b


def add_binding(key: int, kind: int, format: int, cpu: Sequence[torch.Tensor], gpu: Sequence[torch.Tensor],
                vbar: Sequence[int], group: int, fuse: bool, eps: float, axes: Sequence[int], theta: float,
                input_scale: torch.Tensor, optimize_io: bool) -> None:
    """Register module ``key`` (same arguments as native_runtime.cpp:528).

    kind 0: ``gpu`` = [packed INT4 int8/uint8 [N, K/2], fp16 group scales
    [N, K/128]] (format 1, group 128); converted once with prepare_weight.
    kind 1: ``gpu[0]`` = fp32 RMSNorm weight ("w+1" form).  kind 2: ``axes``
    and ``theta`` of the RoPE table.  kind 3/4: ``gpu[0]`` added to inputs.
    ``cpu``, ``vbar`` and ``input_scale`` describe host copies and
    virtual-memory staging of the reference's weight streaming; weights stay
    resident here, so they are accepted and not used."""
    del cpu, vbar, input_scale
    b = Binding(int(key), int(kind), int(format), int(group), bool(fuse), float(eps), [int(a) for a in axes],
                float(theta), bool(optimize_io))
    gpu = list(gpu)
    if b.kind == 0:
        if b.format != 1:
            raise NotImplementedError("only INT4 (format 1) projections are served by the B200 build")
        if b.group != ops.GROUP:
            raise ValueError(f"INT4 projections use group-{ops.GROUP} scales (got {b.group})")
        if len(gpu) > 2 and gpu[2] is not None:
            raise NotImplementedError("projection bias is not part of the W4A4 block path")
        packed, scales = gpu[0], gpu[1]
        if packed.dtype == torch.int8:
            packed = packed.view(torch.uint8)
        b.weight = ops.prepare_weight(packed.contiguous(), scales.to(torch.float16).contiguous())
    elif b.kind == 1:
        b.tensors = [gpu[0].to(torch.float32).contiguous()]
    elif b.kind in (3, 4):
        b.tensors = [gpu[0]]
    elif b.kind not in (2, 5):
        raise ValueError(f"unknown binding kind {kind}")
    with _lock:
        _records[b.key] = b


def release_bindings(keys: Sequence[int]) -> None:
    """Drop registered modules (native_runtime.cpp:573)."""
    with _lock:
        for k in keys:
            _records.pop(int(k), None)


def configure(kernels: str = "", epilogue: str = "", qk: str = "", aimdo: str = "") -> None:
    """The reference dlopens its kernel libraries here (native_runtime.cpp:514-522);
    libk2b is loaded on first use, so the paths are accepted and ignored."""
    del kernels, epilogue, qk, aimdo


def configure_joint(path: str = "") -> None:
    """native_runtime.cpp:523-527: the joint kernels are part of libk2b."""
    del path


def configure_norm_quant(path: str = "") -> None:
    """native_runtime.cpp:528: the fused norm_quant kernel is part of libk2b."""
    del path


def set_route(op: int, key: int, rows: int, path: int) -> None:
    """Recorded for API parity (native_runtime.cpp:429-432).  Every op here has
    exactly one (fused) route."""
    if not (0 <= op <= 3 and rows > 0 and path in (0, 1)):
        raise ValueError("Invalid kernel route")
    with _lock:
        _get(key).routes[int(op) * 1000000000000 + int(rows)] = int(path)


def finish_tuning(keys: Sequence[int]) -> None:
    """No prefetched weights to retire: weights are resident."""
    del keys


def set_lookahead(key: int, next_keys: Sequence[int]) -> None:
    _get(key).lookahead = [int(k) for k in next_keys]


def reset_stats(keys: Sequence[int]) -> None:
    with _lock:
        for k in keys:
            _get(k).stats.clear()


def stats(keys: Sequence[int]) -> Dict[str, int]:
    out: Dict[str, int] = {}
    with _lock:
        for k in keys:
            for name, v in _get(k).stats.items():
                out[name] = out.get(name, 0) + v
    return out


# ---------------------------------------------------------------- helpers


def _norm(key: int) -> Binding:
    b = _get(key)
    if b.kind != 1:
        raise RuntimeError(f"binding {key} is not an RMSNorm")
    return b


def _proj(key: int) -> Binding:
    b = _get(key)
    if b.kind != 0 or b.weight is None:
        raise RuntimeError(f"binding {key} is not an INT4 projection")
    return b


def _rows_len(x: torch.Tensor):
    K = int(x.shape[-1])
    rows = x.numel() // K
    length = int(x.shape[1]) if x.dim() == 3 else rows
    return rows, length, K


def _packed(qa: torch.Tensor, qs: torch.Tensor, K: int):
    if qa.dtype == torch.int8:
        qa = qa.view(torch.uint8)
    if qa.dtype != torch.uint8 or qs.dtype != torch.float16:
        raise RuntimeError("Invalid packed normalized activation (int8 codes + fp16 group scales expected)")
    rows = qa.numel() * 2 // K
    return qa.reshape(rows, K // 2), qs.reshape(rows, K // ops.GROUP)


def _linear_gated(x: torch.Tensor, key: int, gate: Optional[torch.Tensor], residual: Optional[torch.Tensor]):
    b = _proj(key)
    rows, length, K = _rows_len(x)
    xq, xs = ops.rotate_quant(x.reshape(rows, K).contiguous())
    n = b.weight.n
    shape = list(x.shape[:-1]) + [n]
    if gate is None:
        b.count("gemm")
        return ops.gemm_bf16(xq, xs, b.weight).reshape(shape)
    b.count("gated_gemm")
    g = gate.reshape(-1, n).contiguous()
    if g.shape[0] == 1 and rows // length > 1:
        g = g.expand(rows // length, n).contiguous()
    out = ops.gated_residual(xq, xs, b.weight, g, residual.reshape(rows, n).contiguous(), length=length)
    return out.reshape(residual.shape)


def _freqs_for(freqs: torch.Tensor, length: int) -> torch.Tensor:
    f = freqs.to(torch.float32).contiguous()
    if f.numel() != length * 64 * 4:
        raise RuntimeError("RoPE table must be batch-shared fp32 [.., L, 64, 2, 2]")
    return f.reshape(length, 64, 2, 2)


# ------------------------------------------------------------- op bodies


def _norm_quant(x, scale, shift, norm_key, target_key, cut):
    nb, tb = _norm(norm_key), _get(target_key)
    rows, length, K = _rows_len(x)
    if tb.format != 1 or tb.group != ops.GROUP or nb.tensors[0].numel() != K:
        raise RuntimeError("Normalized quantization requires compatible INT4 input")
    q, s = ops.norm_quant(x.reshape(rows, K).contiguous(), nb.tensors[0], scale.reshape(-1, K).contiguous(),
                          shift.reshape(-1, K).contiguous(), length=length, cut=int(cut), eps=nb.eps)
    nb.count("norm_quant_fused")
    return q.view(torch.int8), s


def _norm_mod(x, scale, shift, key, cut):
    nb = _norm(key)
    rows, length, K = _rows_len(x)
    y = ops.norm_mod(x.reshape(rows, K).contiguous(), nb.tensors[0], scale.reshape(-1, K).contiguous(),
                     shift.reshape(-1, K).contiguous(), length=length, cut=int(cut), eps=nb.eps)
    return y.reshape(x.shape)


def _gated(x, gate, residual, key):
    return _linear_gated(x, key, gate, residual)


def _gated_norm_quant(x, gate, residual, scale, shift, key, norm_key, target_key, cut):
    out = _linear_gated(x, key, gate, residual)
    q, s = _norm_quant(out, scale, shift, norm_key, target_key, cut)
    return out, q, s


def _residual_norm(x, gate, residual, scale, shift, key, norm_key):
    out = _linear_gated(x, key, gate, residual)
    return out, _norm_mod(out, scale, shift, norm_key, -1)


def _qkv_common(x, qa, qs, freqs, keys, norms, heads, kvheads):
    B, L = int(x.shape[0]), int(x.shape[1])
    K = int(x.shape[-1])
    a, s = _packed(qa, qs, K)
    wq, wk, wv, wg = (_proj(k) for k in keys)
    nq, nk = _norm(norms[0]), _norm(norms[1])
    if wq.weight.n != heads * HEAD_DIM or wk.weight.n != kvheads * HEAD_DIM or wv.weight.n != kvheads * HEAD_DIM:
        raise RuntimeError("qkv weight widths do not match heads / kvheads")
    q, k, v, g = ops.qkv(a, s, wq.weight, wk.weight, wv.weight, nq.tensors[0], nk.tensors[0],
                         _freqs_for(freqs, L), length=L, eps_q=nq.eps, eps_k=nk.eps, wg=wg.weight)
    wq.count("prepared_qkv")
    # token-major storage viewed as [B, H, L, D] (native_runtime.cpp:413-422)
    q = q.view(B, L, heads, HEAD_DIM).transpose(1, 2)
    k = k.view(B, L, kvheads, HEAD_DIM).transpose(1, 2)
    return q, k, v.view(B, L, kvheads * HEAD_DIM), g.view(B, L, heads * HEAD_DIM)


def _qkv_prepared(x, qa, qs, freqs, keys, norms, heads, kvheads):
    return _qkv_common(x, qa, qs, freqs, keys, norms, heads, kvheads)


def _joint_qkv(x, freqs, keys, norms, heads, kvheads):
    rows, _, K = _rows_len(x)
    qa, qs = ops.rotate_quant(x.reshape(rows, K).contiguous())
    return _qkv_common(x, qa, qs, freqs, keys, norms, heads, kvheads)


def _swiglu_common(x, qa, qs, keys, width):
    K = int(x.shape[-1])
    a, s = _packed(qa, qs, K)
    wg, wu = _proj(keys[0]), _proj(keys[1])
    if wg.weight.n != width or wu.weight.n != width:
        raise RuntimeError("Joint SwiGLU weight contract changed")
    wg.count("prepared_swiglu")
    return ops.swiglu_bf16(a, s, wg.weight, wu.weight).reshape(list(x.shape[:-1]) + [width])


def _swiglu_prepared(x, qa, qs, keys, width):
    return _swiglu_common(x, qa, qs, keys, width)


def _joint_swiglu(x, keys, width):
    rows, _, K = _rows_len(x)
    qa, qs = ops.rotate_quant(x.reshape(rows, K).contiguous())
    return _swiglu_common(x, qa, qs, keys, width)


def _project_many(x, keys, widths):
    outs = [_linear_gated(x, k, None, None) for k in keys]
    for o, w in zip(outs, widths):
        if o.shape[-1] != w:
            raise RuntimeError("projection width mismatch")
    return outs


def _attention_inputs(x, freqs, keys, widths, norms, heads, kvheads):
    if freqs is None or len(norms) != 2:
        outs = _project_many(x, keys, widths)
        return outs[0], outs[1], outs[2], outs[3]
    return _joint_qkv(x, freqs, keys, norms, heads, kvheads)


def _sdpa(q, k, v, enable_gqa):
    return ops.attention(q, k, v)


def _managed(x, key, kind, width):
    b = _get(key)
    if kind == 0:
        return _linear_gated(x, key, None, None)
    if kind == 1:
        rows, _, K = _rows_len(x)
        return ops.norm_mod(x.reshape(rows, K).contiguous(), b.tensors[0], eps=b.eps).reshape(x.shape)
    if kind == 3:
        return x + b.tensors[0].to(x.dtype).unsqueeze(0)
    if kind == 4:
        return x + b.tensors[0].to(x.dtype)
    if kind == 5:
        return torch.nn.functional.gelu(x, approximate="tanh")
    # kind 2: EmbedND table (native_runtime.cpp:508-510): per axis d,
    # omega = theta^-linspace(0, (d-2)/d, d/2), angle = pos * omega
    pieces = []
    for i, d in enumerate(b.axes):
        pos = x.select(-1, i)
        scale = torch.linspace(0.0, (d - 2) / d, d // 2, dtype=torch.float64, device=x.device)
        omega = torch.reciprocal(torch.pow(torch.tensor(b.theta, dtype=torch.float64, device=x.device), scale))
        angle = pos.to(torch.float32).unsqueeze(-1) * omega
        c, s = angle.cos(), angle.sin()
        pieces.append(torch.stack([c, -s, s, c], -1).reshape(*angle.shape, 2, 2).to(torch.float32))
    return torch.cat(pieces, -3).unsqueeze(1)


def _activation(x, kind):
    return ops.elementwise(x.contiguous(), None, None, 0 if kind == "silu" else 1)


def _activate_mul(a, b, kind):
    return ops.elementwise(a.contiguous(), b.contiguous(), None, 0 if kind == "silu" else 1)


def _modulation(x, scale, shift):
    return (1 + scale) * x + shift


def _residual(x, gate, value):
    if gate.dim() > 0 and gate.numel() != gate.shape[-1]:
        return x + gate * value
    return ops.elementwise(gate.contiguous(), value.contiguous(), x.contiguous(), 2, int(gate.numel()))


def _rope(q, k, freqs):
    return ops.rope(q.contiguous(), k.contiguous(), freqs)


def _timestep(t, dim):
    t = t * 1000.0
    freq = torch.exp(-math.log(10000.0) * torch.arange(dim // 2, dtype=torch.float32, device=t.device) / (dim // 2))
    args = t.to(torch.float32).unsqueeze(-1) * freq.unsqueeze(0)
    out = torch.cat([args.cos(), args.sin()], -1)
    if dim % 2:
        out = torch.cat([out, torch.zeros_like(out[..., :1])], -1)
    return out.to(t.dtype) if t.is_floating_point() else out


# ----------------------------------------------------------- registration

SCHEMAS = {
    "norm_quant": "norm_quant(Tensor x, Tensor scale, Tensor shift, int norm_key, int target_key, int cut) -> (Tensor, Tensor)",
    "gated_norm_quant": "gated_norm_quant(Tensor x, Tensor gate, Tensor residual, Tensor scale, Tensor shift, int key, int norm_key, int target_key, int cut) -> (Tensor, Tensor, Tensor)",
    "qkv_prepared": "qkv_prepared(Tensor x, Tensor qa, Tensor qs, Tensor freqs, int[] keys, int[] norms, int heads, int kvheads) -> (Tensor, Tensor, Tensor, Tensor)",
    "swiglu_prepared": "swiglu_prepared(Tensor x, Tensor qa, Tensor qs, int[] keys, int width) -> Tensor",
    "sdpa": "sdpa(Tensor q, Tensor k, Tensor v, bool enable_gqa) -> Tensor",
    "managed": "managed(Tensor x, int key, int kind, int width) -> Tensor",
    "gated": "gated(Tensor x, Tensor gate, Tensor residual, int key) -> Tensor",
    "norm_mod": "norm_mod(Tensor x, Tensor scale, Tensor shift, int key, int cut) -> Tensor",
    "project_many": "project_many(Tensor x, int[] keys, int[] widths) -> Tensor[]",
    "attention_inputs": "attention_inputs(Tensor x, Tensor? freqs, int[] keys, int[] widths, int[] norms, int heads, int kvheads) -> (Tensor, Tensor, Tensor, Tensor)",
    "residual_norm": "residual_norm(Tensor x, Tensor gate, Tensor residual, Tensor scale, Tensor shift, int key, int norm_key) -> (Tensor, Tensor)",
    "joint_swiglu": "joint_swiglu(Tensor x, int[] keys, int width) -> Tensor",
    "joint_qkv": "joint_qkv(Tensor x, Tensor freqs, int[] keys, int[] norms, int heads, int kvheads) -> (Tensor, Tensor, Tensor, Tensor)",
    "activation": "activation(Tensor x, str kind) -> Tensor",
    "activate_mul": "activate_mul(Tensor a, Tensor b, str kind) -> Tensor",
    "modulation": "modulation(Tensor x, Tensor scale, Tensor shift) -> Tensor",
    "residual": "residual(Tensor x, Tensor gate, Tensor value) -> Tensor",
    "rope": "rope(Tensor q, Tensor k, Tensor freqs) -> (Tensor, Tensor)",
    "timestep": "timestep(Tensor t, int dim) -> Tensor",
}

IMPLS = {
    "norm_quant": _norm_quant, "gated_norm_quant": _gated_norm_quant, "qkv_prepared": _qkv_prepared,
    "swiglu_prepared": _swiglu_prepared, "sdpa": _sdpa, "managed": _managed, "gated": _gated, "norm_mod": _norm_mod,
    "project_many": _project_many, "attention_inputs": _attention_inputs, "residual_norm": _residual_norm,
    "joint_swiglu": _joint_swiglu, "joint_qkv": _joint_qkv, "activation": _activation, "activate_mul": _activate_mul,
    "modulation": _modulation, "residual": _residual, "rope": _rope, "timestep": _timestep,
}


def _e(shape, like, dtype=None):
    return torch.empty(shape, device=like.device, dtype=like.dtype if dtype is None else dtype)


def _fake_packed(x):
    rows, K = math.prod(x.shape[:-1]), x.shape[-1]
    return _e((rows, K // 2), x, torch.int8), _e((rows, K // ops.GROUP), x, torch.float16)


def _fake_qkv(x, heads, kvheads):
    B, L = x.shape[0], x.shape[1]
    q = _e((B, L, heads, HEAD_DIM), x).transpose(1, 2)
    k = _e((B, L, kvheads, HEAD_DIM), x).transpose(1, 2)
    return q, k, _e((B, L, kvheads * HEAD_DIM), x), _e((B, L, heads * HEAD_DIM), x)


def _fake_width(x, key):
    b = _records.get(int(key))
    if b is None or b.weight is None:
        raise RuntimeError(f"Native K2 binding released: {key}")
    return b.weight.n


FAKES = {
    "norm_quant": lambda x, scale, shift, norm_key, target_key, cut: _fake_packed(x),
    "gated_norm_quant": lambda x, gate, residual, scale, shift, key, norm_key, target_key, cut:
        (torch.empty_like(residual, memory_format=torch.contiguous_format), *_fake_packed(residual)),
    "qkv_prepared": lambda x, qa, qs, freqs, keys, norms, heads, kvheads: _fake_qkv(x, heads, kvheads),
    "swiglu_prepared": lambda x, qa, qs, keys, width: _e(tuple(x.shape[:-1]) + (width,), x),
    "sdpa": lambda q, k, v, enable_gqa: _e((q.shape[0], q.shape[2], q.shape[1] * q.shape[3]), q),
    "managed": lambda x, key, kind, width: (_e(tuple(x.shape[:-1]) + (width,), x) if kind == 0 else
                                            torch.empty_like(x, memory_format=torch.contiguous_format)),
    "gated": lambda x, gate, residual, key: torch.empty_like(residual),
    "norm_mod": lambda x, scale, shift, key, cut: torch.empty_like(x, memory_format=torch.contiguous_format),
    "project_many": lambda x, keys, widths: [_e(tuple(x.shape[:-1]) + (w,), x) for w in widths],
    "attention_inputs": lambda x, freqs, keys, widths, norms, heads, kvheads: _fake_qkv(x, heads, kvheads),
    "residual_norm": lambda x, gate, residual, scale, shift, key, norm_key:
        (torch.empty_like(residual, memory_format=torch.contiguous_format),
         torch.empty_like(residual, memory_format=torch.contiguous_format)),
    "joint_swiglu": lambda x, keys, width: _e(tuple(x.shape[:-1]) + (width,), x),
    "joint_qkv": lambda x, freqs, keys, norms, heads, kvheads: _fake_qkv(x, heads, kvheads),
    "activation": lambda x, kind: torch.empty_like(x),
    "activate_mul": lambda a, b, kind: torch.empty_like(a),
    "modulation": lambda x, scale, shift: torch.empty_like(x, memory_format=torch.contiguous_format),
    "residual": lambda x, gate, value: torch.empty_like(x, memory_format=torch.contiguous_format),
    "rope": lambda q, k, freqs: (torch.empty(q.shape, device=q.device, dtype=q.dtype),
                                 torch.empty(k.shape, device=k.device, dtype=k.dtype)),
    "timestep": lambda t, dim: _e(tuple(t.shape) + (dim,), t, t.dtype if t.is_floating_point() else torch.float32),
}

_library = torch.library.Library("k2_native", "DEF")
for _name, _schema in SCHEMAS.items():
    _library.define(_schema)
    _library.impl(_name, IMPLS[_name], "CUDA")
    torch.library.register_fake("k2_native::" + _name)(FAKES[_name])


@torch.library.custom_op("k2_fullgraph::kohaku_fa", mutates_args=(), device_types="cuda")
def kohaku_fa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: Optional[torch.Tensor],
              gate: Optional[torch.Tensor], gate_is_sigmoid: bool) -> torch.Tensor:
    """GQA flash attention (KohakuKernelRouter/attention.py:189-193):
    q [B,Hq,L,D], k/v [B,Hkv,Lk,D] -> bf16 [B, L, Hq*D]; optional gate of the
    output's shape (pre-sigmoided when gate_is_sigmoid).  Masks are rejected."""
    return ops.attention(q, k, v, mask=mask, gate=gate, gate_is_sigmoid=gate_is_sigmoid)


@kohaku_fa.register_fake
def _kohaku_fa_fake(q, k, v, mask, gate, gate_is_sigmoid):
    return torch.empty((q.shape[0], q.shape[2], q.shape[1] * q.shape[3]), device=q.device, dtype=q.dtype)


__all__ = ["Binding", "add_binding", "release_bindings", "configure", "configure_joint", "configure_norm_quant",
           "set_route", "finish_tuning", "set_lookahead", "reset_stats", "stats", "kohaku_fa", "SCHEMAS"]
