"""The reference's torch operator surface, served by libk2b.

``torch.ops.k2_native.*`` keeps the schemas of native_runtime.cpp:576-591 and
``torch.ops.k2_fullgraph.kohaku_fa`` the one of KohakuKernelRouter/attention.py:
189-197, so graph code written against the reference (input_quant_ops.py:14-31,
graph_ops.py, graph_model.py:63-65) calls into the B200 kernels unchanged.
Every op has a fake (meta) implementation for torch.compile tracing, as the
reference registers in native_schedule.py:70-114 and input_quant_ops.py:34-42.

Weights are referenced by integer keys through the same registry calls the
reference's extension module exposes (``add_binding`` / ``release_bindings``,
native_runtime.cpp:528, 573).  A projection binding is served in one of two
data contracts, chosen from what is registered:

* the reference's own (``Binding.ref``): format 1 INT4 with ConvRot groups
  16/64/256, packed [N, K/2] weights and fp32 per-channel scales [N]; format
  2 INT8 [N, K]; formats 3/4 FP8 e4m3/e5m2 [N, K] with their scale; format 0
  plain weights.  Activations are quantised per row with one fp32 scale
  ([M, 1]) exactly as the reference's runtime quantises them
  (native_runtime.cpp:266-285) and projected by the tcgen05 GEMM with the
  whole of K in one accumulator (k2b.ref_ops);
* group-128 W4A4 (``Binding.weight``): format 1, group 128 and fp16 group
  scales [N, K/128]; converted once into the GEMM's resident layout; packed
  activations carry fp16 group-128 scales [M, K/128].

Only CUDA implementations are registered: a CPU tensor reaches no kernel and
torch raises, there is no eager fallback.
"""
from __future__ import annotations

import math
import threading
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

from . import ops, ref_ops

HEAD_DIM = 128

# --------------------------------------------------------------- registry


@dataclass
class RefWeight:
    """A projection kept in the checkpoint's own format (reference contract).

    ``w``: int8 packed [np, kp/2] (format 1), int8 [np, kp] (format 2), fp8
    [np, kp] (3/4) or the plain weight [n, k] (format 0), where np / kp are n
    and k rounded up to the GEMM's 128 with zero rows / columns (zero codes
    add nothing to an accumulator; padded output columns are dropped).
    ``ws``: fp32 per-channel [np] or single [1] scale.  ``bias``: fp32 [np],
    rounded the way the reference hands it to the kernel of this format."""

    format: int
    group: int
    w: torch.Tensor
    ws: Optional[torch.Tensor]
    bias: Optional[torch.Tensor]
    input_scale: Optional[torch.Tensor]
    n: int
    k: int

    w8_: Optional[torch.Tensor] = None

    @property
    def padded(self) -> bool:
        return self.format != 0 and (self.n % 128 != 0 or self.k % 128 != 0)

    def codes8(self) -> torch.Tensor:
        """Format 1: the weight codes as e4m3 bytes [np, kp], expanded from the
        packed rows on first use and kept resident (the byte-operand GEMMs)."""
        if self.w8_ is None:
            self.w8_ = ref_ops.codes_e4m3(self.w)
        return self.w8_


@dataclass
class Binding:
    """One registered module (native_runtime.cpp:74-79)."""

    key: int
    kind: int          # 0 projection, 1 RMSNorm, 2 RoPE table, 3/4 bias / modulation add
    format: int        # 0 plain, 1 INT4, 2 INT8, 3 FP8 e4m3, 4 FP8 e5m2
    group: int
    fuse: bool
    eps: float
    axes: List[int]
    theta: float
    optimize_io: bool
    weight: Optional[ops.PreparedWeight] = None
    ref: Optional[RefWeight] = None
    loras: List[Tuple[torch.Tensor, torch.Tensor, float]] = field(default_factory=list)
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


def _pad_rows_cols(t: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    """t [r, c] zero-padded to [rows, cols] (byte view for fp8 / int8)."""
    if tuple(t.shape) == (rows, cols):
        return t.contiguous()
    raw = t.view(torch.uint8) if t.element_size() == 1 else t
    out = torch.zeros((rows, cols), dtype=raw.dtype, device=t.device)
    out[:t.shape[0], :t.shape[1]] = raw
    return out.view(t.dtype) if t.element_size() == 1 else out


def _ref_weight(fmt: int, group: int, gpu: List[torch.Tensor], input_scale: Optional[torch.Tensor]) -> RefWeight:
    """Reference-contract projection weights (native_runtime.cpp:286-311)."""
    w = gpu[0]
    bias = gpu[2] if len(gpu) > 2 and gpu[2] is not None and gpu[2].numel() else None
    if fmt == 0:
        b = None if bias is None else bias.to(torch.bfloat16).contiguous()
        return RefWeight(0, group, w.to(torch.bfloat16).contiguous(), None, b, None, int(w.shape[0]),
                         int(w.shape[1]))
    ws = gpu[1].to(torch.float32).contiguous().reshape(-1)
    n = int(w.shape[0])
    if fmt == 1:
        if group not in ref_ops.GROUPS4:
            raise ValueError(f"INT4 projections use ConvRot groups {ref_ops.GROUPS4} or group 128 (got {group})")
        if w.dtype not in (torch.int8, torch.uint8) or ws.numel() != n:
            raise ValueError("INT4 projection: packed int8 [N, K/2] + fp32 per-channel scales [N] expected")
        k = int(w.shape[1]) * 2
        wd = w.view(torch.int8)
    elif fmt == 2:
        if w.dtype != torch.int8 or ws.numel() not in (1, n) or group not in (0,) + ref_ops.GROUPS4:
            raise ValueError("INT8 projection: int8 [N, K] + fp32 scales [N] or [1], group 0/16/64/256")
        k = int(w.shape[1])
        wd = w
    elif fmt in ref_ops.FP8_FORMATS:
        if w.dtype != ref_ops.FP8_FORMATS[fmt][0] or ws.numel() not in (1, n):
            raise ValueError(f"FP8 projection (format {fmt}): {ref_ops.FP8_FORMATS[fmt][0]} [N, K] + fp32 scale")
        k = int(w.shape[1])
        wd = w
    else:
        raise NotImplementedError(f"projection format {fmt}")
    np_, kp = -(-n // 128) * 128, -(-k // 128) * 128
    wd = _pad_rows_cols(wd, np_, kp // 2 if fmt == 1 else kp)
    if ws.numel() == n and np_ != n:
        ws = torch.cat([ws, ws.new_zeros(np_ - n)])
    b = None
    if bias is not None:
        # gemm4 receives bias.to(fp32); the INT8 / FP8 routes bias.to(x dtype)
        b = bias.to(torch.float32) if fmt == 1 else bias.to(torch.bfloat16).to(torch.float32)
        b = torch.cat([b.reshape(-1), b.new_zeros(np_ - n)]).contiguous()
    isc = None
    if input_scale is not None and input_scale.numel():
        isc = input_scale.to(torch.float32).reshape(1).contiguous()
    return RefWeight(fmt, group, wd, ws, b, isc, n, k)


def add_binding(key: int, kind: int, format: int, cpu: Sequence[torch.Tensor], gpu: Sequence[torch.Tensor],
                vbar: Sequence[int], group: int, fuse: bool, eps: float, axes: Sequence[int], theta: float,
                input_scale: torch.Tensor, optimize_io: bool) -> None:
    """Register module ``key`` (same arguments as native_runtime.cpp:528).

    kind 0: ``gpu`` = [weight, weight scale, optional bias], in the
    checkpoint's format (format 0 plain; 1 INT4 packed [N, K/2] + fp32 [N]
    with ConvRot group 16/64/256; 2 INT8 [N, K] + fp32 [N] or [1]; 3/4 FP8
    [N, K] + fp32 scale, ``input_scale`` the static activation scale if
    non-empty).  Format 1 with group 128 and fp16 group scales [N, K/128]
    selects the group-128 W4A4 contract instead (converted once with
    prepare_weight; no bias).  kind 1: ``gpu[0]`` = fp32 RMSNorm weight ("w+1"
    form).  kind 2: ``axes`` and ``theta`` of the RoPE table.  kind 3/4:
    ``gpu[0]`` added to inputs.  ``cpu`` and ``vbar`` describe host copies and
    virtual-memory staging of the reference's weight streaming; weights stay
    resident here, so they are accepted and not used."""
    del cpu, vbar
    b = Binding(int(key), int(kind), int(format), int(group), bool(fuse), float(eps), [int(a) for a in axes],
                float(theta), bool(optimize_io))
    gpu = list(gpu)
    if b.kind == 0:
        scales = gpu[1] if len(gpu) > 1 else None
        group128 = (b.format == 1 and b.group == ops.GROUP and scales is not None and scales.dim() == 2 and
                    scales.dtype == torch.float16)
        if group128:
            if len(gpu) > 2 and gpu[2] is not None and gpu[2].numel():
                raise NotImplementedError("projection bias is not part of the group-128 W4A4 contract")
            packed = gpu[0]
            if packed.dtype == torch.int8:
                packed = packed.view(torch.uint8)
            b.weight = ops.prepare_weight(packed.contiguous(), scales.contiguous())
        else:
            b.ref = _ref_weight(b.format, b.group, gpu, input_scale)
    elif b.kind == 1:
        b.tensors = [gpu[0].to(torch.float32).contiguous()]
    elif b.kind in (3, 4):
        b.tensors = [gpu[0]]
    elif b.kind not in (2, 5):
        raise ValueError(f"unknown binding kind {kind}")
    with _lock:
        _records[b.key] = b


def set_loras(key: int, factors: Sequence[Tuple[torch.Tensor, torch.Tensor, float]]) -> None:
    """Attach LoRA bypass factors to projection ``key``: (up [N, r], down
    [r, K], strength), as NativePlan.register collects them from ComfyUI's
    bypass hooks (native_schedule.py:169-182; strength = alpha / r *
    multiplier).  The reference applies them after its native projection in
    Python (graph_ops.py:246-249: value + T(T(x down^T) up^T) * s, one factor
    after the other); here the first factor's up-projection is fused into the
    projection's epilogue (``k2b_lora_gemm``) and any further ones follow in
    that order.  Ops on bindings with factors take the per-projection routes,
    as the reference's graph does for them (graph_ops.py:439, 501, 520).  An
    empty list removes the factors.  Only a caller that does not also apply
    them itself should attach them."""
    b = _proj(key)
    n, K = _width(b), (b.weight.k if b.weight is not None else b.ref.k)
    out = []
    for up, down, strength in factors:
        r = int(down.shape[0])
        if tuple(up.shape) != (n, r) or tuple(down.shape) != (r, K):
            raise ValueError(f"LoRA factors must be up [{n}, r] and down [r, {K}]")
        rp = -(-r // 8) * 8  # zero-padded rank (zero columns add nothing)
        u = _pad_rows_cols(up.to(torch.bfloat16), n, rp)
        d = _pad_rows_cols(down.to(torch.bfloat16), rp, K)
        out.append((u, d, float(strength)))
    with _lock:
        b.loras = out


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
    if b.kind != 0 or (b.weight is None and b.ref is None):
        raise RuntimeError(f"binding {key} is not a projection")
    return b


def _width(b: Binding) -> int:
    return b.weight.n if b.weight is not None else b.ref.n


def _rows_len(x: torch.Tensor):
    K = int(x.shape[-1])
    rows = x.numel() // K
    length = int(x.shape[1]) if x.dim() == 3 else rows
    return rows, length, K


def _packed(qa: torch.Tensor, qs: torch.Tensor, K: int):
    """Group-128 packed activation: uint8 codes + fp16 [rows, K/128]."""
    if qa.dtype == torch.int8:
        qa = qa.view(torch.uint8)
    if qa.dtype != torch.uint8 or qs.dtype != torch.float16:
        raise RuntimeError("Invalid packed normalized activation (int8 codes + fp16 group scales expected)")
    rows = qa.numel() * 2 // K
    return qa.reshape(rows, K // 2), qs.reshape(rows, K // ops.GROUP)


def _ref_prepared(x: torch.Tensor, qa: torch.Tensor, qs: torch.Tensor, keys: Sequence[int]):
    """The reference's prepared_input checks (native_runtime.cpp:447-453):
    int8 codes [rows, K/2], one fp32 scale per row, every key INT4 of one
    ConvRot group."""
    if not (qa.dtype == torch.int8 and qs.dtype == torch.float32 and qa.is_contiguous() and qs.is_contiguous() and
            qa.device == x.device and qs.device == x.device and qa.numel() * 2 == x.numel() and
            qs.numel() == x.numel() // x.shape[-1]):
        raise RuntimeError("Invalid packed normalized activation")
    group = _get(keys[0]).group
    for k in keys:
        b = _get(k)
        if b.ref is None or b.format != 1 or b.group != group:
            raise RuntimeError("Packed input cannot be shared across incompatible quantization layouts")
    rows = qs.numel()
    return qa.reshape(rows, -1), qs.reshape(rows, 1)


def _freqs_for(freqs: torch.Tensor, length: int) -> torch.Tensor:
    f = freqs.to(torch.float32).contiguous()
    if f.numel() != length * 64 * 4:
        raise RuntimeError("RoPE table must be batch-shared fp32 [.., L, 64, 2, 2]")
    return f.reshape(length, 64, 2, 2)


# ----------------------------------------- reference contract (Binding.ref)


def _ref_q4(x2: torch.Tensor, group: int):
    """Per-row INT4 after ConvRot (k2_quant4's arithmetic), the codes as e4m3
    bytes when the width allows (the byte-operand GEMMs' container), else
    packed."""
    if x2.shape[1] % 512 == 0:
        return ref_ops.quant4_e4m3(x2, group)
    return ref_ops.quant4(x2, group)


def _codes(a: torch.Tensor) -> torch.Tensor:
    """INT4 codes as e4m3 bytes, expanding packed ones."""
    return a if a.dtype == torch.float8_e4m3fn else ref_ops.codes_e4m3(a)


def _ref_quantize(x2: torch.Tensor, r: RefWeight):
    """native_runtime.cpp:266-285: per-row INT4 / INT8 after ConvRot, or FP8
    with one scale (the binding's input scale, else amax / fmax)."""
    if r.format == 1:
        return _ref_q4(x2, r.group)
    if r.format == 2:
        return ref_ops.quant8(x2, r.group)
    scale = r.input_scale if r.input_scale is not None else ref_ops.fp8_scale(x2, r.format)
    return ref_ops.fp8_quant(x2, r.format, scale), scale


def _pad_k(q: torch.Tensor, r: RefWeight) -> torch.Tensor:
    kq = r.w.shape[1]
    if q.shape[1] == kq:
        return q
    return _pad_rows_cols(q, q.shape[0], kq)


def _ref_project(x2: torch.Tensor, r: RefWeight, q=None) -> torch.Tensor:
    """T(acc * xs * ws [+ bias]) of rows x2 bf16 [m, K] (native_runtime.cpp:
    286-311), bf16 [m, n]."""
    if r.format == 0:
        return torch.nn.functional.linear(x2, r.w, r.bias)
    qa, qs = _ref_quantize(x2, r) if q is None else q
    if r.format == 1:
        a8 = qa if qa.dtype == torch.float8_e4m3fn else ref_ops.codes_e4m3(_pad_k(qa, r))
        out = ref_ops.gemm_f8(a8, qs.reshape(-1), r.codes8(), r.ws, r.bias)
        return out[:, :r.n] if out.shape[1] != r.n else out
    qa = _pad_k(qa, r)
    if r.format == 2:
        out = ref_ops.gemm8(qa, qs.reshape(-1), r.w, r.ws, r.bias)
    else:
        out = ref_ops.gemm_f8(qa, qs.reshape(-1), r.w, r.ws, r.bias)
    return out[:, :r.n] if out.shape[1] != r.n else out


def _ref_cache_key(b: Binding, i: int):
    """Bindings that quantise the input alike share one quantisation
    (native_runtime.cpp:336-340)."""
    if not b.fuse:
        return ("own", i)
    isc = b.ref.input_scale
    return (b.format, b.group, None if isc is None else isc.data_ptr())


def _linear(x: torch.Tensor, key: int, gate: Optional[torch.Tensor] = None,
            residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """native_runtime.cpp:325-332: one projection, optionally
    out = T(residual + T(T(p) * gate)) (fused into the GEMM for INT4)."""
    b = _proj(key)
    if b.loras:
        return _linear_lora(x, b, gate, residual)
    if b.weight is not None:
        return _linear_gated(x, key, gate, residual)
    r = b.ref
    rows, length, K = _rows_len(x)
    x2 = x.reshape(rows, K).contiguous()
    shape = list(x.shape[:-1]) + [r.n]
    if gate is not None and r.format == 1 and b.fuse and r.bias is None and not r.padded:
        g = gate.reshape(-1, r.n).contiguous()
        if g.shape[0] == 1 and rows // length > 1:
            g = g.expand(rows // length, r.n).contiguous()
        qa, qs = _ref_q4(x2, r.group)
        b.count("gated_gemm")
        out = ref_ops.gated_residual8(_codes(qa), qs.reshape(-1), r.codes8(), r.ws, g,
                                      residual.reshape(rows, r.n).contiguous(), length=length)
        return out.reshape(residual.shape)
    out = _ref_project(x2, r).reshape(shape)
    b.count("gemm")
    if gate is None:
        return out
    if gate.dim() > 0 and gate.numel() != gate.shape[-1]:
        return residual + gate * out
    return ops.elementwise(gate.contiguous(), out.contiguous(), residual.contiguous(), 2, int(gate.numel()))


def _linear_lora(x: torch.Tensor, b: Binding, gate: Optional[torch.Tensor], residual: Optional[torch.Tensor]):
    """A projection with LoRA bypass factors (graph_ops.py:246-249): the first
    factor pair's up-projection runs in the projection's epilogue (and with a
    single factor the gated residual too); t = T(x down^T) is the rank-r
    product of the bf16 input, a plain library GEMM as in the reference."""
    rows, length, K = _rows_len(x)
    x2 = x.reshape(rows, K).contiguous()
    n = _width(b)
    up0, down0, s0 = b.loras[0]
    t0 = F.linear(x2, down0)
    fuse_gate = gate is not None and len(b.loras) == 1
    g = None
    if fuse_gate:
        g = gate.reshape(-1, n).contiguous()
        if g.shape[0] == 1 and rows // length > 1:
            g = g.expand(rows // length, n).contiguous()
        res = residual.reshape(rows, n).contiguous()
    r = b.ref
    if b.weight is not None:
        a, sa = ops.rotate_quant(x2)
        out = ops.lora_gemm(a, sa, b.weight, t0, up0, s0, g if fuse_gate else None, res if fuse_gate else None,
                            length=length)
    elif r.format == 1 and not r.padded and not (fuse_gate and r.bias is not None):
        qa, qs = ref_ops.quant4(x2, r.group)
        out = ref_ops.lora_gemm4(qa, qs.reshape(-1), r.w, r.ws, t0, up0, s0, r.bias, g if fuse_gate else None,
                                 res if fuse_gate else None, length=length)
    else:
        out = _ref_project(x2, r) + F.linear(t0, up0) * s0
        fuse_gate = False
    for up, down, st in b.loras[1:]:
        out = out + F.linear(F.linear(x2, down), up) * st
    b.count("lora_gemm")
    if fuse_gate:
        return out.reshape(residual.shape)
    out = out.reshape(list(x.shape[:-1]) + [n])
    return out if gate is None else residual + gate * out


def _no_lora(bs: Sequence[Binding]) -> None:
    """The prepared-input ops receive only the packed normalised activation
    (x is metadata, input_quant_ops.py:23-31): a LoRA delta needs the bf16
    input, so bindings with factors are refused there rather than run without
    them (the reference's graph routes such projections per module)."""
    if any(b.loras for b in bs):
        raise RuntimeError("LoRA factors need the bf16 input: use joint_qkv / joint_swiglu / managed for these keys")


def _all_int4(bs: Sequence[Binding]) -> bool:
    g = bs[0].group
    return all(b.ref is not None and b.format == 1 and b.group == g and b.ref.bias is None and not b.ref.padded
               and not b.loras for b in bs)


def _group(x: torch.Tensor, keys: Sequence[int], prepared=None) -> List[torch.Tensor]:
    """Plain projections of x by each key (native_runtime.cpp:333-358), bf16
    [rows, n]; one quantisation per input layout."""
    rows, _, K = _rows_len(x)
    x2 = x.reshape(rows, K).contiguous()
    cache = {}
    outs = []
    for i, key in enumerate(keys):
        b = _proj(key)
        if b.loras:
            outs.append(_linear(x, key).reshape(rows, -1))
            continue
        if b.weight is not None:
            if ("b128",) not in cache:
                cache[("b128",)] = ops.rotate_quant(x2) if prepared is None else prepared
            a, sa = cache[("b128",)]
            outs.append(ops.gemm_bf16(a, sa, b.weight))
            continue
        ck = _ref_cache_key(b, i)
        if b.format != 0 and ck not in cache:
            cache[ck] = _ref_quantize(x2, b.ref) if prepared is None else prepared
        outs.append(_ref_project(x2, b.ref, cache.get(ck)))
    return outs


def _head_norm(p: torch.Tensor, B: int, L: int, nb: Binding) -> torch.Tensor:
    """Per-head RMSNorm of a projection [B*L, H*128] -> [B, H, L, 128]
    (native_runtime.cpp:352-354)."""
    h = p.shape[-1] // HEAD_DIM
    y = ops.norm_mod(p.reshape(B * L * h, HEAD_DIM).contiguous(), nb.tensors[0], eps=nb.eps)
    return y.view(B, L, h, HEAD_DIM).transpose(1, 2)


def _split_qkv(x, keys, norms, freqs, heads, kvheads, prepared=None, sigmoid_gate=True):
    """The reference's split route: group projections, per-head norm, RoPE
    (native_runtime.cpp:333-358, 460-478)."""
    B, L = int(x.shape[0]), int(x.shape[1])
    p = _group(x, keys, prepared)
    nq, nk = _norm(norms[0]), _norm(norms[1])
    q = _head_norm(p[0], B, L, nq)
    k = _head_norm(p[1], B, L, nk)
    if freqs is not None:
        fb = freqs.to(torch.float32).contiguous()
        q, k = ops.rope(q.contiguous(), k.contiguous(), fb)
    g = p[3] if len(p) > 3 else None
    if g is not None and sigmoid_gate:
        g = ops.elementwise(g.contiguous(), None, None, 1)
    v = p[2].view(B, L, -1)
    return q, k, v, None if g is None else g.view(B, L, -1)


def _ref_qkv(x, qa, qs, freqs, keys, norms, heads, kvheads, sigmoid_gate=True):
    """Joint INT4 QKV over the reference contract (kernels/joint_projection.cu:
    222-225 semantics): Q/K RMSNorm + RoPE in the epilogue, V plain, the gate
    sigmoided."""
    B, L = int(x.shape[0]), int(x.shape[1])
    bs = [_proj(k) for k in keys]
    nq, nk = _norm(norms[0]), _norm(norms[1])
    a8 = _codes(qa)
    ws = [b.ref.ws for b in bs]
    q, k, v, g = ref_ops.qkv8(a8, qs.reshape(-1), [b.ref.codes8() for b in bs[:4 if sigmoid_gate else 3]],
                              ws[:4 if sigmoid_gate else 3], nq.tensors[0], nk.tensors[0], _freqs_for(freqs, L),
                              length=L, eps_q=nq.eps, eps_k=nk.eps)
    if not sigmoid_gate:
        g = ref_ops.gemm_f8(a8, qs.reshape(-1), bs[3].ref.codes8(), ws[3])
    return (q.view(B, L, heads, HEAD_DIM).transpose(1, 2), k.view(B, L, kvheads, HEAD_DIM).transpose(1, 2),
            v.view(B, L, kvheads * HEAD_DIM), None if g is None else g.view(B, L, heads * HEAD_DIM))


# ----------------------------------------- group-128 contract (Binding.weight)


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


def _b128_qkv(x, a, s, freqs, keys, heads, kvheads, norms, sigmoid_gate=True):
    B, L = int(x.shape[0]), int(x.shape[1])
    wq, wk, wv, wg = (_proj(k) for k in keys)
    nq, nk = _norm(norms[0]), _norm(norms[1])
    if wq.weight.n != heads * HEAD_DIM or wk.weight.n != kvheads * HEAD_DIM or wv.weight.n != kvheads * HEAD_DIM:
        raise RuntimeError("qkv weight widths do not match heads / kvheads")
    q, k, v, g = ops.qkv(a, s, wq.weight, wk.weight, wv.weight, nq.tensors[0], nk.tensors[0],
                         _freqs_for(freqs, L), length=L, eps_q=nq.eps, eps_k=nk.eps,
                         wg=wg.weight if sigmoid_gate else None)
    if not sigmoid_gate:
        g = ops.gemm_bf16(a, s, wg.weight)
    # token-major storage viewed as [B, H, L, D] (native_runtime.cpp:413-422)
    q = q.view(B, L, heads, HEAD_DIM).transpose(1, 2)
    k = k.view(B, L, kvheads, HEAD_DIM).transpose(1, 2)
    return q, k, v.view(B, L, kvheads * HEAD_DIM), g.view(B, L, heads * HEAD_DIM)


# ------------------------------------------------------------- op bodies


def _norm_quant(x, scale, shift, norm_key, target_key, cut):
    nb, tb = _norm(norm_key), _get(target_key)
    rows, length, K = _rows_len(x)
    if tb.kind != 0 or tb.format != 1 or nb.tensors[0].numel() != K:
        raise RuntimeError("Normalized quantization requires compatible INT4 input")
    x2 = x.reshape(rows, K).contiguous()
    sc, sh = scale.reshape(-1, K).contiguous(), shift.reshape(-1, K).contiguous()
    if tb.ref is not None:
        q, s = ref_ops.norm_quant4(x2, nb.tensors[0], sc, sh, length=length, cut=int(cut), eps=nb.eps,
                                   group=tb.group)
        nb.count("norm_quant_fused")
        return q, s
    q, s = ops.norm_quant(x2, nb.tensors[0], sc, sh, length=length, cut=int(cut), eps=nb.eps)
    nb.count("norm_quant_fused")
    return q.view(torch.int8), s


def _norm_mod(x, scale, shift, key, cut):
    nb = _norm(key)
    rows, length, K = _rows_len(x)
    y = ops.norm_mod(x.reshape(rows, K).contiguous(), nb.tensors[0], scale.reshape(-1, K).contiguous(),
                     shift.reshape(-1, K).contiguous(), length=length, cut=int(cut), eps=nb.eps)
    return y.reshape(x.shape)


def _gated(x, gate, residual, key):
    return _linear(x, key, gate, residual)


def _gated_norm_quant(x, gate, residual, scale, shift, key, norm_key, target_key, cut):
    out = _linear(x, key, gate, residual)
    q, s = _norm_quant(out, scale, shift, norm_key, target_key, cut)
    return out, q, s


def _residual_norm(x, gate, residual, scale, shift, key, norm_key):
    out = _linear(x, key, gate, residual)
    return out, _norm_mod(out, scale, shift, norm_key, -1)


def _qkv_prepared(x, qa, qs, freqs, keys, norms, heads, kvheads):
    bs = [_proj(k) for k in keys]
    bs[0].count("prepared_qkv")
    _no_lora(bs)
    if qs.dtype == torch.float32:
        a, s = _ref_prepared(x, qa, qs, keys)
        if _all_int4(bs):
            return _ref_qkv(x, a, s, freqs, keys, norms, heads, kvheads)
        return _split_qkv(x, keys, norms, freqs, heads, kvheads, prepared=(a, s))
    a, s = _packed(qa, qs, int(x.shape[-1]))
    return _b128_qkv(x, a, s, freqs, keys, heads, kvheads, norms)


def _joint_qkv(x, freqs, keys, norms, heads, kvheads):
    bs = [_proj(k) for k in keys]
    rows, _, K = _rows_len(x)
    if any(b.loras for b in bs):
        return _split_qkv(x, keys, norms, freqs, heads, kvheads)
    if all(b.weight is not None for b in bs):
        a, s = ops.rotate_quant(x.reshape(rows, K).contiguous())
        bs[0].count("joint_qkv")
        return _b128_qkv(x, a, s, freqs, keys, heads, kvheads, norms)
    if _all_int4(bs):
        a, s = _ref_q4(x.reshape(rows, K).contiguous(), bs[0].group)
        bs[0].count("joint_qkv")
        return _ref_qkv(x, a, s, freqs, keys, norms, heads, kvheads)
    bs[0].count("routed_qkv_split")
    return _split_qkv(x, keys, norms, freqs, heads, kvheads)


def _swiglu_lora(x, keys, width):
    """SwiGLU over bindings with LoRA factors: with group-128 weights and at
    most one factor pair each, both deltas run in the SwiGLU GEMM's epilogue;
    otherwise the per-projection route of the reference (graph_model.py:15-19)."""
    wg, wu = _proj(keys[0]), _proj(keys[1])
    rows, _, K = _rows_len(x)
    shape = list(x.shape[:-1]) + [width]
    if wg.weight is not None and wu.weight is not None and len(wg.loras) <= 1 and len(wu.loras) <= 1:
        x2 = x.reshape(rows, K).contiguous()
        a, s = ops.rotate_quant(x2)
        lo = [None if not b.loras else (F.linear(x2, b.loras[0][1]), b.loras[0][0], b.loras[0][2]) for b in (wg, wu)]
        wg.count("lora_swiglu")
        return ops.lora_swiglu(a, s, wg.weight, wu.weight, lo[0], lo[1]).reshape(shape)
    pg, pu = _group(x, keys)
    return ops.elementwise(pg.contiguous(), pu.contiguous(), None, 0).reshape(shape)


def _swiglu_common(x, a, s, keys, width):
    wg, wu = _proj(keys[0]), _proj(keys[1])
    if _width(wg) != width or _width(wu) != width:
        raise RuntimeError("Joint SwiGLU weight contract changed")
    shape = list(x.shape[:-1]) + [width]
    if wg.weight is not None and wu.weight is not None:
        return ops.swiglu_bf16(a, s, wg.weight, wu.weight).reshape(shape)
    if _all_int4([wg, wu]):
        return ref_ops.swiglu8(_codes(a), s.reshape(-1), wg.ref.codes8(), wg.ref.ws, wu.ref.codes8(),
                               wu.ref.ws).reshape(shape)
    raise RuntimeError("Joint SwiGLU weight contract changed")


def _swiglu_prepared(x, qa, qs, keys, width):
    _proj(keys[0]).count("prepared_swiglu")
    _no_lora([_proj(k) for k in keys])
    if qs.dtype == torch.float32:
        a, s = _ref_prepared(x, qa, qs, keys)
    else:
        a, s = _packed(qa, qs, int(x.shape[-1]))
    return _swiglu_common(x, a, s, keys, width)


def _joint_swiglu(x, keys, width):
    rows, _, K = _rows_len(x)
    bs = [_proj(k) for k in keys]
    x2 = x.reshape(rows, K).contiguous()
    if any(b.loras for b in bs):
        return _swiglu_lora(x, keys, width)
    if all(b.weight is not None for b in bs):
        a, s = ops.rotate_quant(x2)
    elif _all_int4(bs):
        a, s = _ref_q4(x2, bs[0].group)
    else:
        bs[0].count("routed_swiglu_split")
        pg, pu = _group(x, keys)
        return ops.elementwise(pg.contiguous(), pu.contiguous(), None, 0).reshape(list(x.shape[:-1]) + [width])
    bs[0].count("joint_swiglu")
    return _swiglu_common(x, a, s, keys, width)


def _project_many(x, keys, widths):
    outs = _group(x, keys)
    for o, w in zip(outs, widths):
        if o.shape[-1] != w:
            raise RuntimeError("projection width mismatch")
    return [o.reshape(list(x.shape[:-1]) + [o.shape[-1]]) for o in outs]


def _attention_inputs(x, freqs, keys, widths, norms, heads, kvheads):
    """native_runtime.cpp:601 (group with norms): Q and K per-head normalised
    (and RoPE'd when freqs is given) as [B, H, L, 128], V and the gate as
    plain projections [B, L, n] -- the gate is NOT sigmoided here (the graph
    passes gate_is_sigmoid=False for this route, graph_model.py:39-44)."""
    if len(norms) != 2:
        outs = _project_many(x, keys, widths)
        return outs[0], outs[1], outs[2], outs[3]
    bs = [_proj(k) for k in keys]
    if any(b.loras for b in bs):
        return _split_qkv(x, keys, norms, freqs, heads, kvheads, sigmoid_gate=False)
    if freqs is not None and all(b.weight is not None for b in bs):
        rows, _, K = _rows_len(x)
        a, s = ops.rotate_quant(x.reshape(rows, K).contiguous())
        return _b128_qkv(x, a, s, freqs, keys, heads, kvheads, norms, sigmoid_gate=False)
    if freqs is not None and _all_int4(bs):
        rows, _, K = _rows_len(x)
        a, s = _ref_q4(x.reshape(rows, K).contiguous(), bs[0].group)
        return _ref_qkv(x, a, s, freqs, keys, norms, heads, kvheads, sigmoid_gate=False)
    return _split_qkv(x, keys, norms, freqs, heads, kvheads, sigmoid_gate=False)


def _sdpa(q, k, v, enable_gqa):
    return ops.attention(q, k, v)


def _managed(x, key, kind, width):
    b = _get(key)
    if kind == 0:
        return _linear(x, key)
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


def _fake_packed(x, target_key):
    rows, K = math.prod(x.shape[:-1]), x.shape[-1]
    b = _records.get(int(target_key))
    if b is not None and b.ref is not None:
        return _e((rows, K // 2), x, torch.int8), _e((rows, 1), x, torch.float32)
    return _e((rows, K // 2), x, torch.int8), _e((rows, K // ops.GROUP), x, torch.float16)


def _fake_qkv(x, heads, kvheads):
    B, L = x.shape[0], x.shape[1]
    q = _e((B, L, heads, HEAD_DIM), x).transpose(1, 2)
    k = _e((B, L, kvheads, HEAD_DIM), x).transpose(1, 2)
    return q, k, _e((B, L, kvheads * HEAD_DIM), x), _e((B, L, heads * HEAD_DIM), x)


def _fake_width(x, key):
    b = _records.get(int(key))
    if b is None or (b.weight is None and b.ref is None):
        raise RuntimeError(f"Native K2 binding released: {key}")
    return _width(b)


FAKES = {
    "norm_quant": lambda x, scale, shift, norm_key, target_key, cut: _fake_packed(x, target_key),
    "gated_norm_quant": lambda x, gate, residual, scale, shift, key, norm_key, target_key, cut:
        (torch.empty_like(residual, memory_format=torch.contiguous_format), *_fake_packed(residual, target_key)),
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


__all__ = ["Binding", "RefWeight", "add_binding", "set_loras", "release_bindings", "configure", "configure_joint", "configure_norm_quant",
           "set_route", "finish_tuning", "set_lookahead", "reset_stats", "stats", "kohaku_fa", "SCHEMAS"]
