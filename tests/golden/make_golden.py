"""Generates tests/golden/reference_triton.npz from the reference's own kernels.

Runs (in this container only; the reference tree is not needed afterwards):
  * forward_kernels.py::_norm_mod      RMSNorm + adaLN modulation (:13-45)
  * forward_kernels.py::_qk_post       per-head QK RMSNorm + RoPE (:64-98)
  * forward_kernels.py::_activate_mul  SiLU(a) * b (:48-61)
  * KohakuKernelRouter/attention.py::fwd_kernel  GQA flash attention, with and
    without the gated store (:63-110)
under the Triton CPU interpreter (TRITON_INTERPRET=1) on small seeded inputs.
The interpreter lacks the CUDA libdevice externs these kernels call, so they
are bound to their IEEE meaning for this run: div_rn -> correctly rounded
division, exp -> tl.exp.  The interpreter converts fp32 -> bf16 by truncation
(the GPU rounds to nearest even); tests/test_oracle.py switches the oracle to
truncation when comparing.  Nothing of the reference is copied into the
fixtures except its outputs.

    python tests/golden/make_golden.py /path/to/ComfyUI-K2-Precompile
"""
from __future__ import annotations

import importlib.util
import math
import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402
import triton.language as tl  # noqa: E402
from triton.language.extra.cuda import libdevice  # noqa: E402

libdevice.div_rn = lambda a, b, **kw: a / b
libdevice.exp = lambda a, **kw: tl.exp(a)

if len(sys.argv) != 2:
    raise SystemExit("usage: python tests/golden/make_golden.py /path/to/ComfyUI-K2-Precompile")
REF = sys.argv[1]
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_triton.npz")


def load(name, rel):
    spec = importlib.util.spec_from_file_location(name, os.path.join(REF, rel))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main():
    fk = load("ref_forward_kernels", "forward_kernels.py")
    g = torch.Generator().manual_seed(20261201)
    out = {}

    # ---- _norm_mod: 2 latents x 6 rows, D = 1024, modulation per latent
    B, L, D = 2, 6, 1024
    x = (torch.randn(B * L, D, generator=g) * torch.where(torch.rand(D, generator=g) < 0.02, 20.0, 1.0))
    x = x.to(torch.bfloat16)
    w = (torch.rand(D, generator=g) * 0.2 + 0.9).to(torch.bfloat16).float() - 1.0
    scale = (torch.randn(B, D, generator=g) * 0.1).to(torch.bfloat16)
    shift = (torch.randn(B, D, generator=g) * 0.1).to(torch.bfloat16)
    y = torch.empty_like(x)
    fk._norm_mod[(B * L,)](x, w, scale, shift, y, D, L, -1, B, True, 1e-6, 1024, num_warps=4)
    out.update(nm_x=u16(x), nm_w=w.numpy(), nm_scale=u16(scale), nm_shift=u16(shift), nm_y=u16(y),
               nm_L=np.int32(L), nm_eps=np.float32(1e-6))

    # ---- _qk_post: B=1, L=5 tokens, 2 q heads + 1 k head, D = 128
    L2, QH, KH, HD = 5, 2, 1, 128
    q = torch.randn(1, L2, QH * HD, generator=g).to(torch.bfloat16)
    k = torch.randn(1, L2, KH * HD, generator=g).to(torch.bfloat16)
    qw = (torch.rand(HD, generator=g) * 0.2 + 0.9).to(torch.bfloat16).float() - 1.0
    kw = (torch.rand(HD, generator=g) * 0.2 + 0.9).to(torch.bfloat16).float() - 1.0
    pos = torch.arange(L2, dtype=torch.float64)
    omega = 1.0 / torch.pow(10000.0, torch.linspace(0.0, (HD - 2) / HD, HD // 2, dtype=torch.float64))
    ang = pos[:, None] * omega[None, :]
    freqs = torch.stack([ang.cos(), -ang.sin(), ang.sin(), ang.cos()], -1).reshape(1, 1, L2, HD // 2, 2, 2).float()
    qo, ko = torch.empty_like(q), torch.empty_like(k)
    fk._qk_post[(L2 * (QH + KH),)](q, k, qw, kw, freqs, qo, ko, L2, QH, KH, HD, 1, 1e-6, 1e-6, False, False, 128,
                                   num_warps=4)
    out.update(qk_q=u16(q), qk_k=u16(k), qk_qw=qw.numpy(), qk_kw=kw.numpy(), qk_freqs=freqs.numpy(),
               qk_qo=u16(qo), qk_ko=u16(ko))

    # ---- _activate_mul (SiLU): 512 elements
    a = (torch.randn(512, generator=g) * 3).to(torch.bfloat16)
    b = torch.randn(512, generator=g).to(torch.bfloat16)
    yam = torch.empty_like(a)
    fk._activate_mul[(2,)](a, b, yam, 512, 0, 256)
    out.update(am_a=u16(a), am_b=u16(b), am_y=u16(yam))

    # ---- Kohaku fwd_kernel: B=1, Hq=4, Hkv=2, L=40, D=128 (+ gated store).
    # The interpreter's tl.dot mishandles bf16 operands, so the kernel runs on
    # fp32 tensors holding bf16-valued data (P is then not rounded to bf16
    # before the PV product; the comparison allows for that).
    att = load("ref_kohaku_attention", "KohakuKernelRouter/attention.py")
    Bq, Hq, Hk, La, Da = 1, 4, 2, 40, 128
    qa = torch.randn(Bq, Hq, La, Da, generator=g)
    qa = (qa / qa.pow(2).mean(-1, keepdim=True).sqrt()).to(torch.bfloat16)
    ka = torch.randn(Bq, Hk, La, Da, generator=g)
    ka = (ka / ka.pow(2).mean(-1, keepdim=True).sqrt()).to(torch.bfloat16)
    va = torch.randn(Bq, Hk, La, Da, generator=g).to(torch.bfloat16)
    gate = torch.sigmoid(torch.randn(Bq, La, Hq * Da, generator=g)).to(torch.bfloat16)
    qf, kf, vf, gf = qa.float(), ka.float(), va.float(), gate.float()
    for tag, gt, kind in (("plain", None, 0), ("gated", gf, 2)):
        o = torch.empty(Bq, La, Hq * Da, dtype=torch.float32)
        BM, BN = 16, 16
        att.fwd_kernel[(math.ceil(La / BM), Hq, Bq)](
            qf, kf, vf, gt if gt is not None else qf, qf, o, att.LOG2E * Da ** -0.5, La, La,
            *qf.stride(), *kf.stride(), *vf.stride(), 0, 0, 0, 0,
            HQ=Hq, HK=Hk, D=Da, BM=BM, BN=BN, MASK_KIND=0, GATE_KIND=kind, num_warps=4, num_stages=1)
        out[f"fa_{tag}"] = o.numpy()
    out.update(fa_q=u16(qa), fa_k=u16(ka), fa_v=u16(va), fa_gate=u16(gate))
    np.savez_compressed(OUT, **out)
    print("wrote", OUT, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
