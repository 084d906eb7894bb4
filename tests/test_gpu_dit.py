"""The whole DiT forward (k2b.dit): patch embedding, timestep MLP, W4A4
text-fusion blocks at GQA group 1, the W4A4 block stack, the final
RMSNorm + modulation and projection, against the CPU oracle's composition of
the same steps (the plain linears in fp32 on the CPU, rounded to bf16)."""
import numpy as np
import pytest

import oracle as O
from _helpers import TOL_ABS, TOL_COS, bits, cosine, np_block, oracle_block

pytestmark = pytest.mark.gpu

ONE = 0x3F80  # bf16 1.0


def _small():
    from k2b.dit import DiTConfig
    from k2b.model import ModelConfig

    core = ModelConfig(hidden=512, heads=4, kvheads=2, mlp=1024, blocks=2)
    return DiTConfig(core=core, channels=4, patch=2, tdim=64, txtdim=512, txt_heads=4, txt_kvheads=4, txt_mlp=1024,
                     txt_layers=2)


def _lin_cpu(x, wb):
    """bf16(x @ W^T + b) in fp32 on the CPU."""
    import torch

    w, b = wb
    return torch.nn.functional.linear(x.float().cpu(), w.float().cpu(), b.float().cpu()).to(torch.bfloat16)


def _np_text(tb):
    d = {k: getattr(tb, k).cpu().numpy() for k in ("norm1", "norm2", "qnorm", "knorm")}
    for n, (q, s) in tb.packed.items():
        d[n] = (q.cpu().numpy(), bits(s))
    return d


def _oracle_text_block(x, tb, B, Lt, H, Hk, eps=1e-6):
    T = x.shape[1]
    zero = np.zeros((B, T), np.uint16)
    ones = np.full((B, T), ONE, np.uint16)
    ident = np.zeros((Lt, 64, 2, 2), np.float32)
    ident[..., 0, 0] = 1.0
    ident[..., 1, 1] = 1.0
    xq, xs = O.norm_quant(x, tb["norm1"], zero, zero, length=Lt, eps=eps)
    q = O.qk_norm_rope(O.gemm_w4a4(xq, xs, *tb["wq"]), H, tb["qnorm"], eps, ident, Lt)
    k = O.qk_norm_rope(O.gemm_w4a4(xq, xs, *tb["wk"]), Hk, tb["knorm"], eps, ident, Lt)
    v = O.bf16_bits(O.gemm_w4a4(xq, xs, *tb["wv"]))
    g = O.sigmoid_gate(O.gemm_w4a4(xq, xs, *tb["wgate"]))
    t4 = lambda a, h: a.reshape(B, Lt, h, 128).transpose(0, 2, 1, 3)
    o = O.attention(t4(q, H), t4(k, Hk), t4(v, Hk), gate=g.reshape(B, Lt, H * 128)).reshape(B * Lt, -1)
    oq, os_ = O.rotate_quant(o)
    x1 = O.gated_residual(O.gemm_w4a4(oq, os_, *tb["wo"]), ones, x, Lt)
    hq_in, hs_in = O.norm_quant(x1, tb["norm2"], zero, zero, length=Lt, eps=eps)
    hq, hs = O.swiglu_quant(O.gemm_w4a4(hq_in, hs_in, *tb["wg"]), O.gemm_w4a4(hq_in, hs_in, *tb["wu"]))
    return O.gated_residual(O.gemm_w4a4(hq, hs, *tb["wd"]), ones, x1, Lt)


def _close(got, ref, what):
    g, r = O.bf16_float(got).astype(np.float64), O.bf16_float(ref).astype(np.float64)
    cos = cosine(g, r)
    err = float(np.abs(g - r).max())
    scale = float(np.abs(r).max())
    assert cos >= TOL_COS, (what, cos)
    assert err <= max(TOL_ABS, TOL_ABS * scale), (what, err, scale)
    return cos, err


def test_text_fusion_block_matches_oracle(cuda):
    import torch
    from k2b import dit

    cfg = _small()
    w = dit.synthetic_dit(cfg, batch=2, seed=1, device=cuda, keep_packed=True)
    B, Lt = 2, 37
    rng = np.random.default_rng(3)
    xb = O.bf16_bits(rng.standard_normal((B * Lt, cfg.txtdim)).astype(np.float32))
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).to(cuda)
    zero = torch.zeros((B, cfg.txtdim), dtype=torch.bfloat16, device=cuda)
    ones = torch.ones((B, cfg.txtdim), dtype=torch.bfloat16, device=cuda)
    out = dit.text_block(cfg, w.txt[0], x, B, Lt, dit.identity_rope(Lt, cuda), zero, ones)
    ref = _oracle_text_block(xb, _np_text(w.txt[0]), B, Lt, cfg.txt_heads, cfg.txt_kvheads)
    _close(bits(out), ref, "text-fusion block")


def test_dit_forward_stagewise_and_end_to_end(cuda):
    """Every stage of the forward against the oracle's version of that stage,
    fed the GPU's output of the stage before it (the block-stack check of
    test_gpu_block.py: cosine and max abs within 2e-2 of the stream's max;
    the text-fusion blocks as above; the plain linears and the final norm
    within the north_star tolerance).  End to end, the same composition run
    entirely on the oracle agrees to cosine >= 0.999: one-ulp differences of
    the library linears move a few INT4 codes, so only the cosine is held
    end to end."""
    import torch
    from k2b import dit
    from k2b.model import rope_table

    cfg = _small()
    B, Lt = 2, 20
    w = dit.synthetic_dit(cfg, batch=B, seed=2, device=cuda, keep_packed=True)
    g = torch.Generator().manual_seed(5)
    x = torch.randn((B, cfg.channels, 16, 24), generator=g).to(torch.bfloat16)
    ctx = torch.randn((B, Lt, cfg.txtdim), generator=g).to(torch.bfloat16)
    ts = torch.tensor([0.3, 0.8], dtype=torch.float32)
    model = dit.Krea2DiT(cfg, w)
    tr = {}
    out = model.forward(x.to(cuda), ts.to(cuda), ctx.to(cuda), trace=tr)
    torch.cuda.synchronize()
    assert out.shape == x.shape and out.dtype == torch.bfloat16
    tb_ = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)
    hid = cfg.core.hidden

    def stages(gpu):
        """The oracle's forward; each stage reads ``gpu(name, own)``: the GPU's
        copy of the previous stage (stagewise) or the oracle's own (end to end)."""
        res = {}
        img, h, wd = dit.patchify(x, cfg.patch)
        res["img"] = _lin_cpu(img, w.first)
        t = dit.timestep_embedding(ts, cfg.tdim).unsqueeze(1).to(torch.bfloat16)
        t1 = torch.nn.functional.gelu(_lin_cpu(t, w.tmlp1).float(), approximate="tanh").to(torch.bfloat16)
        res["t"] = _lin_cpu(t1, w.tmlp2)
        res["tvec"] = _lin_cpu(gpu("t", res["t"]), w.tproj)
        c = bits(ctx.reshape(B * Lt, -1))
        for i, tb in enumerate(w.txt):
            c = _oracle_text_block(c, _np_text(tb), B, Lt, cfg.txt_heads, cfg.txt_kvheads)
            res[f"txt{i}"] = tb_(c)
            c = bits(gpu(f"txt{i}", res[f"txt{i}"]))
        c = _lin_cpu(tb_(c).view(B, Lt, -1), w.txtmlp)
        res["combined"] = torch.cat([c, gpu("img", res["img"])], 1)
        L = res["combined"].shape[1]
        freqs = rope_table(dit.positions(Lt, h, wd), cfg.axes, cfg.core.theta).numpy()
        tvec = gpu("tvec", res["tvec"]).float().cpu().to(torch.bfloat16)
        mods = (tvec.view(1, B, 6 * hid) + w.mod_lin.cpu().view(-1, 1, 6 * hid)).view(-1, B, 6, hid)
        stream = bits(gpu("combined", res["combined"]).reshape(-1, hid))
        for i, b in enumerate(w.blocks):
            nb = np_block(b)
            nb["mod"] = bits(mods[i].transpose(0, 1).contiguous())
            stream = oracle_block(stream, nb, freqs, B, L, cfg.core.heads, cfg.core.kvheads)
        res["blocks"] = tb_(stream).view(B * L, hid)
        t_ = gpu("t", res["t"]).cpu()
        scale, shift = (t_ + w.last_lin.cpu().unsqueeze(0)).chunk(2, dim=1)
        y = O.norm_mod(bits(gpu("blocks", res["blocks"])), w.last_norm.cpu().numpy(), bits(scale.reshape(B, hid)),
                       bits(shift.reshape(B, hid)), length=L)
        res["normed"] = tb_(y).view(B * L, hid)
        yv = gpu("normed", res["normed"]).cpu().view(B, L, hid)
        res["out"] = dit.unpatchify(_lin_cpu(yv[:, Lt:], w.last), h, wd, cfg.patch, cfg.channels)
        return res

    tr["out"] = out
    step = stages(lambda name, own: tr[name].cpu())
    for name in ("img", "t", "tvec", "txt0", "txt1", "combined", "normed", "out"):
        _close(bits(tr[name]), bits(step[name]), name)
    # the block stack: the block-chain criterion
    gb, rb = O.bf16_float(bits(tr["blocks"])), O.bf16_float(bits(step["blocks"]))
    assert cosine(gb, rb) >= TOL_COS
    assert float(np.abs(gb - rb).max()) <= TOL_ABS * float(np.abs(rb).max())
    assert np.array_equal(bits(tr["normed"]), bits(step["normed"]))  # k2b_norm_mod of the GPU stream: exact
    own = stages(lambda name, o: o)
    assert cosine(O.bf16_float(bits(out)), O.bf16_float(bits(own["out"]))) >= TOL_COS
