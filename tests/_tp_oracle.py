"""The tensor-parallel block choreography of k2b.parallel restated on the CPU
oracle, for checking the sharding plan (heads, MLP columns, K-slices, row
shards with their modulation rows) and the collective helpers on CPU.

``rank_steps`` is a generator per rank: it yields ("gather", q, s) with its
own rows' INT4 codes and receives the group's rows, and ("reduce_scatter", p)
with its fp32 partial [rows, n] and receives its rows of the sum."""
from __future__ import annotations

import numpy as np
import torch

import oracle as O
from _helpers import bf16_x, norm_inputs, packed_weight

from k2b.parallel import TPPlan, shard_packed


def small_model(hidden=512, heads=8, kvheads=4, mlp=1024, batch=2, length=37, blocks=1, seed=11):
    rng = np.random.default_rng(seed)
    shapes = {"wq": (heads * 128, hidden), "wk": (kvheads * 128, hidden), "wv": (kvheads * 128, hidden),
              "wo": (hidden, heads * 128), "wg": (mlp, hidden), "wu": (mlp, hidden), "wd": (hidden, mlp)}
    out = []
    for bi in range(blocks):
        blk = {n: packed_weight(a, b, seed + 17 * bi + i) for i, (n, (a, b)) in enumerate(shapes.items())}
        pre, _, _ = norm_inputs(hidden, 1, seed + 101 + bi)
        post, _, _ = norm_inputs(hidden, 1, seed + 202 + bi)
        blk["prenorm"], blk["postnorm"] = pre, post
        blk["qnorm"] = (O.bf16_round(rng.uniform(0.9, 1.1, 128).astype(np.float32)) - 1).astype(np.float32)
        blk["knorm"] = (O.bf16_round(rng.uniform(0.9, 1.1, 128).astype(np.float32)) - 1).astype(np.float32)
        blk["mod"] = O.bf16_bits(rng.normal(0, 0.1, (6, batch, hidden)).astype(np.float32))
        out.append(blk)
    side = 6
    text = length - (length // side) * side
    t = np.arange(text, dtype=np.float32)
    y = np.repeat(np.arange(length // side, dtype=np.float32), side) + text
    xx = np.tile(np.arange(side, dtype=np.float32), length // side) + text
    pos = np.concatenate([np.stack([t, t], 1), np.stack([y, xx], 1)], 0)
    freqs = O.rope_table(pos, (64, 64), 10000.0)
    x = bf16_x(batch * length, hidden, seed + 7, outliers=False)
    return out, freqs, x


def shard_block(blk, plan: TPPlan):
    """Numpy block dict -> this rank's shard (weights sliced by
    k2b.parallel.shard_packed on CPU tensors)."""
    d = dict(blk)
    for name in ("wq", "wk", "wv", "wo", "wg", "wu", "wd"):
        q, s = blk[name]
        tq, ts = shard_packed(name, torch.from_numpy(q), torch.from_numpy(s.view(np.int16)), plan)
        d[name] = (tq.numpy(), ts.numpy().view(np.uint16))
    return d


def rank_steps(plan: TPPlan, shards, freqs, x_own, batch, length, eps=1e-6, qk_eps=1e-6):
    """One rank's block loop on the oracle; yields at each collective."""
    rows = batch * length
    sh = plan.rows(rows)
    n = sh.count
    idx = (sh.base + np.arange(n)) // length  # modulation row of each own row
    hq_l, kv_l = plan.heads // plan.tp, plan.kvheads // plan.tp
    x = x_own
    for blk in shards:
        mod = blk["mod"]
        xq, xs = O.norm_quant(x, blk["prenorm"], mod[0][idx], mod[1][idx], length=1, eps=eps)
        aq, as_ = yield ("gather", xq, xs)
        pq = O.gemm_w4a4(aq, as_, *blk["wq"])
        pk = O.gemm_w4a4(aq, as_, *blk["wk"])
        pv = O.gemm_w4a4(aq, as_, *blk["wv"])
        q = O.qk_norm_rope(pq, hq_l, blk["qnorm"], qk_eps, freqs, length)
        k = O.qk_norm_rope(pk, kv_l, blk["knorm"], qk_eps, freqs, length)
        v = O.bf16_bits(pv)
        q4 = q.reshape(batch, length, hq_l, 128).transpose(0, 2, 1, 3)
        k4 = k.reshape(batch, length, kv_l, 128).transpose(0, 2, 1, 3)
        v4 = v.reshape(batch, length, kv_l, 128).transpose(0, 2, 1, 3)
        o = O.attention(q4, k4, v4).reshape(rows, hq_l * 128)
        oq, os_ = O.rotate_quant(o)
        red = yield ("reduce_scatter", O.gemm_w4a4(oq, os_, *blk["wo"]))
        x1 = O.gated_residual(red, mod[2][idx], x, 1)
        hq_in, hs_in = O.norm_quant(x1, blk["postnorm"], mod[3][idx], mod[4][idx], length=1, eps=eps)
        aq, as_ = yield ("gather", hq_in, hs_in)
        hq, hs = O.swiglu_quant(O.gemm_w4a4(aq, as_, *blk["wg"]), O.gemm_w4a4(aq, as_, *blk["wu"]))
        red = yield ("reduce_scatter", O.gemm_w4a4(hq, hs, *blk["wd"]))
        x = O.gated_residual(red, mod[5][idx], x1, 1)
    return x


def run_lockstep(plans, gens, rows):
    """Drives the rank generators of one group in one process."""
    tp = len(plans)
    chunk = plans[0].rows(rows).chunk
    results = [None] * tp
    reqs = [next(g) for g in gens]
    while True:
        kind = reqs[0][0]
        assert all(r[0] == kind for r in reqs)
        if kind == "gather":
            q = np.concatenate([r[1] for r in reqs], 0)
            s = np.concatenate([r[2] for r in reqs], 0)
            resp = [(q, s)] * tp
        else:
            pad = np.zeros((chunk * tp,) + reqs[0][1].shape[1:], np.float32)
            total = pad.copy()
            for r in reqs:  # rank order, fp32
                part = pad.copy()
                part[:rows] = r[1]
                total += part
            resp = [total[p.rows(rows).base:p.rows(rows).base + p.rows(rows).count] for p in plans]
        nxt = []
        for i, g in enumerate(gens):
            try:
                nxt.append(g.send(resp[i]))
            except StopIteration as stop:
                results[i] = stop.value
                nxt.append(None)
        if all(r is None for r in nxt):
            return results
        reqs = nxt
