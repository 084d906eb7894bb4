"""Tensor-parallel pieces on the B200: row-shard norm_quant, the gated add of
a reduced projection, half-used GEMM tiles (the 384-column K/V shards of
tp=4), and the sharded block run in lockstep on one GPU against the
unsharded native block loop.  The multi-GPU NCCL run is covered when the
box has two or more GPUs."""
import os

import numpy as np
import pytest

import oracle as O
from _helpers import TOL_COS, bf16_x, bits, cosine, norm_inputs, packed_act, packed_weight, t_bf16, t_f16, t_f32, \
    t_u8

pytestmark = pytest.mark.gpu


def test_norm_quant_rows_matches_unsharded_slices(cuda):
    import torch
    from k2b import ops

    K, batch, length = 1024, 3, 50
    rows = batch * length
    x = t_bf16(bf16_x(rows, K, 1), cuda)
    w, sc, sh = norm_inputs(K, batch, 2)
    w, sc, sh = t_f32(w, cuda), t_bf16(sc, cuda), t_bf16(sh, cuda)
    q_ref, s_ref = ops.norm_quant(x, w, sc, sh, length=length)
    for base, n in [(0, 37), (37, 37), (45, 60), (148, 2), (100, 50)]:
        q, s = ops.norm_quant_rows(x[base:base + n].contiguous(), w, sc, sh, base_row=base, length=length,
                                   batch=batch)
        torch.cuda.synchronize()
        assert torch.equal(q, q_ref[base:base + n]), base
        assert torch.equal(s, s_ref[base:base + n]), base


def test_gated_add_bitexact(cuda):
    import torch
    from k2b import ops

    rows, n, length, base = 90, 512, 40, 25
    rng = np.random.default_rng(3)
    p = (rng.standard_normal((rows, n)) * 3).astype(np.float32)
    gate = O.bf16_bits(rng.normal(0, 0.1, (4, n)).astype(np.float32))
    resid = O.bf16_bits(rng.standard_normal((rows, n)).astype(np.float32))
    out = ops.gated_add(t_f32(p, cuda), t_bf16(gate, cuda), t_bf16(resid, cuda), base_row=base, length=length)
    torch.cuda.synchronize()
    idx = (base + np.arange(rows)) // length
    ref = O.gated_residual(p, gate[idx], resid, 1)
    assert np.array_equal(bits(out), ref)


@pytest.mark.parametrize("M,N,K", [(300, 384, 512), (257, 128, 1536), (129, 640, 1024)])
def test_gemm_half_tile_bitexact(cuda, M, N, K):
    import torch
    from k2b import ops

    a, sa = packed_act(M, K, 5)
    w, sw = packed_weight(N, K, 6)
    W = ops.prepare_weight(t_u8(w, cuda), t_f16(sw, cuda))
    # a guard row after the output: a store past column n of the last row would land there
    buf = torch.full((M + 1, N), float("nan"), device=cuda)
    ops.gemm_f32(t_u8(a, cuda), t_f16(sa, cuda), W, out=buf[:M])
    torch.cuda.synchronize()
    ref = O.gemm_w4a4(a, sa, w, sw)
    assert np.array_equal(buf[:M].cpu().numpy(), ref)
    assert torch.isnan(buf[M]).all()


def test_qkv_kv_shard_of_three_heads(cuda):
    import torch
    from k2b import ops
    from k2b.model import rope_positions, rope_table

    M, length, K = 260, 130, 512
    hq, hkv = 12, 3
    a, sa = packed_act(M, K, 7)
    ws = {n: packed_weight(h * 128, K, 8 + i) for i, (n, h) in enumerate((("q", hq), ("k", hkv), ("v", hkv)))}
    W = {n: ops.prepare_weight(t_u8(q, cuda), t_f16(s, cuda)) for n, (q, s) in ws.items()}
    nq, nk = np.zeros(128, np.float32), np.full(128, 0.05, np.float32)
    freqs = rope_table(rope_positions(10, 10, 12), (64, 64), 10000.0)
    q, k, v, _ = ops.qkv(t_u8(a, cuda), t_f16(sa, cuda), W["q"], W["k"], W["v"], t_f32(nq, cuda), t_f32(nk, cuda),
                         freqs.to(cuda), length=length)
    torch.cuda.synchronize()
    f = freqs.numpy()
    assert np.array_equal(bits(q), O.qk_norm_rope(O.gemm_w4a4(a, sa, *ws["q"]), hq, nq, 1e-6, f, length))
    assert np.array_equal(bits(k), O.qk_norm_rope(O.gemm_w4a4(a, sa, *ws["k"]), hkv, nk, 1e-6, f, length))
    assert np.array_equal(bits(v), O.bf16_bits(O.gemm_w4a4(a, sa, *ws["v"])))


def test_gemm_f32_scatter_places_rows_in_owner_slots(cuda):
    import torch
    from k2b import ops

    M, N, K, tp, rank = 300, 384, 512, 3, 1
    chunk = -(-M // tp)
    a, sa = packed_act(M, K, 21)
    w, sw = packed_weight(N, K, 22)
    W = ops.prepare_weight(t_u8(w, cuda), t_f16(sw, cuda))
    bufs = [torch.full((tp, chunk, N), float("nan"), device=cuda) for _ in range(tp)]
    ops.gemm_f32_scatter(t_u8(a, cuda), t_f16(sa, cuda), W, [b.data_ptr() for b in bufs], rank, chunk)
    torch.cuda.synchronize()
    ref = O.gemm_w4a4(a, sa, w, sw)
    for dest in range(tp):
        lo, hi = dest * chunk, min(M, (dest + 1) * chunk)
        got = bufs[dest][rank, :hi - lo].cpu().numpy()
        assert np.array_equal(got, ref[lo:hi]), dest
        for other in range(tp):  # only slot `rank` is written
            if other != rank:
                assert torch.isnan(bufs[dest][other]).all()


def test_reduce_gated_add_sums_slots_in_order(cuda):
    import torch
    from k2b import ops

    tp, chunk, n, rows, base, length = 3, 40, 256, 37, 80, 50
    rng = np.random.default_rng(8)
    slots = (rng.standard_normal((tp, chunk, n)) * 3).astype(np.float32)
    gate = O.bf16_bits(rng.normal(0, 0.1, (4, n)).astype(np.float32))
    resid = O.bf16_bits(rng.standard_normal((rows, n)).astype(np.float32))
    sl = t_f32(slots, cuda)
    out = torch.empty((rows, n), dtype=torch.bfloat16, device=cuda)
    ops.reduce_gated_add(sl.data_ptr(), tp, chunk * n, t_bf16(gate, cuda), t_bf16(resid, cuda), base_row=base,
                         length=length, out=out)
    torch.cuda.synchronize()
    p = slots[0, :rows].copy()
    for s_ in range(1, tp):
        p = (p + slots[s_, :rows]).astype(np.float32)  # fp32, slot order
    idx = (base + np.arange(rows)) // length
    assert np.array_equal(bits(out), O.gated_residual(p, gate[idx], resid, 1))


def _tp_models(cuda, cfg, tp, batch, length, seed=3, fused=False):
    from k2b.model import synthetic_blocks
    from k2b.parallel import TPBlocks, TPPlan, local_peer_slots, shard_fn

    ranks = []
    for r in range(tp):
        plan = TPPlan.of(cfg, tp, r)
        bw = synthetic_blocks(cfg, batch, seed=seed, device=cuda, shard=shard_fn(plan))
        ranks.append(TPBlocks(cfg, bw, plan, None, batch, length, device=cuda, fused=fused))
    if fused:
        ranks[0]._slot_bufs = local_peer_slots(ranks)  # keep the buffers alive with the ranks
    return ranks


@pytest.mark.parametrize("tp,batch,length", [(2, 2, 150), (4, 1, 203)])
def test_tp_lockstep_fused_scatter_equals_reduce_scatter(cuda, tp, batch, length):
    """The fused scatter path sums the same fp32 partials in the same rank
    order as the reduce-scatter emulation: bit-identical block outputs."""
    import torch
    from k2b.model import ModelConfig, rope_positions, rope_table
    from k2b.parallel import run_lockstep

    cfg = ModelConfig(hidden=1024, heads=8, kvheads=4, mlp=2048, blocks=2)
    side = 12
    freqs = rope_table(rope_positions(length - (length // side) * side, length // side, side), (64, 64)).to(cuda)
    rng = np.random.default_rng(9)
    xb = O.bf16_bits(rng.standard_normal((batch * length, cfg.hidden)).astype(np.float32))
    outs = []
    for fused in (False, True):
        ranks = _tp_models(cuda, cfg, tp, batch, length, fused=fused)
        xs = []
        for m in ranks:
            sh = m.shard
            xr = torch.zeros((sh.chunk, cfg.hidden), dtype=torch.bfloat16, device=cuda)
            xr[:sh.count] = t_bf16(xb[sh.base:sh.base + sh.count], cuda)
            xs.append(xr)
        run_lockstep(ranks, xs, freqs)
        torch.cuda.synchronize()
        outs.append(torch.cat([x[:m.shard.count] for m, x in zip(ranks, xs)], 0))
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("tp,batch,length", [(2, 2, 150), (4, 1, 203)])
def test_tp_lockstep_matches_native_block_loop(cuda, tp, batch, length):
    import torch
    from k2b.model import Krea2Blocks, ModelConfig, rope_positions, rope_table, synthetic_blocks
    from k2b.parallel import run_lockstep

    cfg = ModelConfig(hidden=1024, heads=8, kvheads=4, mlp=2048, blocks=2)
    full = Krea2Blocks(cfg, synthetic_blocks(cfg, batch, seed=3, device=cuda), batch, length, device=cuda)
    side = 12
    freqs = rope_table(rope_positions(length - (length // side) * side, length // side, side), (64, 64)).to(cuda)
    rng = np.random.default_rng(4)
    xb = O.bf16_bits(rng.standard_normal((batch * length, cfg.hidden)).astype(np.float32))
    ref = full.forward_(t_bf16(xb, cuda), freqs)
    ranks = _tp_models(cuda, cfg, tp, batch, length)
    xs = []
    for m in ranks:
        sh = m.shard
        xr = torch.zeros((sh.chunk, cfg.hidden), dtype=torch.bfloat16, device=cuda)
        xr[:sh.count] = t_bf16(xb[sh.base:sh.base + sh.count], cuda)
        xs.append(xr)
    run_lockstep(ranks, xs, freqs)
    torch.cuda.synchronize()
    got = torch.cat([x[:m.shard.count] for m, x in zip(ranks, xs)], 0)
    g, r = bits(got), bits(ref)
    gf, rf = O.bf16_float(g).astype(np.float64), O.bf16_float(r).astype(np.float64)
    assert cosine(gf, rf) >= TOL_COS
    assert np.abs(gf - rf).max() <= 2e-2 * np.abs(rf).max()
    assert (g == r).mean() >= 0.98  # fp32 reassociation of projection sums only


def _nccl_rank(rank, world, port, path, fused=False):
    import datetime

    import torch
    import torch.distributed as dist
    from k2b.model import ModelConfig, rope_positions, rope_table, synthetic_blocks
    from k2b.parallel import PeerWatch, TPBlocks, TPPlan, shard_fn, topology

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        cfg = ModelConfig(hidden=1024, heads=8, kvheads=4, mlp=2048, blocks=2)
        batch, length = 2, 150
        topo = topology(world, rank, world)
        plan = TPPlan.of(cfg, world, rank)
        bw = synthetic_blocks(cfg, batch, seed=3, device=dev, shard=shard_fn(plan))
        watch = PeerWatch(dist.distributed_c10d._get_default_store(), rank, range(world), timeout_s=30)
        m = TPBlocks(cfg, bw, plan, topo.tp_group, batch, length, device=dev, fused=fused, watch=watch)
        freqs = rope_table(rope_positions(6, 12, 12), (64, 64)).to(dev)
        rng = np.random.default_rng(4)
        xb = O.bf16_bits(rng.standard_normal((batch * length, cfg.hidden)).astype(np.float32))
        sh = m.shard
        x = torch.zeros((sh.chunk, cfg.hidden), dtype=torch.bfloat16, device=dev)
        x[:sh.count] = t_bf16(xb[sh.base:sh.base + sh.count], dev)
        m.forward_(x, freqs)
        torch.cuda.synchronize()
        np.save(f"{path}.{rank}.npy", bits(x[:sh.count]))
        m.close()
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fused", [False, True])
def test_tp2_nccl_matches_native_block_loop(cuda, tmp_path, fused):
    import socket

    import torch
    import torch.multiprocessing as mp
    from k2b.model import Krea2Blocks, ModelConfig, rope_positions, rope_table, synthetic_blocks

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    path = str(tmp_path / "tp")
    mp.start_processes(_nccl_rank, args=(2, port, path, fused), nprocs=2, start_method="spawn")
    got = np.concatenate([np.load(f"{path}.{r}.npy") for r in range(2)], 0)
    cfg = ModelConfig(hidden=1024, heads=8, kvheads=4, mlp=2048, blocks=2)
    batch, length = 2, 150
    full = Krea2Blocks(cfg, synthetic_blocks(cfg, batch, seed=3, device=cuda), batch, length, device=cuda)
    freqs = rope_table(rope_positions(6, 12, 12), (64, 64)).to(cuda)
    rng = np.random.default_rng(4)
    xb = O.bf16_bits(rng.standard_normal((batch * length, cfg.hidden)).astype(np.float32))
    ref = bits(full.forward_(t_bf16(xb, cuda), freqs))
    gf, rf = O.bf16_float(got).astype(np.float64), O.bf16_float(ref).astype(np.float64)
    assert cosine(gf, rf) >= TOL_COS
    assert np.abs(gf - rf).max() <= 2e-2 * np.abs(rf).max()
    assert (got == ref).mean() >= 0.98
