"""Multi-GPU execution of the Krea2 W4A4 block stack: batch sharding across
data-parallel groups, KV-head tensor parallelism inside a group.

The reference runs one latent batch on one GPU (graph_model.py:259-295 walks
the blocks of one ``dit`` call); the multi-GPU layouts here are the B200
build's own.  One process per GPU, ``torch.distributed`` over NCCL.

Data parallel (``dp``): latents (prompts x CFG branches) are independent, so
each data-parallel group takes a contiguous range of them and no collective
touches the data path.

KV-head tensor parallel over ``tp`` ranks (``tp`` divides the 12 KV heads;
2 and 4 are the intended degrees).  Rank r owns KV heads
[r*Hkv/tp, (r+1)*Hkv/tp), the Q heads that share them (GQA groups of
Hq/Hkv consecutive Q heads), and MLP columns [r*F/tp, (r+1)*F/tp).  The
residual stream is sharded by rows: rank r holds rows [r*c, (r+1)*c) of the
group's batch*length rows, c = ceil(rows/tp).  One block:

  1. norm_quant of own rows into this rank's slot     -> all-gather (INT4)
  2. Q/K/V projection of own heads (QK norm + RoPE fused), attention of own
     heads with an INT4 output
  3. out-projection over own K-slice, fp32 partial     -> reduce-scatter (sum)
  4. gated residual of own rows; norm_quant of them     -> all-gather (INT4)
  5. gate/up + SwiGLU + requant over own F/tp columns
  6. down-projection over own K-slice, fp32 partial    -> reduce-scatter (sum)
  7. gated residual of own rows.

With ``fused=True`` the reduce-scatter half is done by the projection
itself: its epilogue stores each fp32 partial tile straight into the owner
rank's receive buffer over NVLink (CUDA-IPC mapped peer memory,
k2b_gemm_f32_scatter), so the transfer overlaps the GEMM tile by tile; a
stream-ordered barrier (a one-element NCCL all-reduce) follows, and the owner
sums its slots inside the gated-residual kernel (k2b_reduce_gated_add).

Steps 3-4 and 6-7 are the all-reduce after the out- and down-projections,
split into its reduce-scatter and all-gather halves around the row-local work
between them, so the gated residual and norm_quant run once per row rather
than once per rank, and the gather half moves INT4 codes + fp16 scales
(4.125 bits per element) instead of bf16.  Every INT4 stage works on 128-column groups that no rank
boundary splits (heads are 128 columns; F/tp is a multiple of 128), so each
rank's codes are the column slice of the unsharded codes for the same inputs;
the one numerical difference from one GPU is the fp32 reassociation of the
projection sums (per-rank partials summed by the reduce-scatter) before the
bf16 rounding of the projection.

Failure detection is on the host: ``PeerWatch`` is a per-step heartbeat in
the process group's store, checked before a step launches anything, so a rank
that raised, exited or stalled between steps is reported on every other rank
(``PeerLost``) while none of their kernels or collectives is in flight; a
collective that a peer never joins ends with the process group's own timeout.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Iterator, List, Optional, Sequence, Tuple

import torch

from . import ops
from .model import BlockWeights, ModelConfig

GROUP = 128


# ------------------------------------------------------------------- plans

@dataclass(frozen=True)
class RowShard:
    """This rank's rows of a tensor-parallel group's row space."""

    chunk: int   # rows per rank (the last rank's may be partly padding)
    base: int    # first row owned by this rank
    count: int   # rows owned (chunk, or fewer on the last rank)
    tp: int      # ranks in the group

    @property
    def padded(self) -> int:
        return self.chunk * self.tp


@dataclass(frozen=True)
class TPPlan:
    """Which heads, MLP columns and rows rank ``rank`` of ``tp`` owns."""

    tp: int
    rank: int
    hidden: int = 6144
    heads: int = 48
    kvheads: int = 12
    mlp: int = 16384

    def __post_init__(self):
        if self.tp < 1 or not 0 <= self.rank < self.tp:
            raise ValueError(f"tensor-parallel rank {self.rank} of {self.tp}")
        if self.kvheads % self.tp or self.heads % self.kvheads:
            raise ValueError(f"{self.kvheads} KV heads do not split over {self.tp} ranks")
        if self.mlp % (GROUP * self.tp):
            raise ValueError(f"MLP width {self.mlp} does not split into 128-column groups over {self.tp} ranks")

    @classmethod
    def of(cls, cfg: ModelConfig, tp: int, rank: int) -> "TPPlan":
        return cls(tp, rank, cfg.hidden, cfg.heads, cfg.kvheads, cfg.mlp)

    @property
    def q_heads(self) -> Tuple[int, int]:
        n = self.heads // self.tp
        return self.rank * n, (self.rank + 1) * n

    @property
    def kv_heads(self) -> Tuple[int, int]:
        n = self.kvheads // self.tp
        return self.rank * n, (self.rank + 1) * n

    @property
    def q_cols(self) -> Tuple[int, int]:
        a, b = self.q_heads
        return a * 128, b * 128

    @property
    def kv_cols(self) -> Tuple[int, int]:
        a, b = self.kv_heads
        return a * 128, b * 128

    @property
    def mlp_cols(self) -> Tuple[int, int]:
        n = self.mlp // self.tp
        return self.rank * n, (self.rank + 1) * n

    def rows(self, total: int) -> RowShard:
        chunk = -(-total // self.tp)
        base = min(total, self.rank * chunk)
        return RowShard(chunk, base, max(0, min(chunk, total - base)), self.tp)


# Which axis of each weight [n, k] a rank slices: output rows (n) for the
# column-parallel projections, input columns (k) for the row-parallel ones.
_ROW_SHARDED = {"wq": "q_cols", "wk": "kv_cols", "wv": "kv_cols", "wg": "mlp_cols", "wu": "mlp_cols"}
_K_SHARDED = {"wo": "q_cols", "wd": "mlp_cols"}


def shard_packed(name: str, packed: torch.Tensor, scales: torch.Tensor, plan: TPPlan
                 ) -> Tuple[torch.Tensor, torch.Tensor]:
    """This rank's slice of a packed INT4 weight (u8 [n, k/2]) and its fp16
    group scales ([n, k/128]).  K-slices fall on 128-column group boundaries,
    so the slice of the packed codes and of the scales is exact."""
    if name in _ROW_SHARDED:
        a, b = getattr(plan, _ROW_SHARDED[name])
        return packed[a:b].contiguous(), scales[a:b].contiguous()
    if name in _K_SHARDED:
        a, b = getattr(plan, _K_SHARDED[name])
        if a % GROUP or b % GROUP:
            raise ValueError("K-slices must fall on 128-column groups")
        return packed[:, a // 2:b // 2].contiguous(), scales[:, a // GROUP:b // GROUP].contiguous()
    raise KeyError(name)


def shard_fn(plan: TPPlan):
    """``shard`` callback for model.synthetic_blocks."""
    return lambda name, q, s: shard_packed(name, q, s, plan)


# --------------------------------------------------------------- topology

@dataclass
class Topology:
    world: int
    rank: int
    tp: int
    dp: int
    dp_index: int
    tp_rank: int
    tp_group: Optional[object]  # torch.distributed ProcessGroup, None when tp == 1

    def latent_range(self, latents: int) -> Tuple[int, int]:
        """The contiguous latents this rank's data-parallel group runs."""
        if latents % self.dp:
            raise ValueError(f"{latents} latents do not split over {self.dp} data-parallel groups")
        n = latents // self.dp
        return self.dp_index * n, (self.dp_index + 1) * n


def topology(world: int, rank: int, tp: int, make_groups: bool = True) -> Topology:
    """dp x tp layout: tensor-parallel groups are consecutive ranks
    [d*tp, (d+1)*tp) (every peer is one NVSwitch hop away, so placement does
    not matter).  Every rank creates every group, in the same order."""
    if tp < 1 or world % tp:
        raise ValueError(f"tp={tp} does not divide world={world}")
    dp = world // tp
    group = None
    if tp > 1 and make_groups:
        import torch.distributed as dist

        for d in range(dp):
            g = dist.new_group(list(range(d * tp, (d + 1) * tp)))
            if d == rank // tp:
                group = g
    return Topology(world, rank, tp, dp, rank // tp, rank % tp, group)


# ------------------------------------------------------------ collectives

def gather_rows(bufs: Sequence[torch.Tensor], chunk: int, rank: int, group) -> None:
    """In-place all-gather along rows: each buffer [tp*chunk, ...] holds this
    rank's rows at [rank*chunk, (rank+1)*chunk) and receives the others'."""
    import torch.distributed as dist

    for full in bufs:
        dist.all_gather_into_tensor(full, full[rank * chunk:(rank + 1) * chunk], group=group)


def reduce_scatter_rows(out: torch.Tensor, full: torch.Tensor, group) -> None:
    """out [chunk, n] = sum over ranks of their full[rank*chunk:(rank+1)*chunk]."""
    import torch.distributed as dist

    dist.reduce_scatter_tensor(out, full, op=dist.ReduceOp.SUM, group=group)


# ------------------------------------------------------- tensor-parallel run

PHASES = ["norm_quant_pre", "gather_act", "qkv_qknorm_rope", "attention_quant", "out_proj_partial",
          "reduce_scatter_out", "gated_add_norm_quant_post", "gather_mlp_in", "gate_up_swiglu_quant",
          "down_proj_partial", "reduce_scatter_down", "gated_add"]


class PeerSlots:
    """Receive buffers of one tensor-parallel group for the fused scatter:
    ``ptrs[j]`` is rank j's buffer (fp32 [tp, chunk, n]) as this process sees
    it, ``ptrs[rank]`` its own."""

    def __init__(self, ptrs: Sequence[int], rank: int, owned=None, mapped=()):
        self.ptrs, self.rank = [int(x) for x in ptrs], rank
        self._owned, self._mapped = owned, list(mapped)

    @classmethod
    def ipc(cls, nbytes: int, rank: int, tp: int, group) -> "PeerSlots":
        """Collective over ``group``: every rank allocates its buffer with
        k2b_ipc_alloc and maps the others' through CUDA IPC."""
        import ctypes

        import torch.distributed as dist

        from ._native import check, lib

        L = lib()
        own = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * 64)()
        check(L.k2b_ipc_alloc(nbytes, ctypes.byref(own), handle), "k2b_ipc_alloc")
        handles = [None] * tp
        dist.all_gather_object(handles, bytes(handle), group=group)
        ptrs, mapped = [], []
        for j, h in enumerate(handles):
            if j == rank:
                ptrs.append(own.value)
                continue
            peer = ctypes.c_void_p()
            buf = (ctypes.c_uint8 * 64).from_buffer_copy(h)
            check(L.k2b_ipc_open(buf, ctypes.byref(peer)), "k2b_ipc_open")
            ptrs.append(peer.value)
            mapped.append(peer.value)
        return cls(ptrs, rank, owned=own.value, mapped=mapped)

    def close(self) -> None:
        """Unmap the peers and free the own buffer (call after every rank has
        finished using them)."""
        if self._owned is None and not self._mapped:
            return
        import ctypes

        from ._native import lib

        L = lib()
        for ptr in self._mapped:
            L.k2b_ipc_close(ctypes.c_void_p(ptr))
        if self._owned is not None:
            L.k2b_ipc_free(ctypes.c_void_p(self._owned))
        self._owned, self._mapped = None, []


class PeerLost(RuntimeError):
    """Raised by PeerWatch.check: the listed ranks did not reach the step."""

    def __init__(self, step: int, ranks: List[int]):
        super().__init__(f"step {step}: no heartbeat from rank(s) {ranks}")
        self.step, self.ranks = step, ranks


class PeerWatch:
    """Host-side heartbeat of a group of ranks, one key per rank and step in a
    torch.distributed store (the process group's, or any shared one).

    ``check(step)`` publishes this rank's heartbeat for ``step`` and waits at
    most ``timeout_s`` for every peer's; a missing peer raises ``PeerLost``
    before the caller launches the step, so no GPU work of the survivors
    waits on it.  Keys of step - 2 are removed as the watch advances."""

    def __init__(self, store, rank: int, ranks: Sequence[int], timeout_s: float = 10.0,
                 prefix: str = "k2b/alive"):
        if rank not in ranks:
            raise ValueError("PeerWatch: rank not in its group")
        self.store, self.rank, self.ranks = store, rank, list(ranks)
        self.timeout_s, self.prefix = float(timeout_s), prefix

    def _key(self, step: int, rank: int) -> str:
        return f"{self.prefix}/{step}/{rank}"

    def check(self, step: int) -> None:
        import datetime

        self.store.set(self._key(step, self.rank), "1")
        peers = [r for r in self.ranks if r != self.rank]
        try:
            self.store.wait([self._key(step, r) for r in peers], datetime.timedelta(seconds=self.timeout_s))
        except Exception as err:  # store timeout, or the store's host is gone
            missing = []
            for r in peers:
                try:
                    if not self.store.check([self._key(step, r)]):
                        missing.append(r)
                except Exception:
                    missing.append(r)
            raise PeerLost(step, missing or peers) from err
        if step >= 2:
            try:
                self.store.delete_key(self._key(step - 2, self.rank))
            except Exception:
                pass


class TPBlocks:
    """One rank's share of a KV-head tensor-parallel block stack.

    ``blocks`` hold this rank's weight shards (``shard_packed``) and the full
    modulation of the group's latents; ``batch`` latents of ``length`` rows
    form the group's row space, of which this rank holds ``self.shard``."""

    def __init__(self, cfg: ModelConfig, blocks: List[BlockWeights], plan: TPPlan, group, batch: int, length: int,
                 device="cuda", fused: bool = False, watch: Optional[PeerWatch] = None):
        self.cfg, self.blocks, self.plan, self.group = cfg, blocks, plan, group
        self.watch, self.step = watch, 0
        self.batch, self.length = batch, length
        rows = batch * length
        self.rows = rows
        self.shard = plan.rows(rows)
        c, tp, H = self.shard.chunk, plan.tp, cfg.hidden
        pad = c * tp
        hq = (plan.heads // tp)
        kvh = (plan.kvheads // tp)
        f = plan.mlp // tp
        dev = torch.device(device)
        self.act_q = torch.zeros((pad, H // 2), dtype=torch.uint8, device=dev)
        self.act_s = torch.zeros((pad, H // GROUP), dtype=torch.float16, device=dev)
        if not fused:  # NCCL reduce-scatter buffers (pad rows stay zero)
            self.partial = torch.zeros((pad, H), dtype=torch.float32, device=dev)
            self.reduced = torch.empty((c, H), dtype=torch.float32, device=dev)
        self.x1 = torch.empty((c, H), dtype=torch.bfloat16, device=dev)
        self.hq_heads, self.kv_heads_local, self.f_local = hq, kvh, f
        # fused reduce-scatter: receive slots fp32 [tp, chunk, hidden] per rank
        self.fused = fused
        self.slot_bytes = tp * c * H * 4
        self.peers: Optional[PeerSlots] = None
        if fused and group is not None and tp > 1:
            self.peers = PeerSlots.ipc(self.slot_bytes, plan.rank, tp, group)
        self._flag = torch.zeros(1, dtype=torch.int32, device=dev)

    def attach_peers(self, peers: PeerSlots) -> None:
        """Receive buffers set up by the caller (one process driving all ranks)."""
        self.peers = peers

    def close(self) -> None:
        """Release the receive buffers (collective when they are IPC-mapped:
        every rank waits until all have stopped writing into them)."""
        if self.peers is not None:
            if self.peers._mapped or self.peers._owned is not None:
                import torch.distributed as dist

                torch.cuda.synchronize()
                dist.barrier(group=self.group)
            self.peers.close()
            self.peers = None

    def _steps(self, x: torch.Tensor, freqs: torch.Tensor, events=None) -> Iterator[tuple]:
        """The block loop with its collectives as yielded requests:
        ("gather", (q_full, s_full)) and ("reduce_scatter", out, full)."""
        cfg, sh, L, B = self.cfg, self.shard, self.length, self.batch
        c, base, n = sh.chunk, sh.base, sh.count
        r = self.plan.rank
        rows = self.rows
        slot = slice(r * c, r * c + n)
        mark = (lambda i: events[i].record()) if events is not None else (lambda i: None)
        e = 0
        for blk in self.blocks:
            ps, ph, pg, ss, shf, sg = blk.mod.unbind(0)
            mark(e)
            ops.norm_quant_rows(x[:n], blk.prenorm, ps, ph, base_row=base, length=L, batch=B, eps=cfg.eps,
                                out=(self.act_q[slot], self.act_s[slot]))
            mark(e + 1)
            yield ("gather", (self.act_q, self.act_s))
            mark(e + 2)
            q, k, v, _ = ops.qkv(self.act_q[:rows], self.act_s[:rows], blk.wq, blk.wk, blk.wv, blk.qnorm, blk.knorm,
                                 freqs, length=L, eps_q=cfg.qk_eps, eps_k=cfg.qk_eps)
            mark(e + 3)
            qv = q.view(B, L, self.hq_heads, 128).transpose(1, 2)
            kv = k.view(B, L, self.kv_heads_local, 128).transpose(1, 2)
            vv = v.view(B, L, self.kv_heads_local, 128).transpose(1, 2)
            # codes as e4m3 bytes: the out-projection loads them as they are
            oq, os_ = ops.attention_quant_e4m3(qv, kv, vv)
            del q, k, v, qv, kv, vv
            mark(e + 4)
            if self.fused:
                ops.gemm_f32_scatter(oq, os_, blk.wo, self.peers.ptrs, r, c)
                del oq, os_
                mark(e + 5)
                yield ("barrier",)
                mark(e + 6)
                ops.reduce_gated_add(self.peers.ptrs[r], self.plan.tp, c * cfg.hidden, pg, x[:n], base_row=base,
                                     length=L, out=self.x1[:n])
            else:
                ops.gemm_f32(oq, os_, blk.wo, out=self.partial[:rows])
                del oq, os_
                mark(e + 5)
                yield ("reduce_scatter", self.reduced, self.partial)
                mark(e + 6)
                ops.gated_add(self.reduced[:n], pg, x[:n], base_row=base, length=L, out=self.x1[:n])
            ops.norm_quant_rows(self.x1[:n], blk.postnorm, ss, shf, base_row=base, length=L, batch=B, eps=cfg.eps,
                                out=(self.act_q[slot], self.act_s[slot]))
            mark(e + 7)
            yield ("gather", (self.act_q, self.act_s))
            mark(e + 8)
            # the gathered packed codes expanded once; h stays in e4m3 bytes for down
            hq, hs = ops.swiglu_quant_e4m3(ops.expand_e4m3(self.act_q[:rows]), self.act_s[:rows], blk.wg, blk.wu)
            mark(e + 9)
            if self.fused:
                ops.gemm_f32_scatter(hq, hs, blk.wd, self.peers.ptrs, r, c)
                del hq, hs
                mark(e + 10)
                yield ("barrier",)
                mark(e + 11)
                ops.reduce_gated_add(self.peers.ptrs[r], self.plan.tp, c * cfg.hidden, sg, self.x1[:n],
                                     base_row=base, length=L, out=x[:n])
            else:
                ops.gemm_f32(hq, hs, blk.wd, out=self.partial[:rows])
                del hq, hs
                mark(e + 10)
                yield ("reduce_scatter", self.reduced, self.partial)
                mark(e + 11)
                ops.gated_add(self.reduced[:n], sg, self.x1[:n], base_row=base, length=L, out=x[:n])
            if events is not None:
                e += len(PHASES)
        if events is not None:
            events[e].record()

    def forward_(self, x: torch.Tensor, freqs: torch.Tensor, events=None) -> torch.Tensor:
        """In-place forward of this rank's rows x bf16 [chunk, hidden] (rows
        past ``shard.count`` are ignored).  events: optional list of
        len(blocks)*12 + 1 torch.cuda.Event recorded at the phase boundaries
        (PHASES)."""
        self._check(x, freqs, events)
        if self.watch is not None:  # every peer reached this step: nothing waits on a lost rank
            self.watch.check(self.step)
        self.step += 1
        tp, c = self.plan.tp, self.shard.chunk
        for req in self._steps(x, freqs, events):
            if req[0] == "barrier":
                # stream-ordered: every rank's scatter GEMM has finished before
                # any rank's reduce reads its slots
                if tp > 1:
                    import torch.distributed as dist

                    dist.all_reduce(self._flag, group=self.group)
                continue
            if tp == 1:
                if req[0] == "reduce_scatter":
                    req[1].copy_(req[2][:c])
                continue
            if req[0] == "gather":
                gather_rows(req[1], c, self.plan.rank, self.group)
            else:
                reduce_scatter_rows(req[1], req[2], self.group)
        return x

    def _check(self, x, freqs, events):
        cfg = self.cfg
        ops._cuda(x, freqs)
        ops._need(x.dtype == torch.bfloat16 and tuple(x.shape) == (self.shard.chunk, cfg.hidden),
                  "tensor-parallel forward: x must be this rank's [chunk, hidden] bf16 rows")
        ops._need(freqs.dtype == torch.float32 and freqs.numel() == self.length * 256,
                  "tensor-parallel forward: freqs shape")
        ops._need(not self.fused or self.peers is not None, "fused tensor-parallel forward: receive buffers not set")
        if events is not None:
            ops._need(len(events) == len(PHASES) * len(self.blocks) + 1, "tensor-parallel forward: event count")


def local_peer_slots(ranks: Sequence[TPBlocks]) -> List[torch.Tensor]:
    """Receive buffers for fused ranks driven by one process on one device
    (run_lockstep): every rank sees every buffer directly."""
    bufs = [torch.empty(m.slot_bytes // 4, dtype=torch.float32, device=m._flag.device) for m in ranks]
    ptrs = [b.data_ptr() for b in bufs]
    for m in ranks:
        m.attach_peers(PeerSlots(ptrs, m.plan.rank))
    return bufs


def run_lockstep(ranks: Sequence[TPBlocks], xs: Sequence[torch.Tensor], freqs: torch.Tensor) -> None:
    """Runs the ranks of one tensor-parallel group in one process on one
    device, doing each collective with device copies and sums between their
    step generators: the same kernels and shards as the multi-GPU run,
    for checking the sharded path against the unsharded one."""
    for m, x in zip(ranks, xs):
        m._check(x, freqs, None)
    gens = [m._steps(x, freqs) for m, x in zip(ranks, xs)]
    c = ranks[0].shard.chunk
    while True:
        reqs = [next(g, None) for g in gens]
        if all(r is None for r in reqs):
            return
        if any(r is None or r[0] != reqs[0][0] for r in reqs):
            raise RuntimeError("tensor-parallel ranks diverged")
        if reqs[0][0] == "barrier":  # one stream: the scatter kernels already ran
            continue
        if reqs[0][0] == "gather":
            for j, rj in enumerate(reqs):
                for bi in range(len(rj[1])):
                    src = rj[1][bi][j * c:(j + 1) * c]
                    for i, ri in enumerate(reqs):
                        if i != j:
                            ri[1][bi][j * c:(j + 1) * c].copy_(src)
        else:
            for i, ri in enumerate(reqs):
                acc = reqs[0][2][i * c:(i + 1) * c].clone()
                for rj in reqs[1:]:
                    acc += rj[2][i * c:(i + 1) * c]
                ri[1].copy_(acc)
