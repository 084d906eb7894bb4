"""Failure detection of the multi-GPU path, on the host (gloo ranks on the
CPU, no GPU): a rank that raises or exits between steps is reported on its
peer by k2b.parallel.PeerWatch before the peer launches the step, and a
collective that a live peer never joins ends with the process group's own
timeout instead of waiting for good."""
import json
import os
import socket

import pytest

HEARTBEAT_S = 2.0  # PeerWatch limit
GROUP_S = 3  # process-group (collective) timeout


class InjectedFailure(Exception):
    """A host-side failure of one rank between steps."""


def _fault_rank(rank, world, port, mode, outdir):
    import datetime
    import time

    import torch
    import torch.distributed as dist

    from k2b.parallel import PeerLost, PeerWatch, reduce_scatter_rows

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=GROUP_S))
    watch = PeerWatch(dist.distributed_c10d._get_default_store(), rank, range(world), timeout_s=HEARTBEAT_S)
    record = {"rank": rank, "steps": 0}
    t0 = time.monotonic()
    try:
        for step in range(3):
            if rank == 1 and step == 1:
                if mode == "raise":
                    raise InjectedFailure("rank 1 fails between steps")
                if mode == "exit":
                    os._exit(3)
            t0 = time.monotonic()
            watch.check(step)
            if rank == 1 and step == 1 and mode == "drop":
                time.sleep(GROUP_S + 4)  # alive, but never joins this step's collective
                break
            full = torch.full((world * 4, 8), float(rank + 1))
            out = torch.empty((4, 8))
            reduce_scatter_rows(out, full, None)
            assert float(out[0, 0]) == world * (world + 1) / 2
            record["steps"] = step + 1
    except PeerLost as err:
        record.update(error="PeerLost", ranks=err.ranks, step=err.step, waited=time.monotonic() - t0)
    except RuntimeError as err:  # the process group's collective timeout
        record.update(error=type(err).__name__, waited=time.monotonic() - t0)
    with open(os.path.join(outdir, f"rank{rank}.json"), "w") as f:
        json.dump(record, f)
    os._exit(0)  # no destroy_process_group: the peer may be gone


def _run(mode, outdir, world=2):
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_fault_rank, args=(r, world, port, mode, str(outdir))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()  # this test's own child, by its handle
        p.join()
    assert not alive, "a rank hung"
    recs = {}
    for r in range(world):
        path = os.path.join(outdir, f"rank{r}.json")
        if os.path.exists(path):
            with open(path) as f:
                recs[r] = json.load(f)
    return procs, recs


def test_all_ranks_present_run_every_step(tmp_path):
    procs, recs = _run("none", tmp_path)
    assert [p.exitcode for p in procs] == [0, 0]
    assert recs[0] == {"rank": 0, "steps": 3} and recs[1] == {"rank": 1, "steps": 3}


@pytest.mark.parametrize("mode, code", [("raise", 1), ("exit", 3)])
def test_lost_rank_reported_before_the_step(tmp_path, mode, code):
    procs, recs = _run(mode, tmp_path)
    assert procs[1].exitcode == code and 1 not in recs
    r0 = recs[0]
    assert r0["error"] == "PeerLost" and r0["ranks"] == [1] and r0["step"] == 1
    assert r0["steps"] == 1  # step 0 completed; step 1 launched nothing
    assert HEARTBEAT_S * 0.5 <= r0["waited"] < HEARTBEAT_S + 5


def test_dropped_collective_ends_with_the_group_timeout(tmp_path):
    procs, recs = _run("drop", tmp_path)
    assert [p.exitcode for p in procs] == [0, 0]
    r0 = recs[0]
    assert r0["steps"] == 1 and r0["error"] != "PeerLost"  # the heartbeat of step 1 was there
    assert GROUP_S * 0.5 <= r0["waited"] < GROUP_S + 10
    assert recs[1] == {"rank": 1, "steps": 1}


def test_peer_watch_in_one_process():
    """PeerWatch on an in-process store: a peer's heartbeat present or missing."""
    import datetime

    import torch.distributed as dist

    from k2b.parallel import PeerLost, PeerWatch

    store = dist.HashStore()
    store.set_timeout(datetime.timedelta(seconds=5))
    w0 = PeerWatch(store, 0, [0, 1], timeout_s=0.3)
    with pytest.raises(PeerLost) as lost:
        w0.check(0)  # rank 1 never beats
    assert lost.value.ranks == [1] and lost.value.step == 0
    PeerWatch(store, 1, [0, 1], timeout_s=0.3).check(0)  # rank 0's key for step 0 is already there
    w0.check(0)  # now both keys exist
    with pytest.raises(ValueError):
        PeerWatch(store, 2, [0, 1])
