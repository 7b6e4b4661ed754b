"""Failure detection without any GPU fault: CPU ranks (gloo) where one rank stops.

- a collective that a dead rank never joins ends with an error on the others (short
  process-group timeout) instead of hanging;
- the store heartbeat names the missing or stale rank before the next step is launched."""
import datetime
import os
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests.dist_helpers import _free_port


def _collective_with_dead_peer(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # leaves between steps, never joins the next collective
    t0 = time.time()
    try:
        dist.all_reduce(torch.ones(4))
        q.put(("no error", time.time() - t0))
    except Exception as e:  # noqa: BLE001
        q.put((type(e).__name__, time.time() - t0))
    os._exit(0)


def test_collective_with_dead_peer_errors_instead_of_hanging():
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    ps = [ctx.Process(target=_collective_with_dead_peer, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(60)
    for p in ps:
        if p.is_alive():
            p.kill()
    assert not q.empty(), "rank 0 reported nothing (hung)"
    kind, waited = q.get()
    assert kind != "no error" and waited < 30, (kind, waited)


def _heartbeat(rank, world, port, q):
    from llmt.parallel.health import Heartbeat, PeerFailure
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=20))
    hb = Heartbeat(store, rank, world)
    hb.beat(1)
    store.add("ready", 1)
    while int(store.add("ready", 0)) < world:
        time.sleep(0.05)
    hb.check(max_age_s=10, min_step=1)  # everyone alive at step 1
    if rank == 1:
        store.add("done1", 1)
        time.sleep(3)  # rank 1 stops beating (hung or gone) but keeps the store up for rank 0
        os._exit(0)
    hb.beat(2)
    time.sleep(1.5)
    try:
        hb.check(max_age_s=1.0, min_step=2)
        q.put("no failure detected")
    except PeerFailure as e:
        q.put(f"rank {e.rank}")
    os._exit(0)


def test_heartbeat_names_the_stale_rank():
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    ps = [ctx.Process(target=_heartbeat, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(60)
    for p in ps:
        if p.is_alive():
            p.kill()
    assert not q.empty()
    assert q.get() == "rank 1"


def test_device_error_phase_names():
    from llmt.parallel.health import _phase
    assert "peer 1" in _phase("dp", 101) and "before the update" in _phase("dp", 101)
    assert "reduce-scatter" in _phase("tp", 403)
