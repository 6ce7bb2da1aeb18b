"""Failure detection without any GPU fault: a gloo rank that leaves (or never joins) is reported by
the heartbeat monitor, and a collective whose peer never arrives times out on the host."""

import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q) -> None:  # noqa: ANN001
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    from axrl_b200.runtime.health import HeartbeatMonitor, RankFailure, bounded_collective

    store = dist.distributed_c10d._get_default_store()
    # a generous staleness limit: a loaded CI host can delay a heartbeat thread by a second or more
    hb = HeartbeatMonitor(store, rank, world, interval_s=0.1, timeout_s=4.0).start()
    try:
        t = torch.ones(4)
        dist.all_reduce(t)  # everyone alive: one normal step
        assert t[0].item() == world
        hb.check()
        if rank == 1:  # rank 1 leaves between steps, with nothing in flight
            hb.stop(announce_exit=True)
            q.put((rank, "ok"))
            return
        t0 = time.time()
        while True:
            try:
                hb.check()
            except RankFailure as e:
                assert e.ranks == [1]
                break
            assert time.time() - t0 < 30, "failure not detected"
            time.sleep(0.05)
        # a collective posted anyway cannot complete: it either times out on the host or fails
        # when the transport notices the peer is gone -- both surface as an exception here
        try:
            bounded_collective(dist.all_reduce, torch.ones(4), timeout_s=1.0)
            q.put((rank, "collective unexpectedly completed"))
        except (TimeoutError, RuntimeError):
            q.put((rank, "ok"))
    except Exception:  # noqa: BLE001
        import traceback

        q.put((rank, traceback.format_exc()))
    finally:
        hb.stop(announce_exit=False)
        q.close()
        q.join_thread()  # flush the result before leaving
        os._exit(0)  # do not wait on the abandoned collective


def test_rank_leaves_is_detected_and_collective_is_bounded():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=30)
    assert res == {0: "ok", 1: "ok"}, res


def test_never_joined_rank_reported():
    from axrl_b200.runtime.health import HeartbeatMonitor, RankFailure

    store = dist.HashStore()
    hb = HeartbeatMonitor(store, 0, 3, interval_s=0.05, timeout_s=0.3).start()
    HeartbeatMonitor(store, 1, 3, interval_s=0.05, timeout_s=0.3).start()
    time.sleep(0.5)
    with pytest.raises(RankFailure) as e:
        hb.check()
    assert e.value.ranks == [2]
    hb.stop()
