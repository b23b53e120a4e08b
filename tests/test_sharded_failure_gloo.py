"""Failure of a rank between steps of the point-sharded coupling (two CPU
ranks, gloo): rank 1 completes one rank-ordered sum and then dies without
leaving the process group; rank 0's next sum must end with an error within
the process group's short timeout instead of waiting forever. The failure
is made on the host (a process that exits), never on a GPU."""

import datetime
import os
import socket
import time

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

PG_TIMEOUT_S = 5


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=PG_TIMEOUT_S))
        from flashslice_b200 import sharded
        first = sharded.ordered_sum_many([torch.full((4,), float(rank + 1))])[0]
        if rank == 1:
            q.put((rank, "left", float(first.sum())))
            q.close()
            q.join_thread()  # the message is out before the process dies
            os._exit(0)  # dies between steps: no destroy_process_group, no goodbye
        time.sleep(0.5)
        t0 = time.monotonic()
        try:
            sharded.ordered_sum_many([torch.ones(4)])
            q.put((rank, "no error", time.monotonic() - t0))
        except Exception as e:  # the survivor's collective fails instead of hanging
            q.put((rank, "raised " + type(e).__name__, time.monotonic() - t0))
    except Exception as e:
        q.put((rank, "setup failed: %r" % e, 0.0))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_survivor_raises_when_a_rank_dies_between_steps():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = {}
        for _ in procs:
            try:
                rank, what, val = q.get(timeout=120)
            except Exception:
                break
            res[rank] = (what, val)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert set(res) == {0, 1}, res
    assert res[1][0] == "left" and res[1][1] == 4 * 3.0, res
    what, waited = res[0]
    assert what.startswith("raised"), res
    # the error came from the process group (closed connection or its timeout),
    # well before anything like a hang
    assert waited < 4 * PG_TIMEOUT_S + 30, waited
