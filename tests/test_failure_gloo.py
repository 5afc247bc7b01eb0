"""A rank that leaves between steps of a sharded forward (2 CPU ranks, gloo; no GPU).

The survivor's next collective of the crossbar-sharded layer (RowShardedLinearMem's all-reduce of
the partial sums, crossbar_shard.py) must end with an error within the process group's timeout
instead of waiting for ever.  The leaving rank exits without tearing down its process group, as a
crashed process would.
"""
import datetime
import os
import queue
import socket
import time

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _row_shard(world, rank, bias):
    """The host side of a row-sharded layer (its collective and bias) without programmed crossbars."""
    from memintelli_flash_b200.crossbar_shard import RowShardedLinearMem
    lay = RowShardedLinearMem.__new__(RowShardedLinearMem)
    torch.nn.Module.__init__(lay)
    lay.group, lay.world, lay.rank, lay.full_bias = None, world, rank, bias
    return lay


def _worker(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    lay = _row_shard(world, rank, torch.ones(3))
    y = lay._finish(torch.full((2, 3), float(rank + 1)))          # step 1: every rank takes part
    q.put(("step1", rank, y.tolist()))
    if rank == 1:
        q.close()
        q.join_thread()                                            # deliver step 1's report first
        os._exit(0)                                                # leaves between steps
    t0 = time.time()
    try:
        lay._finish(torch.full((2, 3), 1.0))                       # step 2: the peer is gone
        q.put(("step2", rank, "no error", time.time() - t0))
    except Exception as e:                                         # noqa: BLE001 - any backend error
        q.put(("step2", rank, type(e).__name__, time.time() - t0))
    q.close()
    q.join_thread()
    os._exit(0)


def test_survivor_gets_a_bounded_error_when_a_rank_leaves():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = []
    deadline = time.time() + 120
    while len(got) < 3 and time.time() < deadline:
        try:
            got.append(q.get(timeout=5))
        except queue.Empty:
            pass
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    step1 = [g for g in got if g[0] == "step1"]
    step2 = [g for g in got if g[0] == "step2"]
    assert len(step1) == 2 and all(g[2] == [[4.0, 4.0, 4.0]] * 2 for g in step1)   # 1 + 2 + bias 1
    assert len(step2) == 1, got
    _, rank, outcome, waited = step2[0]
    assert rank == 0 and outcome != "no error"
    assert waited < 60.0
