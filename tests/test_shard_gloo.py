"""Crossbar sharding across 2 CPU ranks (gloo): shard boundaries keep the CIM result exact.

Each rank evaluates its column (or row) shard with the exact oracle; the gathered
(or summed) result must equal the unsharded layer.  This is the host logic of
the multi-GPU path (crossbar_shard.py) without a GPU.
"""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from memintelli_flash_b200.crossbar_shard import shard_bounds

SM = [1, 1, 2, 2, 2]
ENG = dict(HGS=1e-5, LGS=1e-8, g_level=4, rdac=4, radc=4096, rate_stuck_HGS=0.0, read_variation=0.0,
           vnoise=0.0, write_variation=0.0)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from oracle import cim_oracle as O
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(0)
    x = rng.standard_normal((24, 384)).astype(np.float32)
    w = rng.standard_normal((384, 320)).astype(np.float32)
    eng = O.Engine(**ENG)
    xs = O.slice_matrix(x, SM, None, (1, 32), (1, 128))
    # column shard
    lo, hi = shard_bounds(320, 128, world, rank)
    ws = O.slice_matrix(w[:, lo:hi], SM, None, (32, 32), (128, 128))
    y_loc = torch.from_numpy(O.mvm_exact(xs, ws, eng))
    sizes = [shard_bounds(320, 128, world, r)[1] - shard_bounds(320, 128, world, r)[0] for r in range(world)]
    pad = torch.zeros(24, max(sizes), dtype=torch.float64)
    pad[:, : hi - lo] = y_loc
    parts = [torch.zeros_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad)
    y_col = torch.cat([p[:, :n] for p, n in zip(parts, sizes)], dim=1).numpy()
    # row shard (K split on 128-row blocks)
    lo, hi = shard_bounds(384, 128, world, rank)
    xs_r = O.slice_matrix(x[:, lo:hi], SM, None, (1, 32), (1, 128))
    ws_r = O.slice_matrix(w[lo:hi], SM, None, (32, 32), (128, 128))
    y_row = torch.from_numpy(np.ascontiguousarray(O.mvm_exact(xs_r, ws_r, eng)))
    dist.all_reduce(y_row)
    if rank == 0:
        ws_full = O.slice_matrix(w, SM, None, (32, 32), (128, 128))
        y_full = O.mvm_exact(xs, ws_full, eng)
        q.put((np.abs(y_col - y_full).max(), np.abs(y_row.numpy() - y_full).max(), np.abs(y_full).max()))
    dist.barrier()
    dist.destroy_process_group()


def test_column_and_row_shards_are_exact():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    col_err, row_err, scale = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert col_err == 0.0                       # column shards are bit-identical
    assert row_err <= 1e-12 * scale             # row shards: exact up to summation order


def _reject_worker(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from memintelli_flash_b200.crossbar_shard import ColumnShardedLinearMem, RowShardedLinearMem
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    errs = []
    w = torch.zeros(256, 256)
    cases = [
        # a per-matrix weight scale would span both shards
        (RowShardedLinearMem, w, dict(weight_quant_gran="per-matrix")),
        (ColumnShardedLinearMem, w, dict(weight_quant_gran="per-matrix")),
    ]
    if rank == 1:   # 128 output columns in 128-column blocks leave rank 1 without a shard
        cases.append((ColumnShardedLinearMem, torch.zeros(128, 256), dict(weight_quant_gran=(128, 128))))
    for cls, weight, kw in cases:
        try:
            cls(None, weight, None, SM, SM, weight_paral_size=(32, 32), **kw)
            errs.append(None)
        except ValueError as e:          # raised on the host, before any crossbar is programmed
            errs.append(str(e))
    q.put((rank, errs))
    dist.barrier()
    dist.destroy_process_group()


def test_sharding_rejects_string_granularity_and_empty_shards():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_reject_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=240) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in (0, 1):
        assert got[r][0] and "string granularity" in got[r][0]
        assert got[r][1] and "string granularity" in got[r][1]
    assert len(got[0]) == 2
    assert got[1][2] and "empty crossbar shard" in got[1][2]


def test_noise_calls_per_shard():
    """Read variation: one call index per rank (shards draw independently, rank 0 keeps the unsharded
    draw).  Voltage noise: row shards hold different input features (own call); column shards share the
    replicated input (call 0, one draw for all columns as in one crossbar)."""
    from memintelli_flash_b200.crossbar_shard import noise_calls
    assert noise_calls(1, 0, 0) == (0, 0) and noise_calls(1, 0, 1) == (0, 0)
    assert [noise_calls(4, r, 0) for r in range(4)] == [(0, 0), (1, 0), (2, 0), (3, 0)]
    assert [noise_calls(4, r, 1) for r in range(4)] == [(0, 0), (1, 1), (2, 2), (3, 3)]
