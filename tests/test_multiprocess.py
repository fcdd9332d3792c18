"""Multi-rank host logic of the row-sharded encode, on CPU with the gloo backend
(world size 2 and 3): every rank derives the same FLOP-balanced plan, the bands
are disjoint and cover the tile, the per-rank work adds up to the whole tile,
and the max-over-ranks reduction that bench.py applies to timings works. A rank
that fails before the collective makes the others fail fast (short timeout)
instead of hanging."""
import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ORACLE, PKG, REPO


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, fail_rank):
    sys.path[:0] = [str(PKG), str(ORACLE), str(REPO)]
    import bench
    import oracle
    import synth
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        if rank == fail_rank:
            raise RuntimeError("injected failure before the collective")
        tile = synth.make_tile(H=37, W=11, T2=20, Ta=10, Td=10, p=0.5, seed=77, cloudy=True)
        r0, r1 = bench.rank_rows(tile, rank, world)
        t2, t1 = oracle.tile_tokens(tile)
        flop = oracle.pixel_flop(t2, t1).reshape(37, 11)[r0:r1].sum()
        t = torch.tensor([float(r0), float(r1), float(flop), float(rank + 1)], dtype=torch.float64)
        gathered = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(gathered, t)
        mx = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        q.put((rank, [g.tolist() for g in gathered], mx.item(), float(oracle.pixel_flop(t2, t1).sum())))
    except Exception as e:  # report and leave between steps, no collective in flight
        q.put((rank, "error", str(e), None))
    finally:
        dist.destroy_process_group()


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(60)
    return out


@pytest.mark.parametrize("world", [2, 3])
def test_bands_cover_and_agree(world):
    res = _run(world)
    assert all(r[1] != "error" for r in res), res
    views = [r[1] for r in res]
    assert all(v == views[0] for v in views)  # every rank saw the same plan
    bands = sorted((int(v[0]), int(v[1])) for v in views[0])
    assert bands[0][0] == 0 and bands[-1][1] == 37
    assert all(a[1] == b[0] for a, b in zip(bands, bands[1:]))
    total = res[0][3]
    assert abs(sum(v[2] for v in views[0]) - total) < 1e-6 * total
    assert all(r[2] == world for r in res)  # max over ranks


def test_failed_rank_does_not_hang():
    res = _run(2, fail_rank=1)
    by_rank = {r[0]: r for r in res}
    assert by_rank[1][1] == "error"
    assert by_rank[0][1] == "error"  # the survivor's collective ends with an error, not a hang
