"""Replica partitioning and the host aggregation around a measurement, on CPU with gloo.

The box runs one independent replica per GPU (no data-path collective); these tests cover the
host logic with two processes: the request split, the max/sum aggregation bench.py reports, and
a rank that fails before the collective (the survivor's short-timeout group ends with an error
instead of waiting forever).
"""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

import __graft_entry__ as entry

R = entry.load_package().replicas


def test_replica_slice_tiles_exactly():
    for n in (0, 1, 7, 512, 513):
        for world in (1, 2, 3, 4, 8):
            spans = [R.replica_slice(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
                assert a1 == b0
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        R.replica_slice(4, 2, 2)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, mode, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["RANK"] = str(rank)
    os.environ["WORLD_SIZE"] = str(world)
    if mode == "fail" and rank == 1:
        raise SystemExit(3)   # this rank never joins
    try:
        R.init_group(torch, "gloo", timeout_s=5.0)
    except Exception as e:  # the store rendezvous itself timed out
        out.put((rank, "error", type(e).__name__))
        return
    try:
        start, stop = R.replica_slice(512, world, rank)
        secs, toks = R.aggregate(torch, 1.0 + rank, float(stop - start))
        out.put((rank, "ok", (start, stop, secs, toks)))
    except Exception as e:
        out.put((rank, "error", type(e).__name__))
    finally:
        if torch.distributed.is_initialized():
            torch.distributed.destroy_process_group()


def _run(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
    for p in procs:
        if p.is_alive():
            p.kill()
    res = {}
    while not q.empty():
        r, status, val = q.get()
        res[r] = (status, val)
    return res, [p.exitcode for p in procs]


def test_two_replicas_split_and_aggregate():
    res, codes = _run(2, "ok")
    assert codes == [0, 0]
    (s0, v0), (s1, v1) = res[0], res[1]
    assert s0 == s1 == "ok"
    assert (v0[0], v0[1]) == (0, 256) and (v1[0], v1[1]) == (256, 512)
    assert v0[2] == v1[2] == 2.0          # slowest rank's time
    assert v0[3] == v1[3] == 512.0        # all sequences counted once


def test_missing_rank_ends_with_an_error_not_a_hang():
    res, codes = _run(2, "fail")
    assert codes[1] == 3
    assert res.get(0, ("missing",))[0] == "error"
