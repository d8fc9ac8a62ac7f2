"""Batch x head sharding across ranks (world_size 2, gloo, CPU): each rank
computes its block of the (batch, head) grid and one all-gather rebuilds the
global output, equal to the unsharded run.  The per-shard compute here is the
CPU oracle (this checks the partition and the gather; the CUDA kernels behind
each shard are checked by the GPU parity tests)."""
import importlib
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

sh = importlib.import_module("burn-deltanet_b200.sharding")


def test_plan_batch_major():
    p = sh.plan(8, 16, 4)
    assert [(s.b0, s.b1, s.h0, s.h1) for s in p] == [(0, 2, 0, 16), (2, 4, 0, 16), (4, 6, 0, 16), (6, 8, 0, 16)]


def test_plan_head_split():
    p = sh.plan(2, 16, 8)
    assert [(s.b0, s.h0, s.h1) for s in p][:5] == [(0, 0, 4), (0, 4, 8), (0, 8, 12), (0, 12, 16), (1, 0, 4)]
    with pytest.raises(ValueError):
        sh.plan(3, 5, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, batch, heads, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import oracle
        from _inputs import config_inputs

        rng = np.random.default_rng(7)  # every rank builds the same global input
        raw = config_inputs(5, rng, batch, 24, heads, 8, 6)
        raw["g"] = raw["g"] * 0.05
        shards = sh.plan(batch, heads, world)
        me = shards[rank]
        t = lambda k: torch.from_numpy(raw[k]) if raw[k] is not None else None
        loc = {k: sh.take(t(k), me) for k in ("q", "k", "v", "erase", "write", "g")}
        loc["state"] = sh.take(t("state"), me, head_axis=1)
        y, s = oracle.recurrent(*(None if loc[k] is None else loc[k].numpy()
                                  for k in ("q", "k", "v", "erase", "write", "g", "state")))
        y_all = sh.gather(torch.from_numpy(y), shards)
        s_all = sh.gather(torch.from_numpy(s), shards, head_axis=1)
        y0, s0 = oracle.recurrent(raw["q"], raw["k"], raw["v"], raw["erase"], raw["write"], raw["g"], raw["state"])
        result_q.put((rank, float(np.abs(y_all.numpy() - y0).max()), float(np.abs(s_all.numpy() - s0).max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("batch,heads", [(4, 3), (1, 4)])
def test_sharded_equals_unsharded_gloo(batch, heads):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, batch, heads, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    results = sorted(q.get(timeout=5) for _ in range(2))
    for _, ey, es in results:
        assert ey == 0.0 and es == 0.0


def _gather_into_worker(rank, world, port, result_q):
    """gather_into writes every rank's whole-sequence block into a caller-owned buffer, twice in a row into
    the same buffer (the pipelined use), equal to concatenating the blocks."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shards = sh.plan(4, 3, world)
        out = torch.full((4, 5, 3, 2), -1.0)
        ok = True
        for step in range(2):
            local = torch.arange(2 * 5 * 3 * 2, dtype=torch.float32).reshape(2, 5, 3, 2) + 1000 * rank + 10 ** 5 * step
            sh.gather_into(out, local, shards)
            want = torch.cat([torch.arange(60, dtype=torch.float32).reshape(2, 5, 3, 2) + 1000 * r + 10 ** 5 * step
                              for r in range(world)])
            ok = ok and torch.equal(out, want)
        try:
            sh.gather_into(torch.empty(3, 5, 3, 2), local, shards)
            ok = False
        except ValueError:
            pass
        result_q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_gather_into_a_caller_buffer_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_into_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(ok for _, ok in (q.get(timeout=5) for _ in range(2)))


def _failing_worker(rank, world, port, result_q):
    """Rank 1 raises before the gather (it never joins the collective); rank 0 must get an error from the
    gather within the short process-group timeout instead of waiting for ever."""
    import datetime
    import time

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    shards = sh.plan(2, 2, world)
    local = torch.full((1, 3, 2, 4), float(rank))
    if rank == 1:
        raise RuntimeError("rank 1 fails before the gather")
    t0 = time.monotonic()
    try:
        sh.gather(local, shards)
        result_q.put(("no error", time.monotonic() - t0))
    except Exception as e:  # the collective ends with an error
        result_q.put((type(e).__name__, time.monotonic() - t0))
    finally:
        dist.destroy_process_group()


def test_a_rank_that_fails_before_the_gather_ends_the_other_ranks_collective_with_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert procs[1].exitcode != 0  # the failing rank raised
    assert procs[0].exitcode == 0  # the surviving rank returned on its own
    outcome, secs = q.get(timeout=5)
    assert outcome != "no error", "the gather completed without the failed rank"
    assert secs < 60, f"the surviving rank waited {secs:.0f} s"


def _peer_gather_args_worker(rank, world, port, result_q):
    """PeerGather (the copy-engine gather) refuses, on every rank alike and before any exchange, what it
    cannot serve: head-split shards, a shard list of the wrong length and a buffer not on the GPU."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        refused = []
        for out, shards in ((torch.zeros(1, 4), sh.plan(1, 4, world)),      # heads split over the ranks
                            (torch.zeros(4, 4), sh.plan(4, 4, 1)),          # one shard for two ranks
                            (torch.zeros(4, 4), sh.plan(4, 4, world))):     # a host buffer
            try:
                sh.PeerGather(out, shards)
                refused.append(False)
            except ValueError:
                refused.append(True)
        dist.barrier()  # the ranks are still in step: nothing above entered a collective
        result_q.put((rank, all(refused)))
    finally:
        dist.destroy_process_group()


def test_peer_gather_refuses_what_it_cannot_serve_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_gather_args_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(ok for _, ok in (q.get(timeout=5) for _ in range(2)))
