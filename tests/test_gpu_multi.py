"""Two-rank GPU checks of the copy-engine all-gather (sharding.PeerGather): one process per GPU over
NCCL, each rank's block of a batch-major prefill output pushed to its peer by peer-to-peer copies through
CUDA IPC mappings.  The gathered buffer must equal NCCL's all_gather_into_tensor bit for bit, and the
sharded prefill, gathered, must equal the unsharded prefill of the whole batch.  Skipped with fewer than
two GPUs (the multi-process host logic is covered on CPU by tests/test_sharding.py over gloo)."""
import datetime
import importlib
import math
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        dn = importlib.import_module("burn-deltanet_b200")
        sh = importlib.import_module("burn-deltanet_b200.sharding")
        bench = importlib.import_module("bench")
        B, T = 2 * world, 300
        full = bench.make_prefill("deltanet", B, T, 1, "cuda", 77)  # the same global batch on every rank
        shards = sh.plan(B, bench.H, world)
        me = shards[rank]
        x = {k: None if t is None else t[me.b0:me.b1].contiguous() for k, t in full.items()}
        out = torch.zeros(B, T, bench.H, bench.D, device="cuda", dtype=torch.bfloat16)
        pg = sh.PeerGather(out, shards)
        args = lambda z: (z["q"], z["k"], z["v"], z["erase"], z["write"], z["g"], z["state"], False, 64,
                          1.0 / math.sqrt(bench.D))
        dn.delta_chunk_recalculated(*args(x), y_out=out[me.b0:me.b1])
        ev = torch.cuda.Event()
        ev.record()
        for e in pg.push(ev):
            torch.cuda.current_stream().wait_event(e)
        torch.cuda.synchronize()
        dist.barrier()
        ref = torch.empty_like(out)
        dist.all_gather_into_tensor(ref, out[me.b0:me.b1].contiguous())
        y_full, _ = dn.delta_chunk_recalculated(*args(full))
        torch.cuda.synchronize()
        res = (bool(torch.equal(out, ref)), bool(torch.equal(out, y_full)))
        dist.barrier()
        pg.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, res, ""))
    except Exception as e:  # noqa: BLE001 (reported to the parent)
        q.put((rank, None, f"{type(e).__name__}: {e}"))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_gather_matches_nccl_and_the_unsharded_prefill():
    import sys

    import torch.multiprocessing as mp

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    if root not in sys.path:
        sys.path.insert(0, root)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world, port = 2, _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, res, err in results:
        assert not err, f"rank {rank}: {err}"
        assert res == (True, True), f"rank {rank}: equal to NCCL's gather / to the unsharded prefill: {res}"
