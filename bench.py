#!/usr/bin/env python3
"""Benchmark of the delta-rule core on B200: prefill and decode tokens/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload deltanet|deltaproduct2|deltaproduct3|gdn2]

One JSON line on rank 0.  The default workload is BASELINE config 2 (the
DeltaNet prefill in bf16, B=8 T=4096 H=16 dk=dv=128, chunk 64, fp32 state):
a "step" is one dc_chunk_fwd over that batch.  With N GPUs (torchrun, one
rank per GPU) every rank owns its own batch of 8 sequences — batch x head
sharding with no collective on the data path — so the work per GPU is fixed
("scaling": "weak") and ``value`` counts the tokens of all ranks.  The decode
of BASELINE config 3 (256 sequences, H=16, fp32 state, one fused tick per
step) is measured in the same run and reported under "decode", the backward
(dc_chunk_bwd at config 2's shapes) under "backward", and the front-end and
epilogue kernels under "prologue", "gates" and "out_norm".

``--workload gdn2`` is BASELINE config 5: one batch of 16 sequences sharded
over the N GPUs ("scaling": "strong"), and its decode is config 5's own: 512
GDN-2 step() tokens from each rank's prefill final state.

Inputs are synthetic (seeded, the configs' recipes) and larger than L2; every
number is device time from CUDA events on the launching stream, max over ranks.
"""
from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

H, D, L = 16, 128, 64
WORKLOADS = {
    # name: (config index, batch per GPU (or in all, for STRONG), tokens, n_householder, gates)
    "deltanet": (2, 8, 4096, 1, "deltanet"),
    "deltaproduct2": (4, 4, 8192, 2, "deltaproduct"),
    "deltaproduct3": (4, 4, 8192, 3, "deltaproduct"),
    "gdn2": (5, 16, 16384, 1, "gdn2"),
}
# Config 5 is one batch of 16 sequences sharded over the GPUs (strong scaling); the others keep their
# batch per GPU (weak scaling).
STRONG = {"gdn2"}
CFG5_DECODE_STEPS = 512
DECODE_STEPS = 1024  # config 3: 1024 consecutive step() calls
# Flop (2 x multiply-adds) of the chunked backward per token-head, d = 128 and its chunks of L = 32:
# prep 4 L d (A, att, W, U); the scans 2 d^2 forward (V', S) and L d + 3 d^2 back (dV', dS); the gradients
# 3 d^2 + L d (the S products, datt), 2 L d (dT), 2 L d (d(wv), dKg), 2 L^2 (X, dA), 4 L d (F, Fa products).
BWD_L = 32
BWD_FLOP = 2 * (14 * BWD_L * D + 8 * D * D + 2 * BWD_L * BWD_L)
DECODE = dict(batch=256, heads=16, d=128)


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        p = json.load(open(path))
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


# ---------------------------------------------------------------------------
# Synthetic inputs (the configs' recipes), generated on the device.
# ---------------------------------------------------------------------------
def l2n(x):
    return x / torch.sqrt((x.float() * x.float()).sum(-1, keepdim=True) + 1e-6)


def make_prefill(kind, batch, tokens, u, device, seed):
    g = torch.Generator(device=device).manual_seed(seed)
    rn = lambda *s: torch.randn(*s, device=device, generator=g)
    bf = torch.bfloat16
    su = tokens * u
    q = l2n(rn(batch, tokens, H, D)).to(bf)
    k = l2n(rn(batch, su, H, D)).to(bf)
    v = rn(batch, su, H, D).to(bf)
    gate = None
    if kind == "deltanet":
        erase = write = torch.sigmoid(rn(batch, su, H, 1))
    elif kind == "deltaproduct":
        erase = write = 2 * torch.sigmoid(rn(batch, su, H, 1))
        a = torch.rand(1, 1, H, 1, device=device, generator=g) * math.log(16.0)
        gate = (-torch.exp(a) * torch.nn.functional.softplus(rn(batch, tokens, H, 1))).float()
    elif kind == "gdn2":
        erase = torch.sigmoid(rn(batch, su, H, D))
        write = torch.sigmoid(rn(batch, su, H, D))
        a = torch.rand(1, 1, H, D, device=device, generator=g) * math.log(16.0)
        gate = (-torch.exp(a) * torch.nn.functional.softplus(rn(batch, tokens, H, D))).float()
    else:
        raise ValueError(kind)
    # The gates stay float32 (one dtype for erase, write and g; g needs it).
    erase, write = erase.float(), write.float()
    state = torch.zeros(batch, H, D, D, device=device)
    return dict(q=q, k=k, v=v, erase=erase.contiguous(), write=write.contiguous(), g=gate, state=state)


def make_decode(device, seed):
    g = torch.Generator(device=device).manual_seed(seed)
    b, h, d = DECODE["batch"], DECODE["heads"], DECODE["d"]
    rn = lambda *s: torch.randn(*s, device=device, generator=g)
    bf = torch.bfloat16
    a = torch.rand(1, h, 1, device=device, generator=g) * math.log(16.0)
    return dict(
        q=l2n(rn(b, h, d)).to(bf), k=l2n(rn(b, h, d)).to(bf), v=rn(b, h, d).to(bf),
        erase=torch.sigmoid(rn(b, h, 1)), g=(-torch.exp(a) * torch.nn.functional.softplus(rn(b, h, 1))),
        state=torch.randn(b, h, d, d, device=device, generator=g) * 0.02,
    )


# ---------------------------------------------------------------------------
# Clock sampling during the timed region.
# ---------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.25)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, smax, reasons = [], None, set()
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(self.NAMES, parts[3:7]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# Distributed plumbing (one process per GPU).
# ---------------------------------------------------------------------------
def setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}: launch N>1 with torchrun")
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# CPU baseline: the oracle (the reference algorithm restated in C) on the
# host cores, bounded sample.
# ---------------------------------------------------------------------------
def cpu_baseline(workload, budget_s=12.0):
    import oracle

    _, _, tokens_full, u, kind = WORKLOADS[workload]
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(0)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from _inputs import config_inputs

    cfg = {"deltanet": 2, "deltaproduct": 4, "gdn2": 5}[kind]
    tokens = 256
    batch = max(1, -(-threads // H))  # enough (batch, head) pairs for every host thread
    samples = []
    while True:
        raw = config_inputs(cfg, rng, batch, tokens, H, D, D, u=u)
        raw = {k: (None if v is None else v.astype(np.float32)) for k, v in raw.items()}
        t0 = time.perf_counter()
        oracle.householder("chunk", raw["q"], raw["k"], raw["v"], raw["erase"], raw["write"], raw["g"],
                           raw["state"], u, chunk_len=L, dtype=np.float32, threads=threads)
        dt = time.perf_counter() - t0
        samples.append((tokens, dt))
        if dt > budget_s / 4 or tokens >= tokens_full:
            break
        tokens = min(tokens_full, tokens * 4)
    tokens, dt = samples[-1]
    # At the full sequence length, widen the sample toward the workload's own batch, then repeat it until
    # it holds about budget_s of CPU work.
    full_batch = WORKLOADS[workload][1]
    if dt < budget_s / 2 and batch < full_batch:
        batch = min(full_batch, max(batch + 1, int(batch * budget_s / 2 / dt)))
        raw = config_inputs(cfg, rng, batch, tokens, H, D, D, u=u)
        raw = {k: (None if v is None else v.astype(np.float32)) for k, v in raw.items()}
        dt = 0.0
    reps = 0
    total = 0.0
    while total < 0.8 * budget_s and reps < 64:
        t0 = time.perf_counter()
        oracle.householder("chunk", raw["q"], raw["k"], raw["v"], raw["erase"], raw["write"], raw["g"],
                           raw["state"], u, chunk_len=L, dtype=np.float32, threads=threads)
        total += time.perf_counter() - t0
        reps += 1
    return {"value": reps * batch * tokens / total, "unit": "tok/s", "cores": min(threads, batch * H),
            "kind": "port", "cpu_model": cpu_model(), "host_threads": threads,
            "sample": f"oracle chunk path fp32 (chunk 64, OpenMP over heads), B={batch} T={tokens} H={H} d={D}"
                      f"{' u=' + str(u) if u > 1 else ''}, {reps} call(s) in {total:.2f} s"}


# ---------------------------------------------------------------------------
# Measurements
# ---------------------------------------------------------------------------
def algorithmic_bytes(x, tokens_out):
    """Bytes a prefill call must move: every input once, y once, the state in and out."""
    n = sum(t.numel() * t.element_size() for k, t in x.items() if t is not None)
    n += tokens_out * H * D * 2  # y (bf16)
    n += x["state"].numel() * 4  # final state
    return n


def time_prefill(dn, x, u, steps, warmup):
    b, s = x["q"].shape[0], x["q"].shape[1]
    y = torch.empty(b, s, H, D, device="cuda", dtype=torch.bfloat16)
    s_out = torch.empty_like(x["state"])
    gated = x["g"] is not None

    def call():
        dn.delta_chunk_recalculated(x["q"], x["k"], x["v"], x["erase"], x["write"], x["g"], x["state"],
                                    gated, L, 1.0 / math.sqrt(D), n_householder=u, y_out=y, state_out=s_out)

    for _ in range(warmup):
        call()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        call()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def time_prefill_out_norm(dn, x, u, steps, warmup):
    """The prefill followed by the plain output norm (dc_chunk_fwd_out_norm, the norm inside the tensor-core
    kernel's read-out) against the same two steps as separate calls (dc_chunk_fwd, then dc_out_norm in place
    on y).  Returns (ms of the one call, ms as two calls, whether the norm ran inside the prefill kernel)."""
    b, s = x["q"].shape[0], x["q"].shape[1]
    y = torch.empty(b, s, H, D, device="cuda", dtype=torch.bfloat16)
    s_out = torch.empty_like(x["state"])
    w = torch.rand(D, device="cuda", generator=torch.Generator(device="cuda").manual_seed(5)) + 0.5
    args = (x["q"], x["k"], x["v"], x["erase"], x["write"], x["g"], x["state"], x["g"] is not None, L,
            1.0 / math.sqrt(D))

    def fused():
        dn.delta_chunk_recalculated_out_norm(*args, w, n_householder=u, y_out=y, state_out=s_out)

    def two():
        dn.delta_chunk_recalculated(*args, n_householder=u, y_out=y, state_out=s_out)
        dn.out_norm(y, None, w, out=y)

    times = []
    for call in (fused, two):
        for _ in range(max(3, warmup)):
            call()
        torch.cuda.synchronize()
        stream = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            call()
        e1.record(stream)
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) / steps)
    return times[0], times[1], dn.chunk_out_norm_is_fused(*args[:9], w, n_householder=u, out_dtype=torch.bfloat16)


def time_prefill_f32(dn, steps, warmup, batch=8, tokens=4096):
    """Config 2's prefill at the reference's own precision: float32 q, k, v (and y) through the
    fp32-accurate chunked path (dc_chunk_kernel_choice 3, over a workspace), and through the CUDA-core
    kernel it replaces, on the same inputs (inputs larger than L2).  Returns (ms chunked, ms CUDA-core,
    algorithmic bytes per call, choice)."""
    x = make_prefill("deltanet", batch, tokens, 1, "cuda", 21)
    for n in ("q", "k", "v"):
        x[n] = x[n].float()
    args = (x["q"], x["k"], x["v"], x["erase"], x["write"], x["g"], x["state"], False, L, 1.0 / math.sqrt(D))
    y = torch.empty(batch, tokens, H, D, device="cuda")
    s_out = torch.empty_like(x["state"])
    a, _, _ = dn.core._chunk_args(*args[:7], False, L, args[9], 1, torch.float32, False, False, False, y, s_out,
                                  dn.core._check_tensor, None)
    need = int(dn._abi.lib().dc_chunk_workspace_size(a))
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device="cuda")
    a.workspace, a.workspace_bytes = ws.data_ptr(), need
    choice = int(dn._abi.lib().dc_chunk_kernel_choice(a))

    def timed(call, n):
        for _ in range(max(1, min(warmup, 3))):
            call()
        torch.cuda.synchronize()
        stream = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            call()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    ms = timed(lambda: dn.delta_chunk_recalculated(*args, workspace=ws, y_out=y, state_out=s_out), steps)
    ms_simt = timed(lambda: dn.delta_chunk_recalculated(*args, force_simt=True, y_out=y, state_out=s_out), 1)
    nbytes = sum(t.numel() * t.element_size() for t in x.values() if t is not None)
    nbytes += y.numel() * 4 + s_out.numel() * 4
    return ms, ms_simt, nbytes, choice


def time_prefill_gathered(dn, x, u, steps, warmup, world, mode="peer"):
    """Each step: the prefill of this rank's batch, then the all-gather of its y (bf16) into every rank's
    global output [world x batch, T, H, dv] -- the north star's one collective.  Returns (ms per step on
    this rank, whether the gathered output matched NCCL's on this rank); the caller takes the max over
    ranks.  At one GPU there is nothing to gather and this is the plain prefill.

    mode "peer": the prefill writes this rank's block of the global buffer directly and the copy engines
    push it to every peer (sharding.PeerGather); two global buffers alternate, so the copies of step i run
    beside the prefill of step i+1, and the timed region ends once every copy has landed.  mode "nccl":
    dist.all_gather_into_tensor on the prefill's stream after each step (running it beside the next
    step's prefill was measured slower: NCCL's 32 CTAs take SMs the one-wave prefill needs)."""
    if world == 1:
        return time_prefill(dn, x, u, steps, warmup), True
    import torch.distributed as dist
    sh = importlib.import_module("burn-deltanet_b200.sharding")
    rank = dist.get_rank()
    b, s = x["q"].shape[0], x["q"].shape[1]
    shards = sh.plan(b * world, H, world)
    s_out = torch.empty_like(x["state"])
    gated = x["g"] is not None
    prefill = lambda y: dn.delta_chunk_recalculated(x["q"], x["k"], x["v"], x["erase"], x["write"], x["g"],
                                                    x["state"], gated, L, 1.0 / math.sqrt(D), n_householder=u,
                                                    y_out=y, state_out=s_out)
    compute = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if mode == "nccl":
        y = torch.empty(b, s, H, D, device="cuda", dtype=torch.bfloat16)
        out = torch.empty(world * b, s, H, D, device="cuda", dtype=torch.bfloat16)

        def step(_):
            prefill(y)
            sh.gather_into(out, y, shards)

        drain = lambda: None
    else:
        outs = [torch.empty(world * b, s, H, D, device="cuda", dtype=torch.bfloat16) for _ in range(2)]
        pgs = [sh.PeerGather(o, shards, streams=GATHER["streams"], parts=GATHER["parts"]) for o in outs]
        pending = [[], []]
        b0, b1 = shards[rank].b0, shards[rank].b1

        def step(i):
            k = i & 1
            for ev in pending[k]:  # this block's copies of step i - 2 have landed
                compute.wait_event(ev)
            prefill(outs[k][b0:b1])
            ev = torch.cuda.Event()
            ev.record(compute)
            pending[k] = pgs[k].push(ev)

        def drain():
            for lst in pending:
                for ev in lst:
                    compute.wait_event(ev)

    for i in range(warmup):
        step(i)
    drain()
    torch.cuda.synchronize()
    barrier(world)
    e0.record(compute)
    for i in range(steps):
        step(i)
    drain()
    e1.record(compute)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    ok = True
    if mode != "nccl":
        barrier(world)  # every rank's copies have landed everywhere
        last = outs[(steps - 1) & 1]
        ref = torch.empty_like(last)
        dist.all_gather_into_tensor(ref, last[b0:b1].contiguous())
        ok = bool(torch.equal(ref, last))
        barrier(world)
        for pg in pgs:
            pg.close()
        barrier(world)
    return ms, ok


# How the multi-GPU steps gather y: "peer" (copy engines, sharding.PeerGather) when every rank can map its
# peers' buffers, else "nccl"; decided once per run, before any timing, by the same trial on every rank.
GATHER = {"mode": "nccl", "why": "", "streams": 1, "parts": 1}


def gathered(dn, x, u, steps, warmup, world):
    """The gathered step: (ms per step, max over ranks; record for the line).  With the copy-engine gather
    available, both gathers are timed on the same step and the step counts the faster one, named in the
    record with both times: the copy engines win while the gather hides behind the next prefill (N = 2,
    or long prefills), NCCL's kernels can win when the gather is several times the prefill (config 2 at
    N = 8, where the copies run slower than NCCL's NVLink algorithms)."""
    if world == 1:
        return time_prefill(dn, x, u, steps, warmup), None
    nms, _ = time_prefill_gathered(dn, x, u, steps, warmup, world, "nccl")
    nms = max_over_ranks(nms, world)
    rec = {"ms_per_step_nccl_gather": nms}
    if GATHER["mode"] != "peer":
        rec.update(mode="nccl", ms_per_step=nms, peer_gather_unavailable=GATHER["why"])
        return nms, rec
    pms, ok = time_prefill_gathered(dn, x, u, steps, warmup, world, "peer")
    pms = max_over_ranks(pms, world)
    rec["ms_per_step_peer_gather"] = pms
    rec["peer_matches_nccl_gather"] = max_over_ranks(0.0 if ok else 1.0, world) == 0
    mode, ms = ("peer", pms) if pms <= nms else ("nccl", nms)
    rec.update(mode=mode, ms_per_step=ms)
    return ms, rec


def peer_gather_works(world):
    """Whether every rank can map its peers' buffers for the copy-engine gather and gets the right bytes
    back: one small trial.  All ranks take the same collective steps whatever fails locally, and agree on
    the answer.  Returns (works, reason)."""
    import torch.distributed as dist
    sh = importlib.import_module("burn-deltanet_b200.sharding")
    rank = dist.get_rank()
    buf = torch.zeros(world, 256, device="cuda", dtype=torch.bfloat16)
    try:
        pg = sh.PeerGather(buf, sh.plan(world, 1, world))  # raises on every rank together
    except RuntimeError as e:
        return False, str(e)[:300]
    err = ""
    try:
        buf[rank].fill_(rank + 1)
        ev = torch.cuda.Event()
        ev.record()
        for e in pg.push(ev):
            torch.cuda.current_stream().wait_event(e)
        torch.cuda.synchronize()
    except Exception as e:  # noqa: BLE001 (agreed on below)
        err = f"rank {rank}: {type(e).__name__}: {e}"
    barrier(world)
    want = torch.arange(1, world + 1, device="cuda", dtype=torch.bfloat16)[:, None].expand(world, 256)
    if not err and not torch.equal(buf, want):
        err = f"rank {rank}: peer copies gave wrong data"
    errs = [None] * world
    dist.all_gather_object(errs, err)
    pg.close()
    barrier(world)
    bad = [e for e in errs if e]
    return not bad, "; ".join(bad)[:300]


def time_prefill_e2e(dn, x, u, steps, warmup):
    """Through the public host-memory entry point (dc_chunk_fwd_host) from
    pinned host buffers: every step copies the inputs in, runs the kernels and
    copies y and the final state back, slice by slice with the transfers
    overlapping the kernels; timed on the device stream the call drains into."""
    host = {k: (None if t is None else t.cpu().pin_memory()) for k, t in x.items()}
    b, s = x["q"].shape[0], x["q"].shape[1]
    y_host = torch.empty((b, s, H, D), dtype=torch.bfloat16).pin_memory()
    s_host = torch.empty(tuple(x["state"].shape), dtype=torch.float32).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in host.values() if t is not None)
    d2h = y_host.numel() * 2 + s_host.numel() * 4
    gated = x["g"] is not None
    scratch = [None]

    def call():
        _, _ = dn.delta_chunk_recalculated_host(host["q"], host["k"], host["v"], host["erase"], host["write"],
                                                host["g"], host["state"], gated, L, 1.0 / math.sqrt(D),
                                                n_householder=u, scratch=scratch[0], y_out=y_host,
                                                state_out=s_host, synchronize=False)

    need = dn.delta_chunk_host_scratch_size(host["q"], host["k"], host["v"], host["erase"], host["write"],
                                            host["g"], host["state"], gated, L, 1.0 / math.sqrt(D), n_householder=u)
    scratch[0] = torch.empty(need, dtype=torch.uint8, device="cuda")
    for _ in range(warmup):
        call()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        call()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps, h2d, d2h


def time_backward(dn, steps, warmup, batch=8, tokens=4096):
    """The backward (dc_chunk_bwd) at config 2's shapes: d_y and d_final_state in, every input's
    gradient out.  Returns (ms per step, algorithmic bytes per launch)."""
    x = make_prefill("deltanet", batch, tokens, 1, "cuda", 7)
    g = torch.Generator(device="cuda").manual_seed(8)
    dy = torch.randn(batch, tokens, H, D, device="cuda", generator=g)
    dsf = torch.randn(tuple(x["state"].shape), device="cuda", generator=g)
    ws = [None]

    def call():
        out = dn.delta_chunk_recalculated_backward(dy, dsf, x["q"], x["k"], x["v"], x["erase"], x["write"], None,
                                                   x["state"], False, L, 1.0 / math.sqrt(D), workspace=ws[0])
        return out

    from importlib import import_module
    abi = import_module("burn-deltanet_b200._abi")
    for _ in range(max(1, warmup)):
        call()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        call()
    e1.record(stream)
    torch.cuda.synchronize()
    assert abi.lib().dc_device_status(0) == 0
    nb = lambda t: t.numel() * t.element_size()
    read = sum(nb(x[n]) for n in ("q", "k", "v", "erase", "write", "state")) + nb(dy) + nb(dsf)
    written = 4 * (3 * x["q"].numel() + x["erase"].numel() + x["write"].numel() + x["state"].numel())
    return e0.elapsed_time(e1) / steps, read + written


def time_out_norm(dn, steps, warmup, batch=8, tokens=4096):
    """The gated output norm (dc_out_norm) on config 2's read-out: y and gate bf16 [B, T, 16, 128] in,
    bf16 out; inputs (268 MB) larger than L2.  Returns (ms per call, algorithmic bytes per call)."""
    g = torch.Generator(device="cuda").manual_seed(11)
    y = torch.randn(batch, tokens, H, D, device="cuda", generator=g).to(torch.bfloat16)
    gate = torch.randn(batch, tokens, H, D, device="cuda", generator=g).to(torch.bfloat16)
    w = torch.rand(D, device="cuda", generator=g) + 0.5
    out = torch.empty_like(y)
    for _ in range(max(3, warmup)):
        dn.out_norm(y, gate, w, out=out)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        dn.out_norm(y, gate, w, out=out)
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps, 3 * y.numel() * 2 + w.numel() * 4


def time_prologue(dn, steps, warmup, batch=8, tokens=4096):
    """The front-end prologue (dc_qkv_prologue) on config 2's projection: x bf16 [B, T, 3 H D] (the
    [q | k | v] channels), short convolution K = 4 with SiLU, q / k L2 norm, q, k, v bf16 out; inputs
    (403 MB) larger than L2.  Returns (ms per call, algorithmic bytes per call)."""
    g = torch.Generator(device="cuda").manual_seed(12)
    c = 3 * H * D
    x = torch.randn(batch, tokens, c, device="cuda", generator=g).to(torch.bfloat16)
    w = torch.randn(c, 4, device="cuda", generator=g) * 0.5
    win = torch.randn(batch, c, 4, device="cuda", generator=g)
    for _ in range(max(3, warmup)):
        out = dn.qkv_prologue(x, H, D, D, w, None, win)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        out = dn.qkv_prologue(x, H, D, D, w, None, win)
    e1.record(stream)
    torch.cuda.synchronize()
    del out
    return e0.elapsed_time(e1) / steps, 2 * x.numel() * 2 + 2 * win.numel() * 4 + w.numel() * 4


def time_gates(dn, steps, warmup):
    """The front-end's gate producers at config 5's sizes (B=16, T=16384, H=16, dk=128): the per-channel
    log-decay over bf16 [B, T, H dk] (the up projection's output) and the doubled erase gate over bf16
    [B, T, H dk], each float32 out.  Returns (ms per pair of calls, algorithmic bytes per pair)."""
    g = torch.Generator(device="cuda").manual_seed(13)
    x = torch.randn(16, 16384, H * D, device="cuda", generator=g).to(torch.bfloat16)
    bias, a = torch.randn(H * D, device="cuda", generator=g), torch.rand(H, device="cuda", generator=g)
    for _ in range(max(3, warmup)):
        dn.channel_log_decay(x, bias, a, D, -5.0), dn.write_gate(x, doubled=True)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        dn.channel_log_decay(x, bias, a, D, -5.0), dn.write_gate(x, doubled=True)
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps, 2 * (x.numel() * 2 + x.numel() * 4)


def time_decode_cfg5(dn, state, steps, warmup, seed):
    """Config 5's decode: `steps` GDN-2 step() tokens (per-channel erase, write and log-decay) from the
    prefill's final state, for this rank's sequences x 16 heads, the state updated in place; the ticks
    replay from one CUDA graph.  Returns (ms per step, bytes per step)."""
    b = state.shape[0]
    g = torch.Generator(device="cuda").manual_seed(seed)
    rn = lambda *s: torch.randn(*s, device="cuda", generator=g)
    bf = torch.bfloat16
    a = torch.rand(1, 1, H, D, device="cuda", generator=g) * math.log(16.0)
    q, k, v = l2n(rn(steps, b, H, D)).to(bf), l2n(rn(steps, b, H, D)).to(bf), rn(steps, b, H, D).to(bf)
    e, w = torch.sigmoid(rn(steps, b, H, D)), torch.sigmoid(rn(steps, b, H, D))
    gg = -torch.exp(a) * torch.nn.functional.softplus(rn(steps, b, H, D))
    y = torch.empty(steps, b, H, D, device="cuda", dtype=bf)
    st = state.clone()

    def tick(t):
        dn.delta_step(q[t], k[t], v[t], e[t], w[t], gg[t], st, 1.0 / math.sqrt(D), y_out=y[t], state_out=st)

    for t in range(max(3, warmup)):
        tick(t)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            for t in range(steps):
                tick(t)
    torch.cuda.current_stream().wait_stream(side)
    st.copy_(state)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    step_bytes = b * H * (2 * D * D * 4 + 3 * D * 2 + 3 * D * 4 + D * 2)
    del graph
    return ms, step_bytes


def time_decode(dn, steps, warmup):
    """Config 3's decode: one fused tick for 256 sequences x 16 heads per step,
    the state updated in place; the K ticks replay from one CUDA graph."""
    x = make_decode("cuda", 1234)
    y = torch.empty(DECODE["batch"], H, D, device="cuda", dtype=torch.bfloat16)
    st = x["state"]

    def tick():
        dn.delta_step(x["q"], x["k"], x["v"], x["erase"], x["erase"], x["g"], st, 1.0 / math.sqrt(D),
                      y_out=y, state_out=st)

    for _ in range(max(3, warmup)):
        tick()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            for _ in range(steps):
                tick()
    torch.cuda.current_stream().wait_stream(side)
    graph.replay()  # warm
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    heads = DECODE["batch"] * H
    step_bytes = heads * (2 * D * D * 4 + 3 * D * 2 + 2 * 4 + D * 2)
    del graph
    return ms, step_bytes


def cpu_model():
    """The host CPU's model name, for the CPU baseline's record."""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def hbm_roofline(nbytes, ms, hbm_peak, peak_kind, traffic=None):
    achieved = nbytes / (ms / 1e3) / 1e9
    return {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
            "peak_kind": peak_kind, "traffic": traffic, "algorithmic_bytes_per_launch": nbytes}


def measure_cfg4(dn, args, rank, world, hbm_peak, peak_kind):
    """Config 4 (DeltaProduct, u = 2 and 3, B=4 T=8192 per GPU, weak scaling): one dc_chunk_fwd per step
    with the micro-steps folded in-kernel; at N > 1 the value counts the all-gather of y, as in the headline;
    `kernel_ms` is the prefill alone."""
    out = {}
    for u in (2, 3):
        batch, tokens = 4, 8192
        x = make_prefill("deltaproduct", batch, tokens, u, "cuda", 4000 + 10 * u + rank)
        k_ms = max_over_ranks(time_prefill(dn, x, u, args.steps, args.warmup), world)
        ms, grec = gathered(dn, x, u, args.steps, args.warmup, world) if world > 1 else (k_ms, None)
        nbytes = algorithmic_bytes(x, batch * tokens)
        flops = 2 * (5 * L * D + 3 * D * D) * batch * tokens * u * H
        out[f"u{u}"] = {
            "metric": f"prefill tok/s (config 4: DeltaProduct u={u}, bf16 in, fp32 state, B={batch} per GPU, "
                      f"T={tokens}, H={H}, dk=dv={D}; real tokens, not micro-steps)",
            "value": batch * tokens * world / (ms / 1e3), "unit": "tok/s", "ms_per_step": ms,
            "kernel_ms": k_ms, "kernel_value": batch * tokens * world / (k_ms / 1e3), "steps": args.steps,
            "scaling": "weak", "roofline": dict(hbm_roofline(nbytes, k_ms, hbm_peak, peak_kind),
                                                tensor_tflops=flops / (k_ms / 1e3) / 1e12),
            "gpu_launches": args.steps}
        if grec is not None:
            out[f"u{u}"]["gather"] = grec
        del x
        torch.cuda.empty_cache()
    return out


def measure_cfg5(dn, args, rank, world, hbm_peak, peak_kind):
    """Config 5 as the north star runs it: one batch of 16 GDN-2 sequences (T=16384) sharded batch-major over
    the N GPUs (strong scaling), the prefill of each rank's sequences (two launches: prep + scan), the
    all-gather of y into every rank's [16, T, H, dv] output inside the timed step, then 512 GDN-2 step() tokens from each rank's own final state.  At N > 1 every
    rank also runs the whole unsharded batch and checks the gathered y and final state against it bit for
    bit."""
    B5, T5 = 16, 16384
    if B5 % world:
        return {"unavailable": f"16 sequences do not split over {world} GPUs"}
    per = B5 // world
    full = make_prefill("gdn2", B5, T5, 1, "cuda", 5000)  # the same global batch on every rank
    x = {k: (None if t is None else t[rank * per:(rank + 1) * per].contiguous()) for k, t in full.items()}
    steps = max(3, min(args.steps, 10))
    k_ms = max_over_ranks(time_prefill(dn, x, 1, steps, args.warmup), world)
    ms, grec = gathered(dn, x, 1, steps, args.warmup, world) if world > 1 else (k_ms, None)
    nbytes = algorithmic_bytes(x, per * T5)
    flops = 2 * (5 * L * D + 3 * D * D) * per * T5 * H
    traffic = profiled_traffic("gdn2")
    rec = {
        "metric": f"prefill tok/s (config 5: GDN-2, per-channel gates, bf16 in, fp32 state, B={B5} over {world} GPU, "
                  f"T={T5}, H={H}, dk=dv={D}; y all-gathered to every rank inside the step)",
        "value": B5 * T5 / (ms / 1e3), "unit": "tok/s", "ms_per_step": ms, "kernel_ms": k_ms,
        "kernel_value": B5 * T5 / (k_ms / 1e3), "steps": steps, "scaling": "strong",
        "roofline": dict(hbm_roofline(nbytes, k_ms, hbm_peak, peak_kind,
                                      None if traffic is None else traffic * per / B5),
                         tensor_tflops=flops / (k_ms / 1e3) / 1e12, per_gpu=True),
        "gpu_launches": 2 * steps,
    }
    if grec is not None:
        rec["gather"] = grec
    # Sharded == unsharded: this rank's shard, gathered, against the whole batch run on this GPU.
    y_loc, s_loc = dn.delta_chunk_recalculated(x["q"], x["k"], x["v"], x["erase"], x["write"], x["g"], x["state"],
                                               True, L, 1.0 / math.sqrt(D))
    if world > 1:
        sh = importlib.import_module("burn-deltanet_b200.sharding")
        shards = sh.plan(B5, H, world)
        y_all, s_all = sh.gather(y_loc, shards), sh.gather(s_loc, shards, head_axis=1)
        y_full, s_full = dn.delta_chunk_recalculated(full["q"], full["k"], full["v"], full["erase"], full["write"],
                                                     full["g"], full["state"], True, L, 1.0 / math.sqrt(D))
        ok = float(torch.equal(y_all, y_full) and torch.equal(s_all, s_full))
        worst = max_over_ranks(-ok, world)  # -1 when every rank matched
        rec["sharded_equals_unsharded"] = worst < 0
        del y_all, s_all, y_full, s_full
    del full, y_loc
    torch.cuda.empty_cache()
    dec_ms, dec_bytes = time_decode_cfg5(dn, s_loc, CFG5_DECODE_STEPS, args.warmup, 2000 + rank)
    dec_ms = max_over_ranks(dec_ms, world)
    rec["decode"] = {
        "metric": f"decode tok/s (config 5: GDN-2 step, {B5} sequences x {H} heads over {world} GPU, "
                  f"{CFG5_DECODE_STEPS} steps from the prefill's final state, fp32 state)",
        "value": B5 / (dec_ms / 1e3), "unit": "tok/s", "ms_per_step": dec_ms, "steps": CFG5_DECODE_STEPS,
        "roofline": hbm_roofline(dec_bytes, dec_ms, hbm_peak, peak_kind), "gpu_launches": CFG5_DECODE_STEPS}
    del s_loc
    ms_e2e, h2d, d2h = time_prefill_e2e(dn, x, 1, 1, 1)
    ms_e2e = max_over_ranks(ms_e2e, world)
    rec["e2e"] = {"value": B5 * T5 / (ms_e2e / 1e3), "unit": "tok/s", "h2d_bytes_per_step": h2d,
                  "d2h_bytes_per_step": d2h, "ms_per_step": ms_e2e,
                  "note": "each rank's shard from and back to its own host memory (no gather)"}
    del x
    torch.cuda.empty_cache()
    return rec


def run_ours(args):
    rank, world, local = setup(args.gpus)
    dn = importlib.import_module("burn-deltanet_b200")
    hbm_peak, tc_peak, peak_kind = measured_peaks()
    if world > 1:
        works, why = peer_gather_works(world)
        if args.gather == "peer" and works:
            GATHER["mode"], GATHER["why"] = "peer", ""
        else:
            GATHER["mode"], GATHER["why"] = "nccl", (why if args.gather == "peer" else "--gather nccl")
    cfg, batch, tokens, u, kind = WORKLOADS[args.workload]
    strong = args.workload in STRONG and not args.batch
    if strong:
        if batch % world:
            raise SystemExit(f"{args.workload}: {batch} sequences do not split over {world} GPUs")
        batch //= world  # this rank's share of the one batch
    batch = args.batch or batch
    x = make_prefill(kind, batch, tokens, u, "cuda", 1000 + rank)
    # One dc_chunk_fwd per step: one kernel, or two (prep + scan) for per-channel gates.
    launches = args.steps * (2 if kind == "gdn2" else 1)
    clocks = ClockSampler(local)
    barrier(world)
    torch.cuda.synchronize()
    if args.only == "decode":
        dec_ms, dec_bytes = time_decode(dn, DECODE_STEPS, args.warmup)
        if rank == 0:
            print(json.dumps({"decode_ms_per_step": dec_ms, "decode_gbs": dec_bytes / (dec_ms / 1e3) / 1e9}))
        return
    with clocks:
        k_ms = time_prefill(dn, x, u, args.steps, args.warmup)
    barrier(world)
    if args.only == "prefill":
        if rank == 0:
            print(json.dumps({"prefill_ms_per_step": k_ms, "tok_s": batch * tokens * world / (k_ms / 1e3)}))
        return
    if args.only == "gates":
        gt_ms, gt_bytes = time_gates(dn, 10, 3)
        if rank == 0:
            print(json.dumps({"gates_ms": gt_ms, "gates_gbs": gt_bytes / (gt_ms / 1e3) / 1e9}))
        return
    if args.only == "prologue":
        pr_ms, pr_bytes = time_prologue(dn, 20, 3, batch=args.batch or 8)
        if rank == 0:
            print(json.dumps({"prologue_ms": pr_ms, "prologue_gbs": pr_bytes / (pr_ms / 1e3) / 1e9}))
        return
    if args.only == "f32":
        f_ms, fs_ms, f_bytes, f_choice = time_prefill_f32(dn, 5, 3, batch=args.batch or 8)
        if rank == 0:
            print(json.dumps({"f32_ms": f_ms, "f32_cuda_core_ms": fs_ms, "choice": f_choice,
                              "f32_gbs": f_bytes / (f_ms / 1e3) / 1e9}))
        return
    if args.only == "out_norm":
        on_ms, on_bytes = time_out_norm(dn, 20, 3, batch=args.batch or 8)
        if rank == 0:
            print(json.dumps({"out_norm_ms": on_ms, "out_norm_gbs": on_bytes / (on_ms / 1e3) / 1e9}))
        return
    if args.only == "backward":
        bw_ms, bw_bytes = time_backward(dn, 5, 2, batch=args.batch or 8)
        if rank == 0:
            print(json.dumps({"backward_ms_per_step": bw_ms, "backward_gbs": bw_bytes / (bw_ms / 1e3) / 1e9}))
        return
    if args.only == "cfg5":
        rec = measure_cfg5(dn, args, rank, world, hbm_peak, peak_kind)
        if rank == 0:
            print(json.dumps(rec))
        return
    if args.only == "cfg4":
        rec = measure_cfg4(dn, args, rank, world, hbm_peak, peak_kind)
        if rank == 0:
            print(json.dumps(rec))
        return
    k_ms = max_over_ranks(k_ms, world)
    tok_per_rank = batch * tokens
    # The step at N > 1 includes the all-gather of y to every rank.
    ms, grec = gathered(dn, x, u, args.steps, args.warmup, world) if world > 1 else (k_ms, None)
    value = tok_per_rank * world / (ms / 1e3)
    nbytes = algorithmic_bytes(x, batch * tokens)
    ms_e2e, h2d, d2h = time_prefill_e2e(dn, x, u, max(1, min(args.steps, 5)), 1)
    ms_e2e = max_over_ranks(ms_e2e, world)
    pn_ms, pn_two_ms, pn_fused = time_prefill_out_norm(dn, x, u, args.steps, args.warmup)
    pn_ms, pn_two_ms = max_over_ranks(pn_ms, world), max_over_ranks(pn_two_ms, world)
    flops = 2 * (5 * L * D + 3 * D * D) * batch * tokens * u * H
    del x
    torch.cuda.empty_cache()
    dec_ms, dec_bytes = time_decode(dn, DECODE_STEPS, args.warmup)
    dec_ms = max_over_ranks(dec_ms, world)
    bw_ms, bw_bytes = time_backward(dn, 5, 2)
    bw_ms = max_over_ranks(bw_ms, world)
    on_ms, on_bytes = time_out_norm(dn, 20, 3)
    on_ms = max_over_ranks(on_ms, world)
    pr_ms, pr_bytes = time_prologue(dn, 20, 3)
    pr_ms = max_over_ranks(pr_ms, world)
    gt_ms, gt_bytes = time_gates(dn, 10, 3)
    gt_ms = max_over_ranks(gt_ms, world)
    torch.cuda.empty_cache()
    f32_ms, f32_simt_ms, f32_bytes, f32_choice = time_prefill_f32(dn, 5, 3)
    f32_ms, f32_simt_ms = max_over_ranks(f32_ms, world), max_over_ranks(f32_simt_ms, world)
    torch.cuda.empty_cache()
    cfg4 = measure_cfg4(dn, args, rank, world, hbm_peak, peak_kind) if args.workload == "deltanet" else None
    cfg5 = measure_cfg5(dn, args, rank, world, hbm_peak, peak_kind) if args.workload == "deltanet" else None
    dec_tok = DECODE["batch"] * world / (dec_ms / 1e3)
    traffic = profiled_traffic(args.workload)
    line = {
        "metric": f"prefill tok/s ({kind}, bf16 in, fp32 state, H={H} dk=dv={D}, chunk {L})",
        "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong" if strong else "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded, BASELINE config recipes)",
        "config": arm_config(cfg, kind, batch, tokens, u, world, strong),
        "roofline": dict(hbm_roofline(nbytes, k_ms, hbm_peak, peak_kind, traffic),
                         tensor_tflops=flops / (k_ms / 1e3) / 1e12, tensor_peak=tc_peak),
        "kernel_only": {"value": tok_per_rank * world / (k_ms / 1e3), "unit": "tok/s", "ms_per_step": k_ms,
                        "note": "the prefill alone, without the all-gather of y (identical to value at N=1)"},
        "e2e": {"value": tok_per_rank * world / (ms_e2e / 1e3), "unit": "tok/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": ms_e2e},
        "gpu_launches": launches,
        "decode": {"metric": f"decode tok/s (config 3: GDN step, 256 sequences x 16 heads, fp32 state, "
                             f"{DECODE_STEPS} consecutive ticks)",
                   "value": dec_tok, "unit": "tok/s", "ms_per_step": dec_ms, "steps": DECODE_STEPS,
                   "roofline": hbm_roofline(dec_bytes, dec_ms, hbm_peak, peak_kind),
                   "gpu_launches": DECODE_STEPS},
        "backward": {"metric": "backward tok/s (dc_chunk_bwd at config 2's shapes: every input's gradient; "
                               "chunked, fp32-accurate tf32 products on the tensor cores)",
                     "value": 8 * 4096 * world / (bw_ms / 1e3), "unit": "tok/s", "ms_per_step": bw_ms, "steps": 5,
                     "roofline": {"bound": "tensor", "achieved": BWD_FLOP * 8 * 4096 * H / (bw_ms / 1e3) / 1e12,
                                  "peak": tc_peak, "unit": "TFLOP/s",
                                  "frac": BWD_FLOP * 8 * 4096 * H / (bw_ms / 1e3) / 1e12 / tc_peak,
                                  "flop_per_token_head": BWD_FLOP,
                                  "hbm_gbs_of_inputs_and_gradients": bw_bytes / (bw_ms / 1e3) / 1e9},
                     "gpu_launches": 3 * 5},
        "prefill_out_norm": {"metric": "prefill + plain out-norm tok/s (the workload's prefill with the per-head "
                                       "RMSNorm of its read-out fused into the kernel's epilogue, bf16 out)",
                             "value": tok_per_rank * world / (pn_ms / 1e3), "unit": "tok/s",
                             "ms_per_step": pn_ms, "ms_per_step_two_calls": pn_two_ms,
                             "ms_per_step_prefill_alone": k_ms, "steps": args.steps, "fused": pn_fused,
                             "roofline": hbm_roofline(nbytes, pn_ms, hbm_peak, peak_kind),
                             "gpu_launches": launches + (0 if pn_fused else args.steps)},
        "prefill_f32": {"metric": "prefill tok/s at the reference's precision (config 2's shapes with float32 "
                                  "q, k, v and y: the fp32-accurate chunked path, three-part tf32 products)",
                        "value": 8 * 4096 * world / (f32_ms / 1e3), "unit": "tok/s", "ms_per_step": f32_ms,
                        "steps": 5, "kernel_choice": f32_choice,
                        "cuda_core_kernel": {"value": 8 * 4096 * world / (f32_simt_ms / 1e3), "unit": "tok/s",
                                             "ms_per_step": f32_simt_ms, "steps": 1},
                        "roofline": hbm_roofline(f32_bytes, f32_ms, hbm_peak, peak_kind),
                        "gpu_launches": 2 * 5},
        "out_norm": {"metric": "out-norm tok/s (gated per-head RMSNorm after the read-out, config 2's output: "
                               "bf16 y and gate in, bf16 out)",
                     "value": 8 * 4096 * world / (on_ms / 1e3), "unit": "tok/s", "ms_per_step": on_ms, "steps": 20,
                     "roofline": hbm_roofline(on_bytes, on_ms, hbm_peak, peak_kind),
                     "gpu_launches": 20},
        "prologue": {"metric": "prologue tok/s (front-end after the input projection, config 2: short "
                               "convolution K=4 + SiLU + q/k L2 norm, bf16 in and out)",
                     "value": 8 * 4096 * world / (pr_ms / 1e3), "unit": "tok/s", "ms_per_step": pr_ms, "steps": 20,
                     "roofline": hbm_roofline(pr_bytes, pr_ms, hbm_peak, peak_kind),
                     "gpu_launches": 20},
        "gates": {"metric": "gate producers tok/s (config 5: per-channel log-decay and doubled erase gate, bf16 "
                            "[16, 16384, 16 x 128] in, float32 out)",
                  "value": 16 * 16384 * world / (gt_ms / 1e3), "unit": "tok/s", "ms_per_step": gt_ms, "steps": 10,
                  "roofline": hbm_roofline(gt_bytes, gt_ms, hbm_peak, peak_kind),
                  "gpu_launches": 20},
        "clocks": clocks.summary(),
    }
    if cfg4 is not None:
        line["cfg4"] = cfg4
    if cfg5 is not None:
        line["cfg5"] = cfg5
    if world > 1:
        out_bytes = world * tok_per_rank * H * D * 2
        line["allgather"] = dict(grec, **{
            "collective": ("the faster of two gathers of y (bf16), both timed: 'peer', each rank's block pushed "
                           "to every peer by the NVLink copy engines (CUDA IPC), two global buffers "
                           "alternating so the copies of step i run beside the prefill of step i+1; 'nccl', "
                           "all_gather_into_tensor after each step's prefill on the same stream"),
            "bytes_per_rank_out": out_bytes,
            "nvlink_bound_ms": (world - 1) * tok_per_rank * H * D * 2 / 770e9 * 1e3,
            "ms_per_step_with_gather": ms, "ms_per_step_kernel_only": k_ms})
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.workload)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def profiled_traffic(workload):
    """DRAM bytes per launch of the prefill kernel from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", f"chunk_fwd_{workload}.txt")
    if not os.path.exists(path):
        return None
    for line in open(path):
        if line.startswith("traffic_bytes_per_launch:"):
            return float(line.split(":")[1])
    return None


def arm_config(cfg, kind, batch, tokens, u, world, strong=False):
    """The workload both arms report (the reference arm times a bounded sample of it, described in its
    cpu_baseline).  `batch` is per GPU."""
    per = f"B={batch * world} over {world} GPU" if strong else f"B={batch} per GPU"
    return {"workload": f"config {cfg}: {kind} prefill {per}, T={tokens}, H={H}, dk=dv={D}"
                        + (f", u={u}" if u > 1 else ""),
            "global_batch": batch * world, "seq_len": tokens, "parallelism": f"batch x head over {world} GPU",
            "l2": "inputs larger than L2 (no flush needed)"}


def run_reference(args):
    """The reference's algorithm on the host cores: this build cannot compile
    the Rust reference (no cargo, Burn deps not vendored), so the arm times its
    C restatement (oracle/), rank 0 only, one bounded sample per step."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle

    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from _inputs import config_inputs

    cfg, batch, tokens, u, kind = WORKLOADS[args.workload]
    threads = os.cpu_count() or 1
    # Each step is the workload's own batch (config 2: B=8, T=4096, about 2 s on 16 host threads).  The
    # heavier workloads (config 4's micro-steps, config 5's per-channel gates over B=16 T=16384) would take
    # minutes per step, so a step there is a bounded sample of them: the same T up to 4096 tokens and the
    # number of sequences that keeps a step near config 2's work.
    full = kind == "deltanet"
    sample_tokens = tokens if full else min(tokens, 4096)
    sample_batch = batch if full else max(1, min(batch, 8 // u // (4 if kind == "gdn2" else 1)))
    rng = np.random.default_rng(0)
    raw = config_inputs({"deltanet": 2, "deltaproduct": 4, "gdn2": 5}[kind], rng, sample_batch, sample_tokens,
                        H, D, D, u=u)
    raw = {k: (None if v is None else v.astype(np.float32)) for k, v in raw.items()}

    def step():
        oracle.householder("chunk", raw["q"], raw["k"], raw["v"], raw["erase"], raw["write"], raw["g"],
                           raw["state"], u, chunk_len=L, dtype=np.float32, threads=threads)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    value = sample_batch * sample_tokens / dt
    line = {
        "impl": "reference", "metric": f"prefill tok/s ({kind}, bf16 in, fp32 state, H={H} dk=dv={D}, chunk {L})",
        "value": value, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "strong" if args.workload in STRONG else "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded, BASELINE config recipes)",
        "config": arm_config(cfg, kind, batch // args.gpus if args.workload in STRONG else batch, tokens, u,
                             args.gpus, args.workload in STRONG),
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": min(threads, sample_batch * H), "kind": "port",
                         "cpu_model": cpu_model(), "host_threads": threads,
                         "sample": f"oracle chunk path fp32 (the reference algorithm restated in C, OpenMP over "
                                   f"(batch, head)), per step "
                                   + ("the workload's whole batch" if full else "a bounded sample of the workload")
                                   + f": B={sample_batch} T={sample_tokens} H={H}" + (f" u={u}" if u > 1 else "")},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="deltanet")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--gather", choices=["peer", "nccl"], default="peer",
                    help="how multi-GPU steps gather y: NVLink copy engines (default) or NCCL")
    ap.add_argument("--only", choices=["prefill", "decode", "backward", "out_norm", "prologue", "gates", "f32", "cfg4",
                                       "cfg5"], default=None,
                    help="time one kernel alone and print a short line (for profiling runs)")
    ap.add_argument("--batch", type=int, default=None,
                    help="sequences per GPU instead of the workload's own (for small profiling captures)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
