#!/usr/bin/env python
"""Embedding rows/s per round (pull + push + LazyAdam) on B200.

One *round* (= one bench step) over the configured synthetic batch is: one
lookup (gather + sum/mean pooling of every feature, occurrence list and its
coalescing sort) and one push (gradient prescan, coalesced segment-sum fused
with the sparse LazyAdam update, finalize).  rows = id occurrences processed per
round (each is pulled once and contributes one gradient).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--config 1|2|4]

value  : rows/s with inputs resident in HBM, device-timed with CUDA events on
         the launching stream, L2 flushed (256 MiB write) before every timed
         round, summed over the K rounds; max over ranks when N > 1.
e2e    : the same rounds through the C ABI with HOST (pinned) buffers: keys and
         offsets copied in, pooled outputs copied out, gradients copied in and
         the push status read back, all inside the timed region.
roofline: the dominant kernel (the longest single-launch phase with compulsory
         HBM bytes: gather, row updates or prescan) -- its algorithmic bytes per
         launch (byte_model) over its CUDA-event duration, timed by the
         library's phase events in a separate profiled pass of the same rounds,
         against the measured HBM copy bandwidth in MEASURED_PEAKS.json.
cpu_baseline / --impl reference: the UNMODIFIED reference CPU parameter server
         (oracle/_ref, compiled from its own sources) with one shard per host
         core behind its DistributedClient, timed wall-clock on the same batch.
"""
from __future__ import annotations

import argparse
import gc
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "tests"))
METRIC = "embedding rows/s per round (pull+push+Adam)"
UNIT = "rows/s"
FALLBACK_HBM_GBS = 6650.0


def _import_package():
    import importlib.util
    pkg = os.path.join(ROOT, "distributed-recommendation-model-training-system_b200")

    def load(name, path, package=False):
        if name in sys.modules:
            return sys.modules[name]
        kw = {"submodule_search_locations": [pkg]} if package else {}
        spec = importlib.util.spec_from_file_location(name, path, **kw)
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
        return mod

    workloads = load("eps_b200_workloads", os.path.join(pkg, "workloads.py"))
    if os.environ.get("EPS_B200_NO_PACKAGE"):
        return workloads, None
    return workloads, load("eps_b200", os.path.join(pkg, "__init__.py"), package=True)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", type=int, default=2, choices=[1, 2, 4])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--rows", type=int, default=0,
                    help="override the table rows of config 2 (smaller profiling captures)")
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def workload_for(wl, config, rank, rows=0):
    if config == 1:
        return wl.config1(seed=1 + 1000 * rank)
    if config == 4:
        return wl.config4(seed=4 + 1000 * rank)
    if rows:
        return wl.config2(seed=2 + 1000 * rank, rows=rows)
    return wl.config2(seed=2 + 1000 * rank)


def byte_model(w):
    """Compulsory bytes (each byte that must cross HBM once; sort scratch excluded)."""
    N = w.occurrences
    rows_out = w.bags                                    # output / gradient rows
    pooled_offsets = sum(len(f.offsets) for f in w.features if f.pooling != 2)
    dims = {t.id: t.dimension for t in w.tables}
    U_by_dim = {}
    for t in w.tables:
        ks = [f.keys for f in w.features if f.table == t.id]
        if ks:
            U_by_dim[t.id] = len(np.unique(np.concatenate(ks)))
    U = sum(U_by_dim.values())
    row_bytes_u = sum(4 * dims[t] * u for t, u in U_by_dim.items())        # 4D per unique row
    out_bytes = sum(4 * dims[f.table] * f.output_rows for f in w.features)  # 4D per output row
    pull = 8 * N + 8 * pooled_offsets + row_bytes_u + out_bytes
    push = out_bytes + 8 * N + 8 * pooled_offsets + 6 * row_bytes_u + 16 * U
    # per kernel: the gather moves the pull's bytes; the row-update kernel moves
    # the read + write of [w|m|v] (12D each way) and the u64 counter of every
    # row it updates (all rows except those with > 64 occurrences, which the
    # long-row kernel updates); the prescan reads every gradient value once
    long_rows = {}
    for t in w.tables:
        ks = [f.keys for f in w.features if f.table == t.id]
        if ks:
            _, c = np.unique(np.concatenate(ks), return_counts=True)
            long_rows[t.id] = int((c > 64).sum())
    rmw = {t: 24 * dims[t] + 16 for t in U_by_dim}
    apply_kernel = sum(rmw[t] * (U_by_dim[t] - long_rows[t]) for t in U_by_dim)
    long_kernel = sum(rmw[t] * long_rows[t] for t in U_by_dim)
    return {"N": N, "U": U, "B": rows_out, "pull": pull, "push": push,
            "lookup": pull, "apply": apply_kernel, "long": long_kernel, "prescan": out_bytes,
            "sort": 0, "emit": 0, "pieces": 0, "finalize": 0,
            "U_long": sum(long_rows.values())}


def dominant_kernel(prof, bm):
    """The roofline's kernel: the phase with the longest time per call among
    those with compulsory HBM bytes in the byte model (gather, row updates, long
    rows, prescan)."""
    cands = [p for p in prof if bm.get(p) and prof[p]["ms"]]
    return max(cands, key=lambda p: prof[p]["ms"] / max(1, prof[p]["calls"]))


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def load_traffic():
    """ncu DRAM bytes per launch of each phase, from the committed summary."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f)
    except Exception:
        return {}


class Clocks:
    """nvidia-smi samples during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, local_rank):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        self.index = vis.split(",")[local_rank] if vis else str(local_rank)
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.out = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.index, f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=self.out, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def wait_first(self, timeout=15.0):
        """Blocks until nvidia-smi has written its first sample, so that its
        start-up (process spawn, driver library initialisation, first query),
        which can hold up this process's own driver calls for tens of
        milliseconds, is over before any timed round."""
        if not self.proc:
            return
        t0 = time.time()
        while time.time() - t0 < timeout and self.proc.poll() is None:
            self.out.flush()
            if os.path.getsize(self.path) > 0:
                return
            time.sleep(0.02)

    def mark(self):
        """Samples before this call (sampler start-up, allocator priming) are
        left out of the summary."""
        self.skip = 0
        if self.proc:
            self.out.flush()
            with open(self.path) as f:
                self.skip = sum(1 for _ in f)

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.out.close()
        rows = []
        for i, line in enumerate(open(self.path)):
            parts = [p.strip() for p in line.split(",")]
            if i >= getattr(self, "skip", 0) and len(parts) >= 8:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[4:8]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows),
                "window": "warm-up start to the end of a 0.5 s untimed soak of the same rounds"}


# --------------------------------------------------------------- reference arm
def reference_rounds(w, steps, warmup, threads):
    """Times the reference's CPU path (oracle/_ref) on the batch; returns seconds per round."""
    from oracle_lib import Feature, Reference, TableDef, reference_available
    if not reference_available():
        return None
    tables = [TableDef(id=t.id, dimension=t.dimension, learning_rate=1e-3, init_min=-0.05,
                       init_max=0.05, init_seed=42, rows=t.rows) for t in w.tables]
    feats = [Feature(f.table, f.feature, f.pooling, f.keys, f.offsets) for f in w.features]
    ref = Reference(tables, shards=threads, state_bytes=64 << 30)
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        batch, _ = ref.lookup(feats)
        ref.push(batch, feats, w.gradients)
        dt = time.perf_counter() - t0
        if i >= warmup:
            times.append(dt)
    ref.close()
    return times


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def run_reference(args):
    rank, local_rank, world = dist_env()
    if rank != 0:
        return
    wl, _ = _import_package()
    w = workload_for(wl, args.config, 0, args.rows)
    if world > 1:
        # the same job as the GPU arm at this N: every rank's batch, served as one
        # combined request (features rank-major, ids r * F + f) by the CPU shards
        parts = [workload_for(wl, args.config, r, args.rows) for r in range(world)]
        F = len(w.features)
        feats = [type(f)(f.table, r * F + f.feature, f.pooling, f.keys, f.offsets)
                 for r, p in enumerate(parts) for f in p.features]
        grads = [g for p in parts for g in p.gradients]
        w = type(w)(f"{w.name}, {world} batches (one per GPU of the sharded run)", w.tables,
                    feats, grads, w.seed, dict(w.meta))
    threads = host_threads()
    times = reference_rounds(w, args.steps, args.warmup, threads)
    if times is None:
        print(json.dumps({"impl": "reference", "unavailable":
                          "reference CPU build oracle/_ref/libeps_ref.so is missing"}))
        return
    total = sum(times)
    value = w.occurrences * len(times) / total
    sample = (f"{len(times)} full rounds of {w.name} ({w.occurrences} occurrences each) after "
              f"{args.warmup} warm-up rounds, {threads} shards/threads")
    print(json.dumps({
        "metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
        "steps": len(times), "warmup": args.warmup, "ms_per_step": 1e3 * total / len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": w.name, "parallelism": f"cpu x{threads}"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))


# ------------------------------------------------------------------- B200 arm
def run_b200(args):
    import torch
    rank, local_rank, world = dist_env()
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device(f"cuda:{local_rank}"))
    wl, eps = _import_package()
    w = workload_for(wl, args.config, rank, args.rows)
    bm = byte_model(w)
    dev = torch.device(f"cuda:{local_rank}")
    # one shard per rank: keys k with k % world == rank (the table's rows are split)
    store = eps.ParameterStore(device=local_rank, shard_id=rank, shard_count=world,
                               state_bytes=150 << 30)
    for t in w.tables:
        store.create_table(eps.TableDefinition(id=t.id, dimension=t.dimension, key_space=t.rows,
                                               learning_rate=1e-3, shard_count=world))
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)          # flushes and events run on the store's stream

    # ---- device-resident inputs
    feats = [eps.FeatureInput(f.table, f.feature, f.pooling,
                              torch.from_numpy(f.keys.astype(np.int64)).to(dev),
                              torch.from_numpy(f.offsets.astype(np.int64)).to(dev))
             for f in w.features]
    dims = {t.id: t.dimension for t in w.tables}
    outs = [torch.empty((f.output_rows, dims[f.table]), dtype=torch.float32, device=dev)
            for f in w.features]
    grads = [torch.from_numpy(g).to(dev) for g in w.gradients]
    flush = torch.empty(64 << 20, dtype=torch.float32, device=dev)   # 256 MiB > 126 MB L2
    if dist:
        # every rank's batch is routed to the owners over NCCL all-to-all
        import importlib
        D = importlib.import_module("eps_b200.distributed")
        comm = D.NcclComm.from_process_group(local_rank)    # NCCL group calls on our streams
        comm_in = D.NcclComm.from_process_group(local_rank)  # the prepare phase's exchanges
        client = D.NativeClient(store, comm, comm_in)        # the round's host side in C++
        # the next batch's partition + key exchange (prepare) is issued before this
        # round's push, on a high-priority input stream, as a training loop whose
        # loader holds the next batch would; every timed step contains exactly one
        # prepare, one lookup and one push
        ids_stream = torch.cuda.Stream(device=dev, priority=-1)
        nxt = [None]

        def one_round():
            if nxt[0] is None:
                nxt[0] = client.prepare(feats, input_stream=ids_stream)
            handle, _ = client.lookup_prepared(nxt[0], outputs=outs)
            nxt[0] = client.prepare(feats, input_stream=ids_stream)
            client.push(handle, grads)
    else:
        lookup = store.prepare_lookup(feats, outs)
        push = store.prepare_push(grads)

        def one_round():
            ticket = lookup(stream)
            push(ticket, stream, wait=False)

    # the clock sampler first: its start-up must be over before timed work
    clocks = Clocks(local_rank)
    clocks.start()
    clocks.wait_first()
    # allocator priming (untimed): more rounds in flight than the library's
    # limit of enqueued pushes (16), so that the stream-ordered memory pool
    # reaches its steady size before the warm-up and never grows (maps new
    # memory, a host stall of milliseconds) inside the timed rounds
    for _ in range(20):
        one_round()
    store.synchronize()
    clocks.mark()
    # no Python collector pauses inside the warm-up and the timed rounds (a pause
    # longer than the rounds queued ahead of the host would leave the device
    # idle); collecting here, before the warm-up, keeps the device busy right up
    # to the first timed round
    gc.collect()
    gc.disable()
    for _ in range(args.warmup):
        flush.zero_()
        one_round()
    store.synchronize()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    launches0 = store.stats()["kernel_launches"]
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
    torch.cuda.synchronize()
    # after the synchronize the device queue is empty: three extra L2 flushes
    # (untimed, ~40 us each) give the host the head start it has in steady
    # state, so that round 0 does not wait for its own enqueue
    for _ in range(3):
        flush.zero_()
    host_s = []
    for a, b in events:
        flush.zero_()
        a.record(stream)
        h0 = time.perf_counter()
        one_round()
        host_s.append(time.perf_counter() - h0)
        b.record(stream)
    torch.cuda.synchronize()
    store.synchronize()
    gc.enable()
    launches = store.stats()["kernel_launches"] - launches0
    # per-phase device time: the same rounds again with the library's phase events
    # (kept out of the timed rounds above, whose stream they would otherwise join)
    store.profile(1)
    for _ in range(args.steps):
        flush.zero_()
        one_round()
    torch.cuda.synchronize()
    store.synchronize()
    prof = store.profile(0)
    # the timed rounds last milliseconds, less than one nvidia-smi sample period:
    # keep the same load running (untimed) for 0.5 s so the clock record covers it
    # (a fixed round count, the same on every rank, so that collectives match)
    step_ms = sum(a.elapsed_time(b) for a, b in events) / args.steps
    if dist:
        t = torch.tensor([step_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        step_ms = float(t.item())
    for i in range(max(8, int(500.0 / max(step_ms, 1e-3)))):
        one_round()
        if i % 8 == 7:
            store.synchronize()
    store.synchronize()
    clk = clocks.stop()
    if dist:
        dist.barrier()
    total_ms = sum(a.elapsed_time(b) for a, b in events)
    job_N, job_U = bm["N"], bm["U"]          # occurrences / unique rows of the whole job
    if dist:
        t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
        t = torch.tensor([bm["N"], bm["U"]], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        job_N, job_U = int(t[0].item()), int(t[1].item())
    value = job_N * args.steps / (total_ms / 1e3)

    # ---- roofline of the dominant phase
    peak, peak_kind = load_peaks()
    dom = dominant_kernel(prof, bm)
    calls = max(1, prof[dom]["calls"])
    per_call_ms = prof[dom]["ms"] / calls
    alg = bm[dom]
    achieved = alg / (per_call_ms / 1e3) / 1e9 if alg else 0.0
    traffic = load_traffic().get(f"cfg{args.config}", {}).get(dom)
    phases = {p: {"ms_per_round": prof[p]["ms"] / max(1, prof[p]["calls"]),
                  "launches_per_round": prof[p]["launches"] / max(1, prof[p]["calls"]),
                  "alg_GBps": (bm[p] / (prof[p]["ms"] / max(1, prof[p]["calls"]) / 1e3) / 1e9)
                  if bm.get(p) and prof[p]["ms"] else None} for p in prof}

    # ---- e2e through the C ABI with pinned host buffers
    def pinned(a):
        t = torch.empty(a.shape, dtype=torch.from_numpy(a[:0]).dtype, pin_memory=True)
        t.numpy()[...] = a
        return t.numpy()

    hfeats = [eps.FeatureInput(f.table, f.feature, f.pooling, pinned(f.keys), pinned(f.offsets))
              for f in w.features]
    houts = [pinned(np.zeros((f.output_rows, dims[f.table]), np.float32)) for f in w.features]
    hgrads = [pinned(g) for g in w.gradients]
    if dist:
        # host buffers: pinned copies in, the round through ShardedClient, outputs out
        tk = [torch.from_numpy(f.keys.view(np.int64)) for f in hfeats]
        to = [torch.from_numpy(f.offsets.view(np.int64)) for f in hfeats]
        th = [torch.from_numpy(o) for o in houts]
        tg = [torch.from_numpy(g) for g in hgrads]

        def e2e_round():
            with torch.cuda.stream(ids_stream):
                dfeats = [eps.FeatureInput(f.table, f.feature, f.pooling,
                                           k.to(dev, non_blocking=True),
                                           o.to(dev, non_blocking=True))
                          for f, k, o in zip(w.features, tk, to)]
            handle, _ = client.lookup(dfeats, outputs=outs, input_stream=ids_stream)
            for h, o in zip(th, outs):
                h.copy_(o, non_blocking=True)
            client.push(handle, [g.to(dev, non_blocking=True) for g in tg])
            torch.cuda.current_stream(dev).synchronize()
    else:
        hlookup = store.prepare_lookup(hfeats, houts)
        hpush = store.prepare_push(hgrads)

        def e2e_round():
            hpush(hlookup(stream), stream, wait=True)
    e2e_steps = max(3, args.steps // 2)
    for _ in range(2):
        e2e_round()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(e2e_steps)]
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    gc.collect()
    gc.disable()
    for a, b in ev:
        flush.zero_()
        a.record(stream)
        e2e_round()
        b.record(stream)
    torch.cuda.synchronize()
    gc.enable()
    e2e_ms = sum(a.elapsed_time(b) for a, b in ev)
    if dist:
        t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = job_N * e2e_steps / (e2e_ms / 1e3)
    h2d = sum(f.keys.nbytes + f.offsets.nbytes for f in w.features) + \
        sum(g.nbytes for g in w.gradients)
    d2h = sum(o.nbytes for o in houts) + 36      # pooled outputs + push status
    if dist:
        if nxt[0] is not None:
            client.discard(nxt[0])
        torch.cuda.synchronize()
        client.close()
        comm.close()
        comm_in.close()
    store.close()

    # ---- CPU baseline (rank 0, N = 1): reference CPU path, bounded sample
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = host_threads()
        times = reference_rounds(w, steps=2, warmup=1, threads=threads)
        if times:
            cpu = {"value": w.occurrences * len(times) / sum(times), "unit": UNIT,
                   "cores": threads, "kind": "reference",
                   "sample": f"{len(times)} full rounds of the same batch after 1 warm-up round "
                             f"(reference DistributedClient over {threads} CpuParameterService "
                             f"shards, one per host thread)"}

    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": w.name, "occurrences_per_round": job_N,
                   "unique_rows_per_round": bm["U"], "output_rows_per_round": bm["B"],
                   "compulsory_bytes_per_round": bm["pull"] + bm["push"],
                   "l2": "flushed (256 MiB write) before every timed round",
                   "parallelism": "single GPU" if world == 1 else
                   f"{world} shards (rows by key % {world}), NCCL all-to-all of keys, "
                   f"partials and gradients; one batch per GPU"},
        "unique_rows_per_s": job_U * args.steps / (total_ms / 1e3),
        "round_hbm_frac": ((bm["pull"] + bm["push"]) * args.steps / (total_ms / 1e3) / 1e9) / peak,
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic, "alg_bytes_per_launch": alg},
        "phases": phases,
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": launches,
        "host_us_per_round": {"median": 1e6 * float(np.median(host_s)),
                              "max": 1e6 * max(host_s),
                              "argmax": int(np.argmax(host_s)),
                              "rounds_ms": [round(a.elapsed_time(b), 4) for a, b in events]},
        "clocks": clk,
    }
    print(json.dumps(line))


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
