#!/usr/bin/env python
"""Embedding rows/s per round (pull + push + LazyAdam) on B200.

One *round* (= one bench step) over the configured synthetic batch is: one
lookup (gather + sum/mean pooling of every feature, occurrence list and its
coalescing sort) and one push (gradient prescan, coalesced segment-sum fused
with the sparse LazyAdam update, finalize).  rows = id occurrences processed per
round (each is pulled once and contributes one gradient).  Config 4 is the
push-heavy stress: at N = 1 its round is timed without the gather (a push-only
lookup builds the occurrence list and the coalescing sort -- the dedup -- then
the push runs), as BASELINE.json specifies (dedup + segment-sum + Adam only).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--config 1|2|3|4|5] [--no-check] [--no-cpu-baseline]

value  : rows/s of the whole job (every rank's batch) with inputs resident in
         HBM, device-timed with CUDA events on the launching stream, L2 flushed
         (256 MiB write) before every timed round; max over ranks when N > 1.
e2e    : the same rounds through the public API with HOST (pinned) buffers:
         keys and offsets copied in, pooled outputs copied out, gradients copied
         in and the push status read back, all inside the timed region.
roofline: the dominant kernel (the longest single-launch phase with compulsory
         HBM bytes: gather, row updates or prescan) -- the bytes it must move per
         launch (owner-side at N > 1) over its CUDA-event duration, timed by the
         library's phase events in a separate profiled pass of the same rounds,
         against the measured HBM copy bandwidth in MEASURED_PEAKS.json.
parity : one round from freshly initialised tables checked against the
         unmodified reference CPU parameter server (oracle/_ref) serving the same
         job with the same shard count (tests/round_check.py): outputs and the
         rows with <= 64 occurrences bit-exact, longer rows within 1e-6 of their
         sum of |terms|; at N = 1 also the bit-exact mode
         (EPS_B200_FLAG_REFERENCE_ORDER), every row bit-exact.  Runs after all
         timing, never inside a timed region.
cpu_baseline / --impl reference: the UNMODIFIED reference CPU parameter server
         (oracle/_ref, compiled from its own sources) with one shard per host
         core behind its DistributedClient, timed wall-clock on the same job.
"""
from __future__ import annotations

import argparse
import gc
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "distributed-recommendation-model-training-system_b200")
sys.path.insert(0, os.path.join(ROOT, "tests"))
METRIC = "embedding rows/s per round (pull+push+Adam)"
UNIT = "rows/s"
FALLBACK_HBM_GBS = 6650.0
LONG_RUN = 64
# pushes the library keeps enqueued before a lookup waits for the oldest: a
# host hiccup shorter than this many queued rounds (23 ms at cfg2) leaves the
# GPU busy; each enqueued round keeps its lookup's slab (~50 MB at cfg2)
ENQUEUED = 64


def _load(name, path, package=False):
    if name in sys.modules:
        return sys.modules[name]
    kw = {"submodule_search_locations": [PKG]} if package else {}
    spec = importlib.util.spec_from_file_location(name, path, **kw)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def load_workloads():
    """The synthetic input generators only (no library)."""
    return _load("eps_b200_workloads", os.path.join(PKG, "workloads.py"))


def load_package():
    return _load("eps_b200", os.path.join(PKG, "__init__.py"), package=True)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", type=int, default=None, choices=[1, 2, 3, 4, 5],
                    help="BASELINE.json config; default 2 (the single-GPU config) at N = 1 "
                         "and 3 (the config measured at 1/2/4/8 GPUs) at N > 1")
    ap.add_argument("--check-occurrences", type=int, default=1 << 22,
                    help="largest job (occurrences over all ranks) the parity round checks "
                         "at full batch; larger jobs are checked at a proportionally smaller "
                         "batch per rank of the same config")
    ap.add_argument("--probe-nvlink", action="store_true",
                    help="instead of a round: under torchrun, the NCCL all-to-all bandwidth "
                         "of this job's ranks at 32/128/512 MiB per peer (max over ranks); "
                         "in one process, a copy-engine copy from GPU 0 to GPU 1; one JSON line")
    ap.add_argument("--no-scale-base", action="store_true",
                    help="at N = 1 with the default config, skip timing the N > 1 default "
                         "config (3) on this GPU")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-check", action="store_true",
                    help="skip the parity check against the reference after the timed rounds")
    ap.add_argument("--no-bitexact", action="store_true",
                    help="skip timing the bit-exact summation mode at N = 1")
    ap.add_argument("--rows", type=int, default=0,
                    help="override the table rows of config 2/4/5 (smaller profiling captures)")
    ap.add_argument("--batch", type=int, default=0,
                    help="override the batch of config 2/3/5 or the gradient rows of config 4 "
                         "(sub-batches within the reference CUDA backend's staging limits)")
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def cfg5_rows(world: int) -> int:
    """Config 5's table: 1e9 x 32 when it fits, else the largest subset whose
    state ([w|m|v] + counter, 392 B per row) split over `world` GPUs stays
    within 150 GB per GPU."""
    return int(min(1_000_000_000, world * 150_000_000_000 // 392))


# per-rank batch of each config (config 4: gradient rows; config 1 is fixed)
DEFAULT_BATCH = {1: 128, 2: 4096, 3: 65536, 4: 262_144, 5: 131072}


def resolve_config(args, world):
    """The config to run: --config, else 2 at N = 1 (the single-GPU config) and
    3 at N > 1 (the 26-table config BASELINE.json measures at 1/2/4/8 GPUs).
    Both arms resolve it the same way."""
    args.config_default = args.config is None
    if args.config is None:
        args.config = 2 if world == 1 else 3
    return args.config


def workload_for(wl, config, rank, world, rows=0, batch=0, gradients=True):
    """Rank `rank`'s batch: every rank draws its own batch (seed per rank) from
    the same id distribution (the config's shared id map and tables).  Without
    `gradients` the batch's keys are the same and its gradients are None."""
    g = gradients
    if config == 1:
        return wl.config1(seed=1 + 1000 * rank, gradients=g)
    if config == 2:
        return wl.config2(seed=2 + 1000 * rank, rows=rows or 10_000_000, batch=batch or 4096,
                          gradients=g)
    if config == 3:
        return wl.config3(seed=3 + 1000 * rank, batch=batch or 65536, gradients=g)
    if config == 4:
        return wl.config4(seed=4 + 1000 * rank, rows=rows or 100_000_000, n=batch or 262_144,
                          gradients=g)
    return wl.config5(seed=5 + 1000 * rank, rows=rows or cfg5_rows(world), batch=batch or 131072,
                      gradients=g)


def push_only(config, world):
    return config == 4 and world == 1


# ------------------------------------------------------------------ byte model
def _feature_rows(f):
    return len(f.keys) if f.pooling == 2 else len(f.offsets) - 1


def byte_model(tables, feats, world=1, rank=0):
    """Compulsory bytes of one round (each byte that must cross HBM once; sort
    scratch, exchange copies and re-reads excluded) of the job whose features
    are `feats` (every rank's, rank-major), and the bytes the kernels of owner
    `rank` move per launch: its keys, its unique rows, the partial rows it
    serves (kept bags) and their gradients."""
    dims = {t.id: t.dimension for t in tables}
    N = sum(len(f.keys) for f in feats)
    B = sum(_feature_rows(f) for f in feats)
    pooled_offsets = sum(len(f.offsets) for f in feats if f.pooling != 2)
    out_bytes = sum(4 * dims[f.table] * _feature_rows(f) for f in feats)
    U, u_row_bytes = 0, 0
    own = {"N": 0, "U": 0, "long": 0, "kept": 0, "kept_bytes": 0, "offsets": 0, "rows": 0,
           "apply": 0, "longb": 0}
    for t in tables:
        ks = [f.keys for f in feats if f.table == t.id]
        if not ks:
            continue
        uk, cnt = np.unique(np.concatenate(ks), return_counts=True)
        U += len(uk)
        u_row_bytes += 4 * t.dimension * len(uk)
        mine = (uk % np.uint64(world)) == np.uint64(rank)
        nu, nl = int(mine.sum()), int((mine & (cnt > LONG_RUN)).sum())
        own["U"] += nu
        own["long"] += nl
        own["rows"] += 4 * t.dimension * nu
        own["apply"] += (24 * t.dimension + 16) * (nu - nl)
        own["longb"] += (24 * t.dimension + 16) * nl
    for f in feats:
        d = dims[f.table]
        sel = (f.keys % np.uint64(world)) == np.uint64(rank)
        own["N"] += int(sel.sum())
        if f.pooling == 2:
            kept = int(sel.sum())
        elif world == 1:
            kept = len(f.offsets) - 1
            own["offsets"] += len(f.offsets)
        else:
            lengths = np.diff(f.offsets.astype(np.int64))
            bag = np.repeat(np.arange(len(lengths)), lengths)
            kept = len(np.unique(bag[sel]))
            own["offsets"] += kept + 1
        own["kept"] += kept
        own["kept_bytes"] += 4 * d * kept
    pull = 8 * N + 8 * pooled_offsets + u_row_bytes + out_bytes
    push = out_bytes + 8 * N + 8 * pooled_offsets + 6 * u_row_bytes + 16 * U
    owner = {"lookup": 8 * own["N"] + 8 * own["offsets"] + own["rows"] + own["kept_bytes"],
             "apply": own["apply"], "long": own["longb"], "prescan": own["kept_bytes"]}
    return {"N": N, "U": U, "B": B, "pull": pull, "push": push, "owner": owner,
            "owner_U": own["U"], "owner_U_long": own["long"], "owner_N": own["N"]}


def job_parts(wl, args, world, grads_for=None, batch=0):
    """Every rank's batch.  Only the ranks in `grads_for` (all when None) carry
    gradients; the others' keys describe the job (byte model, config)."""
    return [workload_for(wl, args.config, r, world, args.rows, batch or args.batch,
                         gradients=grads_for is None or r in grads_for) for r in range(world)]


def scaled_batch(args, frac):
    """The per-rank batch that is `frac` of the configured one (at least 1)."""
    full = args.batch or DEFAULT_BATCH[args.config]
    if args.config == 1 or frac >= 1.0:
        return 0 if not args.batch else args.batch
    return max(1, int(full * frac))


FLUSH_S = 40e-6   # device time of one L2 flush (a 256 MiB fill)


def head_start_flushes(round_host_s, world):
    """L2 flushes queued (untimed) before the first timed round, so that the host
    starts the timed rounds with the lead it has in steady state.

    At least one round's host time, and at least 250 (10 ms): the timed rounds'
    whole enqueue (~2 ms at N = 1) then ends before the first of them starts, so
    that a host stall of a few milliseconds (an nvidia-smi query holds the
    driver; one of 8.5 ms fell on the third timed round of a default run with a
    3-flush head start) cannot leave the device idle inside a timed round; at
    most 1,500.  At N > 1 exactly 1,500 (60 ms): after the synchronize a sharded
    round runs at about twice its steady time for ~50 ms (measured at N = 2, the
    same whether 1, 2 or 3 batches are prepared ahead), and a longer head start
    shortens that transient by its own length."""
    head = int(min(1500, max(250, np.ceil(round_host_s / FLUSH_S))))
    return max(head, 1500) if world > 1 else head


def job_features(parts):
    """Every rank's features as the one combined request (ids r * F + f)."""
    F = len(parts[0].features)
    feats, grads = [], []
    for r, p in enumerate(parts):
        for f, g in zip(p.features, p.gradients):
            feats.append(type(f)(f.table, r * F + f.feature, f.pooling, f.keys, f.offsets))
            grads.append(g)
    return feats, grads


def job_config(parts, bm, config, world):
    """The `config` object both arms print (identical for the same job)."""
    only_push = push_only(config, world)
    return {"workload": parts[0].name, "config": config, "batches": len(parts),
            "occurrences_per_round": bm["N"], "unique_rows_per_round": bm["U"],
            "output_rows_per_round": bm["B"],
            "compulsory_bytes_per_round": bm["push"] if only_push else bm["pull"] + bm["push"],
            "timed": ("push only: dedup (coalescing sort) + segment-sum + LazyAdam, no gather"
                      if only_push else "pull + push + LazyAdam")}


def dominant_kernel(prof, owner):
    """The roofline's kernel: the phase with the longest time per call among
    those with compulsory HBM bytes (gather, row updates, long rows, prescan)."""
    cands = [p for p in prof if owner.get(p) and prof[p]["ms"]]
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


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


class Clocks:
    """nvidia-smi samples during the timed region: SM clocks and throttle
    reasons of every GPU of the job, by ONE sampler (local rank 0's).  A query
    can hold up driver calls for tens of milliseconds: one sampler per rank (8
    queries per period at N = 8) showed as host stalls of 13-60 ms inside timed
    rounds, and the power reading is left out for the same reason."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, local_rank, local_world=1):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        ids = vis.split(",") if vis else [str(i) for i in range(local_world)]
        self.index = ",".join(ids[:local_world])
        self.owner = local_rank == 0
        self.proc = None
        self.path = None

    def start(self):
        if not self.owner:
            return
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.out = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.index, f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
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
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[4:8]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "gpus": self.index, "samples": len(rows),
                "window": "warm-up start to the end of a 0.5 s untimed soak of the same rounds"}


# --------------------------------------------------------------- reference arm
def reference_rounds(wl, args, world, steps, warmup, threads, budget_s=60.0, round_s=2.0):
    """Times the reference's CPU path (oracle/_ref: DistributedClient over
    `threads` CpuParameterService shards) on a bounded sample of the job: every
    rank's batch as one combined request -- at the configured batch when one
    round of the whole job takes about `round_s` seconds or less, else at a
    proportionally smaller batch per rank of the same config (same tables, id
    distribution and seeds), sized from one untimed probe round of at most 2^18
    occurrences.  Push-only configs time the push alone.  Stops early (at least
    2 timed rounds) once `budget_s` of timed work is done.  Returns (seconds of
    each timed round, the sampled parts), or None without the reference build."""
    from oracle_lib import Feature, Reference, reference_available
    import round_check
    if not reference_available():
        return None
    full = job_parts(wl, args, world, grads_for=())
    n_full = sum(p.occurrences for p in full)
    tables = round_check.table_defs(full[0])
    del full
    ref = Reference(tables, shards=threads, state_bytes=256 << 30)
    only_push = push_only(args.config, world)

    def request(parts):
        feats, grads = job_features(parts)
        return [Feature(f.table, f.feature, f.pooling, f.keys, f.offsets) for f in feats], grads

    probe_frac = min(1.0, (1 << 18) / n_full)
    probe = job_parts(wl, args, world, batch=scaled_batch(args, probe_frac))
    feats, grads = request(probe)
    t0 = time.perf_counter()
    batch, _ = ref.lookup(feats)
    ref.push(batch, feats, grads)
    cost = (time.perf_counter() - t0) / max(1, sum(p.occurrences for p in probe))
    frac = min(1.0, round_s / max(cost * n_full, 1e-9))
    sample = job_parts(wl, args, world, batch=scaled_batch(args, frac))
    feats, grads = request(sample)
    times, spent = [], 0.0
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        batch, _ = ref.lookup(feats)
        if only_push:
            t0 = time.perf_counter()
        ref.push(batch, feats, grads)
        dt = time.perf_counter() - t0
        if i >= warmup:
            times.append(dt)
            spent += dt
            if spent > budget_s and len(times) >= 2:
                break
    ref.close()
    return times, sample


def sample_text(sample, n_job, rounds, warmup, what, threads):
    n = sum(p.occurrences for p in sample)
    per = len(sample[0].features[0].offsets) - 1
    part = ("the whole job" if n >= n_job else
            f"a sample of the job: {per} samples per rank of the same config "
            f"({n} of its {n_job} occurrences)")
    return (f"{rounds} rounds ({what}) of {part}, {len(sample)} batch(es) as one request, "
            f"after {warmup} warm-up rounds; DistributedClient over {threads} "
            f"CpuParameterService shards (one per host thread)")


def run_reference(args):
    rank, local_rank, world = dist_env()
    if rank != 0:
        return
    wl = load_workloads()              # the generators only: no repo library is loaded
    resolve_config(args, world)
    parts = job_parts(wl, args, world, grads_for=())
    feats, _ = job_features(parts)
    bm = byte_model(parts[0].tables, feats, world, 0)
    del feats
    threads = host_threads()
    got = reference_rounds(wl, args, world, args.steps, args.warmup, threads)
    if got is None:
        print(json.dumps({"impl": "reference", "unavailable":
                          "reference CPU build oracle/_ref/libeps_ref.so is missing"}))
        return
    times, smp = got
    total = sum(times)
    value = sum(p.occurrences for p in smp) * len(times) / total
    what = "push" if push_only(args.config, world) else "lookup + push"
    sample = sample_text(smp, bm["N"], len(times), args.warmup, what, threads)
    print(json.dumps({
        "metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
        "steps": len(times), "warmup": args.warmup, "ms_per_step": 1e3 * total / len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": job_config(parts, bm, args.config, world),
        "parallelism": f"cpu x{threads}",
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "reference",
                         "cpu_model": cpu_model(), "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))


# ------------------------------------------------------------------- B200 arm
def _create_tables(eps, store, w, world):
    for t in w.tables:
        store.create_table(eps.TableDefinition(id=t.id, dimension=t.dimension, key_space=t.rows,
                                               learning_rate=1e-3, shard_count=world))


def parity_check(eps, torch, wl, args, parts, rank, world, dev, comms, bitexact):
    """One round from fresh tables against the reference (tests/round_check.py),
    through the same path as the timed rounds (the NCCL round at N > 1).  The
    job is the timed one when it has at most --check-occurrences occurrences,
    else the same config at a proportionally smaller batch per rank (every rank
    runs the reference on the whole job).  Returns this rank's reports (default
    order; at N = 1 also the bit-exact mode)."""
    import round_check as rc
    n_job = sum(p.occurrences for p in parts)
    frac = min(1.0, args.check_occurrences / n_job)
    if world > 1 or frac < 1.0:
        parts = job_parts(wl, args, world, batch=scaled_batch(args, frac))
    w = parts[rank]
    ref_result = rc.reference_round(parts)
    checked = {"check_occurrences": sum(p.occurrences for p in parts),
               "check_samples_per_rank": len(parts[0].features[0].offsets) - 1,
               "job_occurrences": n_job}
    reports = []
    modes = [False, True] if (world == 1 and bitexact) else [False]
    for reference_order in modes:
        store = eps.ParameterStore(device=dev.index, shard_id=rank, shard_count=world,
                                   state_bytes=170 << 30, reference_order=reference_order)
        try:
            _create_tables(eps, store, w, world)
            feats = [eps.FeatureInput(f.table, f.feature, f.pooling,
                                      torch.from_numpy(f.keys.astype(np.int64)).to(dev),
                                      torch.from_numpy(f.offsets.astype(np.int64)).to(dev))
                     for f in w.features]
            grads = [torch.from_numpy(g).to(dev) for g in w.gradients]
            if world == 1:
                ticket, outs = store.lookup(feats)
                store.push(ticket, grads)
            else:
                import importlib
                D = importlib.import_module("eps_b200.distributed")
                client = D.NativeClient(store, comms[0], comms[1])
                handle, outs = client.lookup(feats)
                client.push(handle, grads, wait=True)
                torch.cuda.synchronize()
                client.close()
            outs = [o.cpu().numpy() for o in outs]
            rep = rc.check_round(parts, rank, outs, store.read_state,
                                 reference_order=reference_order, ref_result=ref_result)
            rep.update(checked)
        finally:
            store.close()
        reports.append(rep)
    ref_result[0].close()
    return reports


def e2e_pipelined(eps, torch, store, stream, w, hfeats, houts, hgrads, flush, steps, dev):
    """End-to-end rounds through the public API from pinned host buffers, with
    the copies of consecutive rounds overlapped as a training loop overlaps
    them: round k + 1's keys and offsets are copied in while round k runs; round
    k's pooled outputs are copied out as soon as its gather ends (its coalescing
    sort still running); its gradients, which a training step computes from
    those outputs, are copied in after them; then its push, whose status the
    library copies back.  Two sets of device buffers alternate.  One window of
    CUDA events on the store's stream covers every round, the L2 flush before
    each round included.  Returns the window in milliseconds."""
    nb = 2
    dk = [[torch.empty(len(f.keys), dtype=torch.int64, device=dev) for f in hfeats] for _ in range(nb)]
    do = [[torch.empty(len(f.offsets), dtype=torch.int64, device=dev) for f in hfeats]
          for _ in range(nb)]
    dout = None if houts is None else [[torch.empty(o.shape, dtype=torch.float32, device=dev)
                                         for o in houts] for _ in range(nb)]
    hout2 = None if houts is None else [
        houts, [torch.empty(o.shape, dtype=torch.float32, pin_memory=True).numpy() for o in houts]]
    dg = [[torch.empty(g.shape, dtype=torch.float32, device=dev) for g in hgrads] for _ in range(nb)]
    tk = [torch.from_numpy(f.keys.view(np.int64)) for f in hfeats]
    to = [torch.from_numpy(f.offsets.view(np.int64)) for f in hfeats]
    tg = [torch.from_numpy(g) for g in hgrads]
    looks, pushes = [], []
    for b in range(nb):
        feats_b = [eps.FeatureInput(f.table, f.feature, f.pooling, dk[b][i], do[b][i])
                   for i, f in enumerate(hfeats)]
        looks.append(store.prepare_lookup(feats_b, None if dout is None else dout[b]))
        pushes.append(store.prepare_push(dg[b]))
    sk = torch.cuda.Stream(device=dev)       # keys / offsets in
    so = torch.cuda.Stream(device=dev)       # outputs out
    sg = torch.cuda.Stream(device=dev)       # gradients in
    E = lambda: torch.cuda.Event()           # noqa: E731

    def copy_keys(b):
        with torch.cuda.stream(sk):
            for i in range(len(hfeats)):
                dk[b][i].copy_(tk[i], non_blocking=True)
                do[b][i].copy_(to[i], non_blocking=True)
        e = E()
        e.record(sk)
        return e

    def run(nrounds, timed):
        keys_ready = [None] * nb
        free_in = [None] * nb                 # the buffer set's lookup has read its inputs
        free_out = [None] * nb                # its outputs have been copied out
        free_g = [None] * nb                  # its push has read its gradients
        keys_ready[0] = copy_keys(0)
        t0 = t1 = None
        for k in range(nrounds):
            b = k % nb
            flush.zero_()
            if timed and k == 0:
                t0 = torch.cuda.Event(enable_timing=True)
                t0.record(stream)
            stream.wait_event(keys_ready[b])
            if free_out[b] is not None:
                stream.wait_event(free_out[b])
            ticket = looks[b](stream)
            looked = E()
            looked.record(stream)
            free_in[b] = looked
            if k + 1 < nrounds:               # the next round's keys, during this round
                b2 = (k + 1) % nb
                if free_in[b2] is not None:
                    sk.wait_event(free_in[b2])
                keys_ready[b2] = copy_keys(b2)
            after = looked
            if dout is not None:
                so.wait_event(looked)
                with torch.cuda.stream(so):
                    for h, o in zip(hout2[b], dout[b]):
                        torch.from_numpy(h).copy_(o, non_blocking=True)
                after = E()
                after.record(so)
                free_out[b] = after
            sg.wait_event(after)
            if free_g[b] is not None:
                sg.wait_event(free_g[b])
            with torch.cuda.stream(sg):
                for d, h in zip(dg[b], tg):
                    d.copy_(h, non_blocking=True)
            gready = E()
            gready.record(sg)
            stream.wait_event(gready)
            pushes[b](ticket, stream, wait=False)
            pushed = E()
            pushed.record(stream)
            free_g[b] = pushed
        if timed:
            t1 = torch.cuda.Event(enable_timing=True)
            t1.record(stream)
        torch.cuda.synchronize()
        store.synchronize()                    # every push's status, read back
        return t0, t1

    run(3, False)
    gc.collect()
    gc.disable()
    t0, t1 = run(steps, True)
    gc.enable()
    return t0.elapsed_time(t1)


def scale_base_rounds(eps, torch, wl, args, dev, local_rank):
    """Config 3 -- the default at N > 1 -- timed on this one GPU as the main
    rounds are (inputs resident, L2 flushed before every round, CUDA events on
    the store's stream): the N = 1 point of the scaling curve that the N > 1
    lines measure."""
    w = workload_for(wl, 3, 0, 1)
    store = eps.ParameterStore(device=local_rank, state_bytes=170 << 30,
                               max_enqueued_pushes=ENQUEUED)
    try:
        _create_tables(eps, store, w, 1)
        stream = torch.cuda.current_stream(dev)
        dims = {t.id: t.dimension for t in w.tables}
        feats = [eps.FeatureInput(f.table, f.feature, f.pooling,
                                  torch.from_numpy(f.keys.astype(np.int64)).to(dev),
                                  torch.from_numpy(f.offsets.astype(np.int64)).to(dev))
                 for f in w.features]
        outs = [torch.empty((f.output_rows, dims[f.table]), dtype=torch.float32, device=dev)
                for f in w.features]
        grads = [torch.from_numpy(g).to(dev) for g in w.gradients]
        flush = torch.empty(64 << 20, dtype=torch.float32, device=dev)
        lookup = store.prepare_lookup(feats, outs)
        push = store.prepare_push(grads)
        for _ in range(ENQUEUED + 4 + args.warmup):
            flush.zero_()
            push(lookup(stream), stream, wait=False)
        store.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
        torch.cuda.synchronize()
        for _ in range(head_start_flushes(0.0, 1)):   # the main rounds' head start
            flush.zero_()
        for a, b in ev:
            flush.zero_()
            a.record(stream)
            push(lookup(stream), stream, wait=False)
            b.record(stream)
        torch.cuda.synchronize()
        store.synchronize()
        ms = sum(a.elapsed_time(b) for a, b in ev) / args.steps
        return {"workload": w.name, "config": 3, "n_gpus": 1, "steps": args.steps,
                "ms_per_step": ms, "value": w.occurrences / (ms / 1e3), "unit": UNIT,
                "note": "config 3 (the default at N > 1) on one GPU, timed like the main "
                        "rounds: the N = 1 point of the curve the N > 1 lines continue"}
    finally:
        store.close()


def run_b200(args):
    import torch
    rank, local_rank, world = dist_env()
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device(f"cuda:{local_rank}"))
    wl = load_workloads()
    eps = load_package()
    resolve_config(args, world)
    parts = job_parts(wl, args, world, grads_for={rank})
    w = parts[rank]
    jfeats, _ = job_features(parts)
    bm = byte_model(w.tables, jfeats, world, rank)
    only_push = push_only(args.config, world)
    dev = torch.device(f"cuda:{local_rank}")
    # one shard per rank: keys k with k % world == rank (the table's rows are split)
    store = eps.ParameterStore(device=local_rank, shard_id=rank, shard_count=world,
                               state_bytes=170 << 30, max_enqueued_pushes=ENQUEUED)
    _create_tables(eps, store, w, world)
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)          # flushes and events run on the store's stream

    # ---- device-resident inputs
    feats = [eps.FeatureInput(f.table, f.feature, f.pooling,
                              torch.from_numpy(f.keys.astype(np.int64)).to(dev),
                              torch.from_numpy(f.offsets.astype(np.int64)).to(dev))
             for f in w.features]
    dims = {t.id: t.dimension for t in w.tables}
    outs = None if only_push else [
        torch.empty((f.output_rows, dims[f.table]), dtype=torch.float32, device=dev)
        for f in w.features]
    grads = [torch.from_numpy(g).to(dev) for g in w.gradients]
    flush = torch.empty(64 << 20, dtype=torch.float32, device=dev)   # 256 MiB > 126 MB L2
    comms = (None, None)
    if dist:
        # every rank's batch is routed to the owners over NCCL all-to-all
        import importlib
        D = importlib.import_module("eps_b200.distributed")
        comm = D.NcclComm.from_process_group(local_rank)    # NCCL group calls on our streams
        comm_in = D.NcclComm.from_process_group(local_rank)  # the prepare phase's exchanges
        comms = (comm, comm_in)
        client = D.NativeClient(store, comm, comm_in)        # the round's host side in C++
        # batches are prepared (partition + count exchange) two rounds ahead on a
        # high-priority input stream, as a training loop whose loader holds the
        # next batches would: a prepare issues the key exchange of the batch
        # before it, whose counts arrived a round earlier, so the host never
        # waits for the device; every timed step contains exactly one prepare,
        # one lookup and one push
        ids_stream = torch.cuda.Stream(device=dev, priority=-1)
        from collections import deque
        nxt = deque()

        def one_round():
            while len(nxt) < 2:
                nxt.append(client.prepare(feats, input_stream=ids_stream))
            handle, _ = client.lookup_prepared(nxt.popleft(), outputs=outs)
            nxt.append(client.prepare(feats, input_stream=ids_stream))
            client.push(handle, grads)
    else:
        lookup = store.prepare_lookup(feats, outs)
        push = store.prepare_push(grads)

        def one_round():
            ticket = lookup(stream)
            push(ticket, stream, wait=False)

    # the clock sampler first: its start-up must be over before timed work
    clocks = Clocks(local_rank, int(os.environ.get("LOCAL_WORLD_SIZE", world)))
    clocks.start()
    clocks.wait_first()
    # allocator priming (untimed): more rounds in flight than the library's
    # limit of enqueued pushes, so that the stream-ordered memory pool reaches
    # its steady size before the warm-up and never grows (maps new memory, a
    # host stall of milliseconds) inside the timed rounds
    for _ in range(ENQUEUED + 4):
        one_round()
    store.synchronize()
    clocks.mark()
    # no Python collector pauses inside the warm-up and the timed rounds (a pause
    # longer than the rounds queued ahead of the host would leave the device
    # idle); collecting here, before the warm-up, keeps the device busy right up
    # to the first timed round
    gc.collect()
    gc.disable()
    warm_host = []
    for _ in range(args.warmup):
        flush.zero_()
        h0 = time.perf_counter()
        one_round()
        warm_host.append(time.perf_counter() - h0)
    store.synchronize()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    launches0 = store.stats()["kernel_launches"]
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
    torch.cuda.synchronize()
    # after the synchronize the device queue is empty: extra L2 flushes (untimed,
    # queued before round 0's start event) give the host its steady-state head
    # start (see head_start_flushes)
    head = head_start_flushes(float(np.median(warm_host)), world)
    if dist:
        t = torch.tensor([head], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)      # the same count on every rank
        head = int(t.item())
    for _ in range(head):
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
    if dist:
        client.profile(1)
    for _ in range(args.steps):
        flush.zero_()
        one_round()
    torch.cuda.synchronize()
    store.synchronize()
    prof = store.profile(0)
    exch = client.profile(0) if dist else None
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
    if dist:
        t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    value = bm["N"] * args.steps / (total_ms / 1e3)

    # ---- roofline of the dominant phase (bytes the owner's kernels move)
    peak, peak_kind = load_peaks()
    owner = bm["owner"]
    dom = dominant_kernel(prof, owner)
    calls = max(1, prof[dom]["calls"])
    per_call_ms = prof[dom]["ms"] / calls
    alg = owner[dom]
    achieved = alg / (per_call_ms / 1e3) / 1e9 if alg else 0.0
    tr = load_traffic().get(f"cfg{args.config}", {}).get(dom) if world == 1 else None
    traffic = tr.get("bytes") if tr else None
    traffic_capture = tr.get("capture") if tr else None
    phases = {p: {"ms_per_round": prof[p]["ms"] / max(1, prof[p]["calls"]),
                  "launches_per_round": prof[p]["launches"] / max(1, prof[p]["calls"]),
                  "alg_GBps": (owner[p] / (prof[p]["ms"] / max(1, prof[p]["calls"]) / 1e3) / 1e9)
                  if owner.get(p) and prof[p]["ms"] else None} for p in prof}

    # ---- NVLink: this rank's exchanges per round, against the all-to-all
    # bandwidth measured here on the same communicator (256 MiB to every peer:
    # smaller messages do not reach the links' rate)
    nvlink = None
    if dist:
        per = 256 << 20
        src = torch.empty(world * per // 4, dtype=torch.float32, device=dev)
        dst = torch.empty_like(src)
        for _ in range(2):
            comm.all_to_all_single(dst, src)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(5):
            comm.all_to_all_single(dst, src)
        b.record(stream)
        torch.cuda.synchronize()
        a2a_ms = a.elapsed_time(b) / 5
        t = torch.tensor([a2a_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        peak_nv = per * (world - 1) / (float(t.item()) / 1e3) / 1e9
        del src, dst
        calls = max(1, args.steps)
        ex = {k: {"ms_per_round": v["ms"] / calls, "bytes_out_per_round": v["bytes"] / calls,
                  "GBps_out": (v["bytes"] / (v["ms"] / 1e3) / 1e9) if v["ms"] else None}
              for k, v in exch.items()}
        out_bytes = sum(v["bytes"] for v in exch.values()) / calls
        out_ms = sum(v["ms"] for v in exch.values()) / calls
        nvlink = {"bytes_out_per_round": out_bytes, "exchange_ms_per_round": out_ms,
                  "achieved_GBps_out": out_bytes / (out_ms / 1e3) / 1e9 if out_ms else None,
                  "alltoall_peak_GBps_out": peak_nv,
                  "frac": (out_bytes / (out_ms / 1e3) / 1e9) / peak_nv if out_ms else None,
                  "exchanges": ex,
                  "peak": f"NCCL all-to-all of {per >> 20} MiB to every peer on the round's "
                          f"communicator, this rank's outgoing bytes / time (max over ranks)"}

    # ---- e2e through the public API with pinned host buffers
    def pinned(a):
        t = torch.empty(a.shape, dtype=torch.from_numpy(a[:0]).dtype, pin_memory=True)
        t.numpy()[...] = a
        return t.numpy()

    hfeats = [eps.FeatureInput(f.table, f.feature, f.pooling, pinned(f.keys), pinned(f.offsets))
              for f in w.features]
    houts = None if only_push else [pinned(np.zeros((f.output_rows, dims[f.table]), np.float32))
                                    for f in w.features]
    hgrads = [pinned(g) for g in w.gradients]
    if dist:
        # host buffers: pinned copies in, the round through the C++ client, outputs out
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
    e2e_steps = max(3, args.steps // 2)
    if dist:
        for _ in range(2):
            e2e_round()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(e2e_steps)]
        torch.cuda.synchronize()
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
    else:
        e2e_ms = e2e_pipelined(eps, torch, store, stream, w, hfeats, houts, hgrads, flush,
                               e2e_steps, dev)
    if dist:
        t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = bm["N"] * e2e_steps / (e2e_ms / 1e3)
    h2d = sum(f.keys.nbytes + f.offsets.nbytes for f in w.features) + \
        sum(g.nbytes for g in w.gradients)
    d2h = (0 if houts is None else sum(o.nbytes for o in houts)) + 36  # outputs + push status
    if dist:
        while nxt:
            client.discard(nxt.popleft())
        torch.cuda.synchronize()
        client.close()
    store.close()
    del flush

    # ---- the bit-exact summation mode (EPS_B200_FLAG_REFERENCE_ORDER) at N = 1:
    # the same timed rounds on a fresh store that sums every row serially
    bitexact = None
    if world == 1 and not args.no_bitexact:
        store = eps.ParameterStore(device=local_rank, state_bytes=170 << 30, reference_order=True)
        _create_tables(eps, store, w, world)
        flush = torch.empty(64 << 20, dtype=torch.float32, device=dev)
        lookup = store.prepare_lookup(feats, outs)
        push = store.prepare_push(grads)
        for _ in range(args.warmup + 4):
            flush.zero_()
            push(lookup(stream), stream, wait=False)
        store.synchronize()
        bev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        torch.cuda.synchronize()
        for a, b in bev:
            flush.zero_()
            a.record(stream)
            push(lookup(stream), stream, wait=False)
            b.record(stream)
        torch.cuda.synchronize()
        store.synchronize()
        bms = sum(a.elapsed_time(b) for a, b in bev) / args.steps
        bitexact = {"ms_per_step": bms, "value": bm["N"] / (bms / 1e3), "unit": UNIT,
                    "mode": "EPS_B200_FLAG_REFERENCE_ORDER: every row summed serially in "
                            "occurrence order (bit-exact on every row)"}
        store.close()
        del flush

    # ---- parity: one round from fresh tables against the reference (checker only)
    parity = None
    if not args.no_check:
        reports = parity_check(eps, torch, wl, args, parts, rank, world, dev, comms,
                               bitexact=not args.no_bitexact)
        ok = all(r["parity"] for r in reports)
        if dist:
            t = torch.tensor([1.0 if ok else 0.0], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MIN)
            ok = bool(t.item() == 1.0)
            gathered = [None] * world
            dist.all_gather_object(gathered, reports)
            reports = [r for g in gathered for r in g]
        parity = {"parity": ok,
                  "outputs_bitexact": all(r["outputs_bitexact"] for r in reports),
                  "rows_bitexact": all(r["rows_bitexact"] for r in reports),
                  "rows_checked": sum(r["rows_checked"] for r in reports
                                      if not r["reference_order"]),
                  "long_rows": sum(r["long_rows"] for r in reports),
                  "long_max_norm_err": {k: max(r["long_max_norm_err"][k] for r in reports)
                                        for k in ("w", "m", "v")},
                  "long_max_rel_err": {k: max(r["long_max_rel_err"][k] for r in reports)
                                       for k in ("w", "m", "v")},
                  "bitexact_mode_checked": any(r["reference_order"] for r in reports),
                  "job_occurrences_checked": reports[0]["check_occurrences"],
                  "samples_per_rank_checked": reports[0]["check_samples_per_rank"],
                  "job": ("the timed job" if reports[0]["check_occurrences"] ==
                          reports[0]["job_occurrences"] else
                          "the same config at a smaller batch per rank (every rank runs the "
                          "reference on the whole job)")}
    if dist:
        comms[0].close()
        comms[1].close()

    # ---- CPU baseline (rank 0, N = 1): reference CPU path, bounded sample
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = host_threads()
        got = reference_rounds(wl, args, world, steps=args.steps, warmup=1, threads=threads,
                               budget_s=15.0, round_s=1.0)
        if got:
            times, smp = got
            what = "push" if only_push else "lookup + push"
            cpu = {"value": sum(p.occurrences for p in smp) * len(times) / sum(times),
                   "unit": UNIT, "cores": threads, "kind": "reference", "cpu_model": cpu_model(),
                   "sample": sample_text(smp, bm["N"], len(times), 1, what, threads) +
                   "; at most ~15 s of timed rounds"}

    # ---- at N = 1 with the default config: the N > 1 default config (3) on this
    # GPU, device-timed as above, the base of its weak-scaling curve
    scale_base = None
    if world == 1 and args.config_default and not args.no_scale_base:
        scale_base = scale_base_rounds(eps, torch, wl, args, dev, local_rank)

    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": job_config(parts, bm, args.config, world),
        "parallelism": "single GPU" if world == 1 else
        f"{world} shards (rows by key % {world}), NCCL all-to-all of keys, partials and "
        f"gradients; one batch per GPU",
        "l2": "flushed (256 MiB write) before every timed round",
        "head_start_flushes": head,
        "unique_rows_per_s": bm["U"] * args.steps / (total_ms / 1e3),
        "round_hbm_frac": ((bm["push"] if only_push else bm["pull"] + bm["push"]) * args.steps /
                           (total_ms / 1e3) / 1e9) / (peak * world),
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic, "traffic_capture": traffic_capture,
                     "alg_bytes_per_launch": alg,
                     "bytes": "owner-side" if world > 1 else "single GPU"},
        "phases": phases,
        "nvlink": nvlink,
        "owner": {"occurrences": bm["owner_N"], "unique_rows": bm["owner_U"],
                  "long_rows": bm["owner_U_long"]},
        "parity": parity,
        "bitexact_mode": bitexact,
        "cpu_baseline": cpu,
        "scale_base": scale_base,
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


def probe_nvlink(args):
    """NVLink bandwidth available to the round's exchanges.  Under torchrun: the
    NCCL all-to-all of this job's ranks at 32 / 128 / 512 MiB to every peer
    (CUDA events, 5 calls after 3, max over ranks).  Without it (one process
    seeing two or more GPUs): a copy-engine copy of 128 / 512 MiB from GPU 0 to
    GPU 1 with peer access enabled."""
    import torch
    rank, local_rank, world = dist_env()

    def timed(fn, stream, k=5):
        for _ in range(3):
            fn()
        stream.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(k):
            fn()
        b.record(stream)
        stream.synchronize()
        return a.elapsed_time(b) / k

    if "WORLD_SIZE" not in os.environ:
        if torch.cuda.device_count() < 2 or not torch.cuda.can_device_access_peer(0, 1):
            print(json.dumps({"probe": "peer_copy", "unavailable": "needs two GPUs with peer access"}))
            return
        ce = {}
        with torch.cuda.device(0):
            s0 = torch.cuda.Stream(device=0)
            for mib in (128, 512):
                x = torch.empty((mib << 20) // 4, device="cuda:0")
                y = torch.empty_like(x, device="cuda:1")
                with torch.cuda.stream(s0):
                    ms = timed(lambda: y.copy_(x, non_blocking=True), s0)
                torch.cuda.synchronize(1)
                ce[mib] = (mib << 20) / (ms / 1e3) / 1e9
                del x, y
        print(json.dumps({"probe": "peer_copy", "copy_engine_GBps_by_MiB": ce,
                          "path": "GPU 0 -> GPU 1, one process, peer access enabled"}))
        return
    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device(f"cuda:{local_rank}"))
    a2a = {}
    stream = torch.cuda.current_stream()
    for mib in (32, 128, 512):
        per = mib << 20
        src = torch.empty(world * per // 4, device="cuda")
        dst = torch.empty_like(src)
        ms = timed(lambda: dist.all_to_all_single(dst, src), stream)
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        a2a[mib] = per * (world - 1) / (t.item() / 1e3) / 1e9
        del src, dst
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print(json.dumps({"probe": "nvlink", "n_gpus": world,
                          "nccl_env": {k: v for k, v in os.environ.items() if k.startswith("NCCL_")},
                          "alltoall_GBps_out_by_MiB_per_peer": a2a}))


def main():
    args = parse()
    if args.probe_nvlink:
        probe_nvlink(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
