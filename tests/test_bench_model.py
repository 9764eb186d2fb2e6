"""bench.py's byte model and roofline-kernel choice (CPU): the compulsory HBM
bytes per round, recomputed here independently on a multi-table workload with
mixed dimensions, pooling modes and rows hot enough to take the long-row path."""
import importlib.util
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def load_bench():
    spec = importlib.util.spec_from_file_location("eps_bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_byte_model_matches_an_independent_count(workloads):
    bench = load_bench()
    w = workloads.small(5, rows=40)
    bm = bench.byte_model(w.tables, w.features)
    dims = {t.id: t.dimension for t in w.tables}
    n = sum(len(f.keys) for f in w.features)
    uniq, longs = {}, {}
    for t in w.tables:
        ks = np.concatenate([f.keys for f in w.features if f.table == t.id])
        u, c = np.unique(ks, return_counts=True)
        uniq[t.id], longs[t.id] = len(u), int((c > 64).sum())
    outs = sum(4 * dims[f.table] * f.output_rows for f in w.features)
    offs = sum(len(f.offsets) for f in w.features if f.pooling != 2)
    rows_u = sum(4 * dims[t] * u for t, u in uniq.items())
    assert bm["N"] == n and bm["U"] == sum(uniq.values())
    assert bm["pull"] == 8 * n + 8 * offs + rows_u + outs
    assert bm["push"] == outs + 8 * n + 8 * offs + 6 * rows_u + 16 * sum(uniq.values())
    own = bm["owner"]
    assert own["apply"] == sum((24 * dims[t] + 16) * (uniq[t] - longs[t]) for t in uniq)
    assert own["long"] == sum((24 * dims[t] + 16) * longs[t] for t in uniq)
    assert sum(longs.values()) > 0 and bm["owner_U_long"] == sum(longs.values())
    assert own["prescan"] == outs and own["lookup"] == bm["pull"]
    assert "sort" not in own and "pieces" not in own


def test_owner_bytes_split_the_job_across_shards(workloads):
    """At n shards each owner's kernels move its own keys, its own unique rows
    and the partial rows of the bags that have keys on it; the owners' shares
    add up to the job's keys and rows."""
    bench = load_bench()
    parts = [workloads.small(7 + r, rows=60) for r in range(2)]
    feats, _ = bench.job_features(parts)
    job = bench.byte_model(parts[0].tables, feats)
    owners = [bench.byte_model(parts[0].tables, feats, 2, r) for r in range(2)]
    assert all(o["N"] == job["N"] and o["U"] == job["U"] for o in owners)
    assert sum(o["owner_N"] for o in owners) == job["N"]
    assert sum(o["owner_U"] for o in owners) == job["U"]
    dims = {t.id: t.dimension for t in parts[0].tables}
    for r, o in enumerate(owners):
        kept = 0
        for f in feats:
            own = (f.keys % np.uint64(2)) == np.uint64(r)
            if f.pooling == 2:
                kept += 4 * dims[f.table] * int(own.sum())
            else:
                lengths = np.diff(f.offsets.astype(np.int64))
                bag = np.repeat(np.arange(len(lengths)), lengths)
                kept += 4 * dims[f.table] * len(np.unique(bag[own]))
        assert o["owner"]["prescan"] == kept


def test_dominant_kernel_is_the_longest_phase_with_bytes():
    bench = load_bench()
    bm = {"lookup": 10, "apply": 20, "long": 5, "prescan": 1, "sort": 0, "pieces": 0, "emit": 0}
    prof = {"lookup": {"ms": 2.0, "calls": 20}, "sort": {"ms": 9.0, "calls": 20},
            "apply": {"ms": 1.9, "calls": 20}, "pieces": {"ms": 3.0, "calls": 20},
            "long": {"ms": 0.5, "calls": 20}, "prescan": {"ms": 0.3, "calls": 20},
            "emit": {"ms": 0.4, "calls": 20}, "finalize": {"ms": 0.0, "calls": 0}}
    assert bench.dominant_kernel(prof, bm) == "lookup"      # the sort and pieces have no bytes
    prof["apply"]["ms"] = 2.5
    assert bench.dominant_kernel(prof, bm) == "apply"


def test_default_config_per_world_size():
    """Config 2 at N = 1 (the single-GPU config), config 3 at N > 1 (the
    26-table config measured at 1/2/4/8 GPUs); an explicit --config wins."""
    bench = load_bench()
    import argparse
    for world, want in ((1, 2), (2, 3), (8, 3)):
        a = argparse.Namespace(config=None)
        assert bench.resolve_config(a, world) == want and a.config_default
    a = argparse.Namespace(config=5)
    assert bench.resolve_config(a, 8) == 5 and not a.config_default


def test_gradient_free_parts_keep_the_keys(workloads):
    """Other ranks' parts are generated without gradients; their keys (drawn
    first from the same seeded stream) must equal the full generation's."""
    for make in (lambda g: workloads.config2(seed=7, rows=100_000, batch=64, gradients=g),
                 lambda g: workloads.config3(seed=7, batch=64, row_scale=1e-3, gradients=g),
                 lambda g: workloads.config4(seed=7, rows=100_000, n=256, gradients=g),
                 lambda g: workloads.config5(seed=7, rows=100_000, batch=64, gradients=g)):
        full, keys_only = make(True), make(False)
        assert all(g is None for g in keys_only.gradients)
        for a, b in zip(full.features, keys_only.features):
            assert np.array_equal(a.keys, b.keys) and np.array_equal(a.offsets, b.offsets)


def test_scaled_batch_and_samples():
    """The parity and reference samples shrink the per-rank batch in proportion,
    never below one sample; config 1's fixed batch is never scaled."""
    bench = load_bench()
    import argparse
    a = argparse.Namespace(config=3, batch=0)
    assert bench.scaled_batch(a, 1.0) == 0                    # 0: the configured batch
    assert bench.scaled_batch(a, 0.25) == 65536 // 4
    assert bench.scaled_batch(a, 1e-9) == 1
    a = argparse.Namespace(config=1, batch=0)
    assert bench.scaled_batch(a, 0.1) == 0


def test_head_start_covers_host_stalls():
    """The untimed flushes queued before the first timed round: at N = 1 at least
    10 ms (250 flushes of 40 us), more when one round's host time is longer, at
    most 60 ms; at N > 1 always 60 ms (1,500 flushes)."""
    bench = load_bench()
    assert bench.head_start_flushes(90e-6, 1) == 250            # a cfg2 round's host time
    assert bench.head_start_flushes(0.0, 1) == 250
    assert bench.head_start_flushes(20e-3, 1) == 500            # 20 ms of host time per round
    assert bench.head_start_flushes(1.0, 1) == 1500
    for world in (2, 8):
        assert bench.head_start_flushes(90e-6, world) == 1500
    assert 250 * bench.FLUSH_S >= 10e-3
