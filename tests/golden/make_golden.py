"""Generates tests/golden/*.npz from the UNMODIFIED reference CPU parameter server.

The reference core is compiled from its own sources by oracle/Makefile
(`make -C oracle ref`) and driven through DistributedClient over n in-process
CpuParameterService shards (oracle/ref_harness.cpp).  For every case the file
records the inputs, the lookup outputs at 1, 2 and 3 shards, and the state
(w, m, v, row_updates) of every touched row after `steps` lookup+push rounds.

Run from the repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
import conftest  # noqa: E402  (package loader)
from oracle_lib import Feature, Reference, TableDef  # noqa: E402

wl = conftest.import_workloads()


def table_defs(w, lr=1e-3, bounds=None):
    return [TableDef(id=t.id, dimension=t.dimension, learning_rate=lr, beta1=0.9, beta2=0.999,
                     epsilon=1e-8, initial_beta1_power=0.9, initial_beta2_power=0.999,
                     bounds=bounds, init_min=-0.05, init_max=0.05, init_seed=42, rows=t.rows)
            for t in w.tables]


def feats(w):
    return [Feature(f.table, f.feature, f.pooling, f.keys, f.offsets) for f in w.features]


def run(name, w, steps=3, lr=1e-3, bounds=None, grad_scale=1.0):
    defs = table_defs(w, lr, bounds)
    out = {"name": np.array(name)}
    out["table_ids"] = np.array([t.id for t in w.tables], np.uint32)
    out["table_dims"] = np.array([t.dimension for t in w.tables], np.uint32)
    out["table_rows"] = np.array([t.rows for t in w.tables], np.uint64)
    out["lr"] = np.float32(lr)
    out["bounds"] = np.array(bounds if bounds else [np.nan, np.nan], np.float32)
    out["feature_count"] = np.int64(len(w.features))
    for i, f in enumerate(w.features):
        out[f"f{i}_meta"] = np.array([f.table, f.feature, f.pooling], np.uint32)
        out[f"f{i}_keys"] = f.keys
        out[f"f{i}_offsets"] = f.offsets
    for shards in (1, 2, 3):
        ref = Reference(defs, shards=shards)
        _, outs = ref.lookup(feats(w), read_only=True)
        for i, o in enumerate(outs):
            out[f"lookup_s{shards}_f{i}"] = o
        ref.close()
    ref = Reference(defs, shards=1)
    rng = np.random.Generator(np.random.Philox(99))
    for step in range(steps):
        batch, outs = ref.lookup(feats(w))
        grads = [(rng.normal(0, 1e-2, size=o.shape) * grad_scale).astype(np.float32) for o in outs]
        for i, g in enumerate(grads):
            out[f"grad_step{step}_f{i}"] = g
        ref.push(batch, feats(w), grads)
    for t in w.tables:
        keys = np.unique(np.concatenate([f.keys for f in w.features if f.table == t.id]))
        ws, ms, vs, us = [], [], [], []
        for k in keys:
            a, b, c, u = ref.read(t.id, int(k))
            ws.append(a); ms.append(b); vs.append(c); us.append(u)
        out[f"t{t.id}_keys"] = keys
        out[f"t{t.id}_w"] = np.array(ws, np.float32)
        out[f"t{t.id}_m"] = np.array(ms, np.float32)
        out[f"t{t.id}_v"] = np.array(vs, np.float32)
        out[f"t{t.id}_updates"] = np.array(us, np.uint64)
    out["steps"] = np.int64(steps)
    ref.close()
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
    print(name, "occurrences", w.occurrences, "unique", w.unique())


def main():
    run("small_multi_table", wl.small(11, dims=(2, 32, 64, 128), bags=24, max_bag=9, rows=200))
    run("small_bounded", wl.small(12, dims=(64,), bags=32, max_bag=6, rows=50), lr=0.05,
        bounds=(-0.06, 0.06))
    run("hot_segments", wl.hot(13, dim=16, rows=500, n=3000), steps=2)
    run("cfg1_shape", wl.config1(1), steps=2)


if __name__ == "__main__":
    main()
