"""Snapshots in the reference's checksummed shard format (src/store/snapshot.cpp).

CPU (no GPU needed): the library's host-side reader against files written by the
reference itself (DrainAndFlush of the unmodified CPU core in oracle/_ref) and
against the reference's own format-1 fixture (tests/fixtures/snapshot-v1-
unbounded.bin, read from the reference checkout when it is present).
GPU: a reference snapshot restored into a B200 store, a B200 snapshot restored
by the reference, round trips that continue training identically, and corrupt
files rejected with nothing changed.
"""
from __future__ import annotations

import os
import tempfile

import numpy as np
import pytest

from conftest import import_package
from oracle_lib import SEQUENCE, SUM, MEAN, Feature, Oracle, Reference, TableDef, reference_available

REFERENCE = os.environ.get("EPS_REFERENCE", os.path.join(
    os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))), "reference"))
FIXTURE = os.path.join(REFERENCE, "tests", "fixtures", "snapshot-v1-unbounded.bin")


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def tables():
    return [TableDef(id=3, dimension=8, learning_rate=0.05, init_min=-0.05, init_max=0.05, rows=97,
                     bounds=(-0.08, 0.08)),
            TableDef(id=1, dimension=4, learning_rate=0.1, init_min=0.25, init_max=0.25, rows=31)]


def rounds(step):
    rng = np.random.default_rng(step)
    feats = [Feature(3, 0, SUM, rng.integers(0, 97, size=20).astype(np.uint64),
                     [0, 5, 5, 12, 20]),
             Feature(1, 1, MEAN, rng.integers(0, 31, size=9).astype(np.uint64), [0, 4, 9]),
             Feature(3, 2, SEQUENCE, rng.integers(0, 97, size=6).astype(np.uint64), [0, 3, 6])]
    grads = [rng.normal(0, 0.2, size=(f.output_rows, 8 if f.table == 3 else 4)).astype(np.float32)
             for f in feats]
    return feats, grads


def reference_after(steps, run, snapshot_dir):
    r = Reference(tables(), shards=1, run=run, snapshot_dir=snapshot_dir)
    for step in range(steps):
        feats, grads = rounds(step)
        batch, _ = r.lookup(feats)
        r.push(batch, feats, grads)
    return r


needs_ref = pytest.mark.skipif(not reference_available(), reason="oracle/_ref not built")


@needs_ref
def test_reader_parses_reference_written_snapshot():
    eps = import_package()
    with tempfile.TemporaryDirectory() as d:
        r = reference_after(3, "writer", d)
        path = r.snapshot("s1")
        meta, tabs = eps.snapshot_inspect(path)
        assert meta["format"] == 2 and meta["run"] == "writer"
        assert (meta["shard"], meta["shard_count"], meta["partition_epoch"]) == (0, 1, 1)
        assert [t["id"] for t in tabs] == [1, 3]                 # ascending ids
        for i, t in enumerate(tabs):
            dim = 4 if t["id"] == 1 else 8
            assert t["optimizer_sequence"] == 3
            keys, upd, w, m, v = eps.snapshot_rows(path, i, t["rows"], dim)
            for k, u, a, b, c in zip(keys, upd, w, m, v):
                rw, rm, rv, ru = r.read(t["id"], int(k))
                assert u == ru and np.array_equal(bits(a), bits(rw))
                assert np.array_equal(bits(b), bits(rm)) and np.array_equal(bits(c), bits(rv))
        # a flipped payload byte fails the checksum
        data = bytearray(open(path, "rb").read())
        data[-9] ^= 1
        bad = os.path.join(d, "bad.bin")
        open(bad, "wb").write(bytes(data))
        with pytest.raises(eps.EpsError):
            eps.snapshot_inspect(bad)
        r.close()


@pytest.mark.skipif(not os.path.exists(FIXTURE), reason="reference checkout not present")
def test_reader_parses_reference_format1_fixture():
    """tests/fixtures/README.md of the reference: run legacy-unbounded, shard 0 of 1,
    epoch 1, table 1 (dim 2, lr 0.1, constant init 0.25, seed 42, unbounded), key 1
    with weights [0.25, 0.25], zero moments and zero updates."""
    eps = import_package()
    meta, tabs = eps.snapshot_inspect(FIXTURE)
    assert meta["format"] == 1 and meta["run"] == "legacy-unbounded"
    assert (meta["shard"], meta["shard_count"], meta["partition_epoch"]) == (0, 1, 1)
    assert len(tabs) == 1 and tabs[0]["id"] == 1 and tabs[0]["dimension"] == 2
    assert tabs[0]["has_weight_bounds"] == 0 and tabs[0]["learning_rate"] == float(np.float32(0.1))
    assert tabs[0]["initialization_seed"] == 42 and tabs[0]["optimizer_sequence"] == 0
    keys, upd, w, m, v = eps.snapshot_rows(FIXTURE, 0, tabs[0]["rows"], 2)
    assert list(keys) == [1] and list(upd) == [0]
    assert w.tolist() == [[0.25, 0.25]] and not m.any() and not v.any()


def _store(eps):
    s = eps.ParameterStore(device=0, state_bytes=1 << 30)
    for t in tables():
        s.create_table(eps.TableDefinition(
            id=t.id, dimension=t.dimension, key_space=t.rows, learning_rate=t.learning_rate,
            weight_bounds=t.bounds, initialization_min=t.init_min, initialization_max=t.init_max,
            initialization_seed=t.init_seed))
    return s


def _train(s, start, steps):
    eps = import_package()
    for step in range(start, start + steps):
        feats, grads = rounds(step)
        ticket, _ = s.lookup([eps.FeatureInput(f.table, f.feature, f.pooling, f.keys, f.offsets)
                              for f in feats])
        s.push(ticket, grads)


def _same_as_reference(s, r):
    """Every row the reference holds matches bit for bit; rows it never created
    hold their initial value and no updates in the B200 store."""
    init = Oracle(tables())
    for t in tables():
        keys = np.arange(t.rows, dtype=np.uint64)
        w, m, v, u = s.read_state(t.id, keys)
        st0, _ = init.state(t.id)
        for k in range(t.rows):
            try:
                rw, rm, rv, ru = r.read(t.id, k)
            except ValueError:                         # "unknown parameter row"
                assert u[k] == 0 and np.array_equal(bits(w[k]), bits(st0[k, 0]))
                assert not m[k].any() and not v[k].any()
                continue
            assert np.array_equal(bits(w[k]), bits(rw)) and np.array_equal(bits(m[k]), bits(rm))
            assert np.array_equal(bits(v[k]), bits(rv)) and u[k] == ru


@pytest.mark.gpu
@needs_ref
def test_snapshots_cross_restore_with_the_reference():
    eps = import_package()
    with tempfile.TemporaryDirectory() as d:
        # the reference's snapshot restored into a B200 store
        r = reference_after(3, "writer", d)
        path = r.snapshot("s1")
        s = _store(eps)
        with pytest.raises(eps.EpsError):
            s.snapshot_read(path, "writer")                # a restore needs a new run
        s.snapshot_read(path, "resumed")
        _same_as_reference(s, r)
        assert s.optimizer_state(3)[0] == 3
        # training continues identically from the restored state
        r2 = Reference(tables(), shards=1, run="resumed-ref", snapshot_dir=d, define=False)
        r2.restore(path)
        r2.define()                                        # the client learns the tables
        _train(s, 3, 2)
        for step in range(3, 5):
            feats, grads = rounds(step)
            batch, _ = r2.lookup(feats)
            r2.push(batch, feats, grads)
        _same_as_reference(s, r2)
        # the B200 store's snapshot restored by the reference
        mine = os.path.join(d, "b200.bin")
        s.snapshot_write(mine, "b200-run")
        with pytest.raises(eps.EpsError):
            s.snapshot_write(mine, "b200-run")             # never overwrites
        r3 = Reference(tables(), shards=1, run="third", snapshot_dir=d, define=False)
        r3.restore(mine)
        r3.define()
        _same_as_reference(s, r3)
        # round trip into a fresh store; a corrupt file changes nothing
        s2 = _store(eps)
        s2.snapshot_read(mine, "fourth")
        for t in tables():
            a = s.read_state(t.id, np.arange(t.rows, dtype=np.uint64))
            b = s2.read_state(t.id, np.arange(t.rows, dtype=np.uint64))
            assert all(np.array_equal(x.view(np.uint32) if x.dtype == np.float32 else x,
                                      y.view(np.uint32) if y.dtype == np.float32 else y)
                       for x, y in zip(a, b))
        data = bytearray(open(mine, "rb").read())
        data[100] ^= 1
        bad = os.path.join(d, "bad.bin")
        open(bad, "wb").write(bytes(data))
        before = s2.read_state(3, np.arange(97, dtype=np.uint64))
        with pytest.raises(eps.EpsError):
            s2.snapshot_read(bad, "fifth")
        after = s2.read_state(3, np.arange(97, dtype=np.uint64))
        assert np.array_equal(before[0].view(np.uint32), after[0].view(np.uint32))
        for x in (r, r2, r3):
            x.close()
        s.close()
        s2.close()
