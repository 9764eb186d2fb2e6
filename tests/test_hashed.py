"""Hashed tables (key_space == 0): any 64-bit key, a row created on its first
touch with the reference initializer, as the reference's ShardStore::Ensure does
(src/store/shard_store.cpp:76-115, reached from src/access/batch_access.cpp:34
for every lookup, read-only ones included).

Checked against the unmodified reference CPU parameter server (oracle/_ref),
which keeps its rows in a hash map and creates them lazily:
* lookups + pushes with random 64-bit keys (the all-ones key included): pooled
  outputs, the coalesced occurrence lists (eps_b200_ticket_coalesced: each key's
  occurrences, sources and scales in reference order; rows sorted by key, as a
  hashed table's rows come in slot order) and every touched row's w / m / v /
  updates bit-exact, on one shard and as the owner of one of three shards (keys
  of other shards refused);
* a read-only lookup creates the rows it touches (their initial values);
* a table that is full refuses new keys with capacity_exceeded, keeping the
  keys it holds;
* a snapshot of a hashed table restores into a fresh store and into the
  reference, row for row.
"""
import os
import tempfile

import numpy as np
import pytest

import round_check as rc
from oracle_lib import MEAN, SEQUENCE, SUM, Feature, Reference, TableDef, reference_available

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not reference_available(), reason="oracle/_ref not built")]

U64_MAX = (1 << 64) - 1


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def key_pool(rng, n, shards=1, shard=0):
    """n distinct 64-bit keys owned by `shard` of `shards` (the all-ones key
    included when it is owned)."""
    keys = set()
    if U64_MAX % shards == shard:
        keys.add(U64_MAX)
    while len(keys) < n:
        k = int(rng.integers(0, 1 << 63, dtype=np.int64)) * 2 + int(rng.integers(0, 2))
        if k % shards == shard:
            keys.add(k)
    return np.array(sorted(keys), dtype=np.uint64)


def rows_by_key(got):
    """A coalesced CSR with its rows reordered by (table, key)."""
    order = np.lexsort((got["keys"], got["tables"]))
    ro = got["row_offsets"].astype(np.int64)
    idx = (np.concatenate([np.arange(ro[i], ro[i + 1]) for i in order]) if len(order)
           else np.zeros(0, np.int64))
    out = {"tables": got["tables"][order], "keys": got["keys"][order],
           "row_offsets": np.concatenate([[0], np.cumsum(np.diff(ro)[order])]).astype(np.uint64)}
    for k in ("features", "sources", "scales"):
        out[k] = got[k][idx]
    return out


def features(rng, pool, dim, bags=64):
    out = []
    for fid, pooling in enumerate((SUM, MEAN, SEQUENCE)):
        lens = rng.integers(0, 9, size=bags)
        offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.uint64)
        keys = pool[rng.integers(0, len(pool), size=int(offs[-1]))]
        out.append(Feature(1, fid, pooling, keys, offs))
    return out


def table(eps, dim, capacity, shards=1):
    return eps.TableDefinition(id=1, dimension=dim, key_space=0, capacity=capacity,
                               learning_rate=0.01, shard_count=shards)


def ref_table(dim):
    return TableDef(id=1, dimension=dim, learning_rate=0.01, init_min=-0.05, init_max=0.05,
                    init_seed=42)


@pytest.mark.parametrize("dim", [32, 64])
def test_hashed_round_against_reference(eps, dim):
    rng = np.random.default_rng(dim)
    pool = key_pool(rng, 700)
    store = eps.ParameterStore(device=0, state_bytes=1 << 30)
    store.create_table(table(eps, dim, capacity=1000))
    ref = Reference([ref_table(dim)], shards=1)
    for step in range(3):
        feats = features(rng, pool, dim)
        ins = [eps.FeatureInput(f.table, f.feature, f.pooling, f.keys, f.offsets) for f in feats]
        ticket, outs = store.lookup(ins)
        batch, want = ref.lookup(feats)
        for a, b in zip(outs, want):
            assert np.array_equal(bits(a), bits(b)), step
        got = store.coalesced(ticket)
        assert len(got["keys"]) == len(np.unique(np.concatenate([f.keys for f in feats])))
        assert rc.check_coalesced(rows_by_key(got), feats), step
        grads = [rng.normal(0, 0.01, size=o.shape).astype(np.float32) for o in outs]
        store.push(ticket, grads)
        ref.push(batch, feats, grads)
    touched = np.unique(np.concatenate([f.keys for f in feats]))
    w, m, v, u = store.read_state(1, touched)
    rw, rm, rv, ru = ref.read_many(1, touched)
    assert np.array_equal(bits(w), bits(rw)) and np.array_equal(bits(m), bits(rm))
    assert np.array_equal(bits(v), bits(rv)) and np.array_equal(u, ru)
    ref.close()
    store.close()


def test_hashed_owner_shard_and_read_only_creation(eps):
    """Shard 1 of 3 holds the keys k % 3 == 1 of any size; a read-only lookup
    creates rows (their initial values), other shards' keys are refused."""
    rng = np.random.default_rng(7)
    dim = 32
    pool = key_pool(rng, 300, shards=3, shard=1)
    store = eps.ParameterStore(device=0, shard_id=1, shard_count=3, state_bytes=1 << 30)
    store.create_table(table(eps, dim, capacity=400, shards=3))
    ref = Reference([ref_table(dim)], shards=3)
    feats = features(rng, pool, dim)
    ins = [eps.FeatureInput(f.table, f.feature, f.pooling, f.keys, f.offsets) for f in feats]
    _, outs = store.lookup(ins, read_only=True, shard_partial=True)
    batch, _ = ref.lookup(feats, read_only=True)
    ref.release(batch)
    touched = np.unique(np.concatenate([f.keys for f in feats]))
    w, m, v, u = store.read_state(1, touched)
    rw, rm, rv, ru = ref.read_many(1, touched)
    assert np.array_equal(bits(w), bits(rw)) and not m.any() and not v.any() and not u.any()
    bad = np.array([int(pool[0]) + 1], dtype=np.uint64)        # owned by shard 2
    with pytest.raises(eps.EpsError):
        store.lookup([eps.FeatureInput(1, 0, SUM, bad, np.array([0, 1], np.uint64))],
                     read_only=True, shard_partial=True)
    ref.close()
    store.close()


def test_hashed_capacity_is_enforced(eps):
    rng = np.random.default_rng(3)
    pool = key_pool(rng, 40)
    store = eps.ParameterStore(device=0, state_bytes=1 << 28)
    store.create_table(table(eps, 32, capacity=24))
    first = [eps.FeatureInput(1, 0, SUM, pool[:20], np.array([0, 20], np.uint64))]
    store.lookup(first, read_only=True)
    with pytest.raises(eps.EpsError) as e:
        store.lookup([eps.FeatureInput(1, 0, SUM, pool[20:], np.array([0, 20], np.uint64))],
                     read_only=True)
    assert e.value.code == eps.CAPACITY_EXCEEDED
    store.lookup(first, read_only=True)                          # held keys still work
    w, _, _, _ = store.read_state(1, pool[:20])
    assert np.isfinite(w).all()
    store.close()


def test_hashed_snapshot_round_trip(eps):
    rng = np.random.default_rng(11)
    dim = 32
    pool = key_pool(rng, 200)
    store = eps.ParameterStore(device=0, state_bytes=1 << 30)
    store.create_table(table(eps, dim, capacity=300))
    feats = features(rng, pool, dim)
    ins = [eps.FeatureInput(f.table, f.feature, f.pooling, f.keys, f.offsets) for f in feats]
    ticket, outs = store.lookup(ins)
    store.push(ticket, [rng.normal(0, 0.01, size=o.shape).astype(np.float32) for o in outs])
    touched = np.unique(np.concatenate([f.keys for f in feats]))
    want = store.read_state(1, touched)
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "hashed.snap")
        store.snapshot_write(path, "run-a")
        fresh = eps.ParameterStore(device=0, state_bytes=1 << 30)
        fresh.create_table(table(eps, dim, capacity=300))
        fresh.snapshot_read(path, "run-b")
        got = fresh.read_state(1, touched)
        for a, b in zip(got, want):
            assert np.array_equal(np.asarray(a).view(np.uint32), np.asarray(b).view(np.uint32))
        fresh.close()
        # the reference restores the same file (its own snapshot format)
        ref = Reference([ref_table(dim)], shards=1, define=False, run="run-c")
        ref.restore(path)
        rw, rm, rv, ru = ref.read_many(1, touched)
        assert np.array_equal(bits(rw), bits(want[0])) and np.array_equal(bits(rm), bits(want[1]))
        assert np.array_equal(bits(rv), bits(want[2])) and np.array_equal(ru, want[3])
        ref.close()
    store.close()
