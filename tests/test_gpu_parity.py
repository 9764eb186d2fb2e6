"""GPU parity: the CUDA path (through the C ABI) against the reference's golden
vectors and the CPU oracle, on the same seeded inputs.

Bars (fp32):
* lookup outputs (sum, mean, sequence; 1-shard client merge and 2-shard partials):
  bit-exact;
* coalescing + LazyAdam with the reference summation order flag: w, m, v and
  row_updates bit-exact, beta powers and optimizer sequence exact;
* default order: rows with at most 64 occurrences per push bit-exact; the reduced
  gradient of longer rows (summed in parallel pieces) within
  |g - g_exact| <= 1e-6 * sum|terms| (test_long_rows_condition_aware);
* a rejected push leaves every row, counter and beta power unchanged.
"""
import numpy as np
import pytest

import golden_cases
from oracle_lib import MEAN, SEQUENCE, SUM, Feature, Oracle, TableDef

pytestmark = pytest.mark.gpu

F32 = np.float32


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def make_store(eps, tables, reference_order=False, shard_count=1, shard_id=0, register_rows=False):
    s = eps.ParameterStore(device=0, reference_order=reference_order, shard_count=shard_count,
                           shard_id=shard_id, state_bytes=8 << 30, register_rows=register_rows)
    for t in tables:
        s.create_table(eps.TableDefinition(
            id=t.id, dimension=t.dimension, key_space=t.rows, learning_rate=t.learning_rate,
            beta1=t.beta1, beta2=t.beta2, epsilon=t.epsilon,
            initial_beta1_power=t.initial_beta1_power, initial_beta2_power=t.initial_beta2_power,
            weight_bounds=t.bounds, initialization_min=t.init_min, initialization_max=t.init_max,
            initialization_seed=t.init_seed, shard_count=shard_count))
    return s


def inputs(eps, feats):
    return [eps.FeatureInput(f.table, f.feature, f.pooling, f.keys, f.offsets) for f in feats]


def occurrence_counts(feats, table):
    ks = [f.keys for f in feats if f.table == table]
    if not ks:
        return {}
    u, c = np.unique(np.concatenate(ks), return_counts=True)
    return dict(zip(u.tolist(), c.tolist()))


# ----------------------------------------------------------------- golden
@pytest.mark.parametrize("name", golden_cases.CASES)
def test_lookup_bit_exact_vs_reference(eps, name):
    case = golden_cases.load(name)
    s = make_store(eps, case.tables)
    _, outs = s.lookup(inputs(eps, case.features), read_only=True)
    for got, want in zip(outs, case.lookup[1]):
        assert got.shape == want.shape
        assert np.array_equal(bits(got), bits(want)), name


@pytest.mark.parametrize("register_rows", [False, True])
@pytest.mark.parametrize("reference_order", [True, False])
@pytest.mark.parametrize("name", golden_cases.CASES)
def test_push_vs_reference(eps, name, reference_order, register_rows):
    case = golden_cases.load(name)
    s = make_store(eps, case.tables, reference_order=reference_order, register_rows=register_rows)
    for step in range(case.steps):
        ticket, outs = s.lookup(inputs(eps, case.features))
        s.push(ticket, case.grads[step])
    for t in case.tables:
        keys, w, m, v, upd = case.state[t.id]
        gw, gm, gv, gu = s.read_state(t.id, keys)
        assert np.array_equal(gu, upd)
        counts = occurrence_counts(case.features, t.id)
        short = np.array([counts[int(k)] <= 64 for k in keys])
        if reference_order:
            short[:] = True
        for got, want in ((gw, w), (gm, m), (gv, v)):
            # rows with > 64 occurrences are covered by test_long_rows_condition_aware
            assert np.array_equal(bits(got[short]), bits(want[short])), name
        seq, b1p, b2p = s.optimizer_state(t.id)
        assert seq == case.steps
        e1, e2 = F32(0.9), F32(0.999)
        for _ in range(case.steps):
            e1, e2 = F32(e1 * F32(0.9)), F32(e2 * F32(0.999))
        assert F32(b1p) == e1 and F32(b2p) == e2
    s.close()


@pytest.mark.parametrize("reference_order", [False, True])
def test_long_rows_condition_aware(eps, workloads, reference_order):
    """Rows coalesced from many occurrences (Zipf heads): the reduced gradient of
    every row, recovered from m = (1-b1)*g after one push from m = 0, is within
    |g - g_exact| <= 1e-6 * sum|terms| (+ 2 ulp of the recovery) of the float64
    sum of the same terms."""
    w = workloads.hot(31, dim=64, rows=700, n=40000)
    t = [TableDef(id=1, dimension=64, learning_rate=1e-3, rows=700)]
    s = make_store(eps, t, reference_order=reference_order)
    feats = [Feature(f.table, f.feature, f.pooling, f.keys, f.offsets) for f in w.features]
    ticket, _ = s.lookup(inputs(eps, feats))
    s.push(ticket, w.gradients)
    g64 = {}
    a64 = {}
    for f, g in zip(w.features, w.gradients):
        for b in range(len(f.offsets) - 1):
            lo, hi = int(f.offsets[b]), int(f.offsets[b + 1])
            sc = F32(1) / F32(hi - lo) if f.pooling == MEAN and hi > lo else F32(1)
            for i in range(lo, hi):
                row = (g[i] if f.pooling == SEQUENCE else g[b]) * sc   # float32 product, as the kernel
                k = int(f.keys[i])
                g64[k] = g64.get(k, 0.0) + row.astype(np.float64)
                a64[k] = a64.get(k, 0.0) + np.abs(row.astype(np.float64))
    counts = occurrence_counts(feats, 1)
    long_keys = np.array(sorted(k for k, c in counts.items() if c > 64), np.uint64)
    assert len(long_keys) >= 5 and max(counts.values()) > 64 * 20
    _, m, _, upd = s.read_state(1, long_keys)
    assert (upd == 1).all()
    omb1 = np.float64(F32(1) - F32(0.9))
    worst = 0.0
    for i, k in enumerate(long_keys.tolist()):
        g_gpu = m[i].astype(np.float64) / omb1
        bound = 1e-6 * a64[k] + 4 * np.finfo(F32).eps * np.abs(g64[k]) + 1e-30
        err = np.abs(g_gpu - g64[k])
        worst = max(worst, float((err / (a64[k] + 1e-30)).max()))
        assert (err <= bound).all(), (k, counts[k], err.max())
    print(f"long rows: {len(long_keys)}, max normalised error {worst:.3e}")


@pytest.mark.parametrize("register_rows", [False, True])
@pytest.mark.parametrize("reference_order", [False, True])
def test_checked_mode_applies_large_finite_gradients(eps, workloads, reference_order, register_rows):
    """Gradients too large for the single-pass overflow proof (3 * N * max|g| >
    1e17) take the validate-then-apply path (stages A and B validate, stage C
    applies); every finite update must still equal the oracle's: rows with at
    most 64 occurrences bit-exact (every row in reference order), counters and
    beta powers advanced once."""
    w = workloads.hot(37, dim=64, rows=700, n=20000)
    t = [TableDef(id=1, dimension=64, learning_rate=1e-3, rows=700)]
    s = make_store(eps, t, reference_order=reference_order, register_rows=register_rows)
    o = Oracle(t)
    feats = [Feature(f.table, f.feature, f.pooling, f.keys, f.offsets) for f in w.features]
    grads = [np.ascontiguousarray(g * F32(1e15), F32) for g in w.gradients]
    assert 3 * sum(len(f.keys) for f in feats) * max(float(np.abs(g).max()) for g in grads) > 1e17
    ticket, _ = s.lookup(inputs(eps, feats))
    s.push(ticket, grads)
    assert o.push(feats, grads) == 0
    counts = occurrence_counts(feats, 1)
    keys = np.array(sorted(k for k, c in counts.items() if reference_order or c <= 64), np.uint64)
    assert len(keys) > 100
    gw, gm, gv, gu = s.read_state(1, keys)
    st, upd = o.state(1)
    k = keys.astype(np.int64)
    assert np.isfinite(gv).all() and float(gv.max()) > 1e20
    for got, want in ((gw, st[k, 0]), (gm, st[k, 1]), (gv, st[k, 2])):
        assert np.array_equal(bits(got), bits(want))
    assert np.array_equal(gu, upd[k])
    assert s.optimizer_state(1) == (1, F32(F32(0.9) * F32(0.9)), F32(F32(0.999) * F32(0.999)))
    s.close()


@pytest.mark.parametrize("register_rows", [False, True])
@pytest.mark.parametrize("dim,tables", [(32, 45), (128, 3)])
def test_many_tables_one_dimension(eps, workloads, dim, tables, register_rows):
    """Pushes whose tables share one dimension in {32, 64, 128} take the ring row
    updates and the uniform piece sums (register_rows=False); with more than 32
    tables and 128 features those kernels read the table and feature
    descriptors from global memory instead of shared memory.  Two rounds must
    equal the oracle bit for bit for every row with at most 64 occurrences per
    push (and the first round's pooled outputs), counters and beta powers
    exactly."""
    w = workloads.small(11 + dim, dims=(dim,) * tables, bags=24, max_bag=10, rows=40)
    defs = [TableDef(id=x.id, dimension=x.dimension, learning_rate=1e-2, rows=x.rows) for x in w.tables]
    s = make_store(eps, defs, register_rows=register_rows)
    o = Oracle(defs)
    feats = [Feature(f.table, f.feature, f.pooling, f.keys, f.offsets) for f in w.features]
    assert len(feats) > 128 or tables <= 32
    for step in range(2):
        ticket, outs = s.lookup(inputs(eps, feats))
        want = o.lookup(feats)
        if step == 0:
            # pooled outputs are bit-exact until a row with > 64 occurrences has
            # been updated (its piece tree differs from the serial sum in the
            # last bits); the second round's bags may read such rows
            for got, ref in zip(outs, want):
                assert np.array_equal(bits(got), bits(ref))
        s.push(ticket, w.gradients)
        assert o.push(feats, w.gradients) == 0
    long_seen = 0
    for x in w.tables:
        counts = occurrence_counts(feats, x.id)
        keys = np.array(sorted(counts), np.uint64)
        gw, gm, gv, gu = s.read_state(x.id, keys)
        st, upd = o.state(x.id)
        k = keys.astype(np.int64)
        short = np.array([counts[int(q)] <= 64 for q in keys])
        long_seen += int((~short).sum())
        for got, want in ((gw, st[k, 0]), (gm, st[k, 1]), (gv, st[k, 2])):
            assert np.array_equal(bits(got[short]), bits(want[short])), x.id
        assert np.array_equal(gu, upd[k])
        assert s.optimizer_state(x.id)[0] == 2
    if dim == 128:
        assert long_seen > 0           # the long-row path ran too
    s.close()


def test_shard_partials_merge_bit_exact(eps):
    """Two shard stores (key % 2) return the ParameterService::Lookup partials; merged
    in shard order and divided once for mean they equal the reference's 2-shard
    DistributedClient output bit for bit."""
    case = golden_cases.load("small_multi_table")
    stores = [make_store(eps, case.tables, shard_count=2, shard_id=i) for i in range(2)]
    parts = []
    for sid, st in enumerate(stores):
        feats, positions = [], []
        for f in case.features:
            mask = (f.keys % 2) == sid
            keys = f.keys[mask]
            bag = np.repeat(np.arange(len(f.offsets) - 1), np.diff(f.offsets).astype(np.int64))
            counts = np.bincount(bag[mask], minlength=len(f.offsets) - 1)
            offs = np.zeros(len(f.offsets), np.uint64)
            np.cumsum(counts, out=offs[1:])
            lens = np.diff(f.offsets).astype(np.uint64)
            feats.append(eps.FeatureInput(f.table, f.feature, f.pooling, keys, offs, lens))
            positions.append(np.nonzero(mask)[0])
        _, outs = st.lookup(feats, read_only=True, shard_partial=True)
        parts.append((outs, positions))
    for fi, f in enumerate(case.features):
        d = outs[fi].shape[1]
        out = np.zeros((f.output_rows, d), F32)
        for outs_s, pos in parts:
            if f.pooling == SEQUENCE:
                out[pos[fi]] = outs_s[fi]
            else:
                out += outs_s[fi]
        if f.pooling == MEAN:
            lens = np.diff(f.offsets).astype(np.int64)
            nz = lens > 0
            out[nz] = out[nz] / lens[nz, None].astype(F32)
        assert np.array_equal(bits(out), bits(case.lookup[2][fi]))
    for st in stores:
        st.close()


# -------------------------------------------------------------- known answers
def kat_tables():
    return [TableDef(id=1, dimension=2, learning_rate=0.1, init_min=0.25, init_max=0.25, rows=8)]


def test_pooling_and_update_kat(eps):
    # tests/core_tests.cpp:68-85 of the reference
    s = make_store(eps, kat_tables())
    o = Oracle(kat_tables())
    feats = [Feature(1, 0, SUM, [1, 1, 2], [0, 3, 3]), Feature(1, 1, MEAN, [1, 3], [0, 2])]
    ticket, outs = s.lookup(inputs(eps, feats))
    assert abs(outs[0][0, 0] - 0.75) < 1e-5 and outs[0][1, 0] == 0
    assert abs(outs[1][0, 0] - 0.25) < 1e-5
    grads = [np.array([[1, 2], [0, 0]], F32), np.array([[4, 6]], F32)]
    s.push(ticket, grads)
    assert o.push(feats, grads) == 0
    w, m, v, u = s.read_state(1, [1, 2, 3])
    st, upd = o.state(1)
    assert np.array_equal(bits(w), bits(st[[1, 2, 3], 0])) and np.array_equal(bits(m), bits(st[[1, 2, 3], 1]))
    assert np.array_equal(bits(v), bits(st[[1, 2, 3], 2])) and list(u) == [1, 1, 1]
    assert abs(m[0, 0] - 0.4) < 1e-5 and abs(v[0, 1] - 0.049) < 1e-5 and abs(w[0, 0] - 0.15) < 1e-5
    # a repeated Push of the same ticket is acknowledged without effect
    s.push(ticket, grads)
    assert s.read_state(1, [1])[3][0] == 1
    assert s.stats()["duplicate_requests"] == 1


def test_bounded_closed_form(eps):
    # tests/weight_bounds_tests.cpp:28-43 of the reference, checked against the oracle
    t = [TableDef(id=1, dimension=2, learning_rate=1.0, init_min=0.5, init_max=0.5,
                  bounds=(-0.1, 0.2), rows=8)]
    s, o = make_store(eps, t), Oracle(t)
    f = [Feature(1, 0, SEQUENCE, [1], [0, 1])]
    for seq in range(1, 7):
        g = [np.full((1, 2), 10 if seq <= 2 else -10, F32)]
        ticket, outs = s.lookup(inputs(eps, f))
        assert np.array_equal(bits(outs[0]), bits(o.lookup(f)[0]))
        s.push(ticket, g)
        assert o.push(f, g) == 0
        w, m, v, _ = s.read_state(1, [1])
        st, _ = o.state(1)
        assert np.array_equal(bits(w[0]), bits(st[1, 0])) and np.array_equal(bits(v[0]), bits(st[1, 2]))


def test_rejected_push_leaves_state_unchanged_and_is_retryable(eps):
    # tests/core_tests.cpp:98-105 and :214-222 of the reference
    s = make_store(eps, kat_tables())
    f = [Feature(1, 0, SEQUENCE, [1, 2], [0, 2])]
    ticket, _ = s.lookup(inputs(eps, f))
    before = s.read_state(1, [1, 2])
    bad = np.array([[1, 1], [np.finfo(F32).max, 1]], F32)
    with pytest.raises(eps.EpsError) as e:
        s.push(ticket, [bad])
    assert e.value.code == eps.INVALID_ARGUMENT and "overflow" in e.value.message
    after = s.read_state(1, [1, 2])
    for a, b in zip(before, after):
        assert np.array_equal(np.asarray(a).view(np.uint32) if a.dtype == F32 else a,
                              np.asarray(b).view(np.uint32) if b.dtype == F32 else b)
    assert s.optimizer_state(1) == (0, F32(0.9), F32(0.999))
    with pytest.raises(eps.EpsError) as e:
        s.push(ticket, [np.array([[np.nan, 0], [0, 0]], F32)])
    assert "non-finite" in e.value.message
    with pytest.raises(eps.EpsError):
        s.push(ticket, [np.zeros((3, 2), F32)])             # layout mismatch
    good = np.array([[1, 2], [3, 4]], F32)
    s.push(ticket, [good])                                    # same ticket, retried
    o = Oracle(kat_tables())
    assert o.push(f, [good]) == 0
    w, m, v, u = s.read_state(1, [1, 2])
    st, _ = o.state(1)
    assert np.array_equal(bits(w), bits(st[[1, 2], 0])) and list(u) == [1, 1]


def test_release_and_unknown_ticket(eps):
    s = make_store(eps, kat_tables())
    f = [Feature(1, 0, SUM, [1, 2], [0, 2])]
    ticket, _ = s.lookup(inputs(eps, f))
    assert s.stats()["live_tickets"] == 1
    s.release(ticket)
    assert s.stats()["live_tickets"] == 0
    with pytest.raises(eps.EpsError):
        s.push(ticket, [np.zeros((1, 2), F32)])


def test_invalid_host_inputs_are_rejected(eps):
    s = make_store(eps, kat_tables())
    with pytest.raises(eps.EpsError):                        # key outside the table
        s.lookup([eps.FeatureInput(1, 0, SUM, np.array([9], np.uint64), np.array([0, 1], np.uint64))])
    with pytest.raises(eps.EpsError):                        # decreasing offsets
        s.lookup([eps.FeatureInput(1, 0, SUM, np.array([1, 2], np.uint64),
                                   np.array([0, 2, 1, 2], np.uint64))])
    with pytest.raises(eps.EpsError):                        # offsets not ending at key count
        s.lookup([eps.FeatureInput(1, 0, SUM, np.array([1, 2], np.uint64), np.array([0, 1], np.uint64))])
    with pytest.raises(eps.EpsError):                        # unknown table
        s.lookup([eps.FeatureInput(7, 0, SUM, np.array([1], np.uint64), np.array([0, 1], np.uint64))])
    with pytest.raises(eps.EpsError):                        # duplicate feature id
        f = eps.FeatureInput(1, 0, SUM, np.array([1], np.uint64), np.array([0, 1], np.uint64))
        s.lookup([f, f])
    assert s.stats()["live_tickets"] == 0


def _drop_padding(f, pad):
    """Host restatement of PrepareAdapterInput (src/access/prepare_queue.cpp:69-77):
    the compacted feature and, for sequence, the kept positions."""
    keys, offs = [], [0]
    positions = []
    for b in range(len(f.offsets) - 1):
        for i in range(int(f.offsets[b]), int(f.offsets[b + 1])):
            if int(f.keys[i]) != pad:
                keys.append(int(f.keys[i]))
                positions.append(i)
        offs.append(len(keys))
    return Feature(f.table, f.feature, f.pooling, np.array(keys, np.uint64), offs), positions


def test_padding_keys_are_dropped(eps):
    """Adapter padding (EpsFeature::has_padding): padding keys contribute no row and
    no gradient, mean divides by the kept count, sequence positions read 0."""
    t = [TableDef(id=1, dimension=32, learning_rate=0.01, init_min=-0.05, init_max=0.05, rows=200)]
    pad = 197                                   # a key inside the table: must be skipped
    rng = np.random.default_rng(11)
    feats = []
    for fi, pool in enumerate([SUM, MEAN, SEQUENCE, MEAN]):
        lens = rng.integers(0, 7, size=40)
        offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.uint64)
        keys = rng.integers(0, 200, size=int(offs[-1])).astype(np.uint64)
        keys[rng.random(len(keys)) < 0.3] = pad
        if len(lens) > 3 and lens[3]:
            keys[int(offs[3]):int(offs[4])] = pad      # a bag of padding only
        feats.append(Feature(1, fi, pool, keys, offs))
    s, o = make_store(eps, t), Oracle(t)
    ins = [eps.FeatureInput(f.table, f.feature, f.pooling, f.keys, f.offsets, padding_key=pad)
           for f in feats]
    ticket, outs = s.lookup(ins)
    compact = [_drop_padding(f, pad) for f in feats]
    ref = o.lookup([c for c, _ in compact])
    for f, (c, pos), a, r in zip(feats, compact, outs, ref):
        if f.pooling == SEQUENCE:
            want = np.zeros_like(a)
            want[pos] = r
        else:
            want = r
        assert np.array_equal(bits(a), bits(want)), f.feature
    grads = [rng.normal(0, 0.01, size=a.shape).astype(F32) for a in outs]
    s.push(ticket, grads)
    cgrads = [g[pos] if f.pooling == SEQUENCE else g for f, (c, pos), g in zip(feats, compact, grads)]
    assert o.push([c for c, _ in compact], cgrads) == 0
    keys = np.arange(200, dtype=np.uint64)
    w, m, v, u = s.read_state(1, keys)
    st, upd = o.state(1)
    assert np.array_equal(bits(w), bits(st[:, 0])) and np.array_equal(bits(m), bits(st[:, 1]))
    assert np.array_equal(bits(v), bits(st[:, 2])) and np.array_equal(u, upd)
    assert u[pad] == 0                           # the padding key's row was never touched
    with pytest.raises(eps.EpsError):           # padding derives the lengths itself
        s.lookup([eps.FeatureInput(1, 0, SUM, feats[0].keys, feats[0].offsets,
                                   valid_lengths=np.diff(feats[0].offsets), padding_key=pad)])


def test_empty_and_ragged_features(eps):
    t = [TableDef(id=1, dimension=64, learning_rate=0.01, rows=100)]
    s, o = make_store(eps, t), Oracle(t)
    feats = [Feature(1, 0, SUM, np.array([], np.uint64), [0]),            # no bags
             Feature(1, 1, MEAN, np.array([], np.uint64), [0, 0, 0]),     # empty bags
             Feature(1, 2, SEQUENCE, np.array([5], np.uint64), [0, 0, 1, 1]),
             Feature(1, 3, SUM, np.array([5, 5, 7], np.uint64), [0, 0, 3])]
    ticket, outs = s.lookup(inputs(eps, feats))
    for a, b in zip(outs, o.lookup(feats)):
        assert a.shape == b.shape and np.array_equal(bits(a), bits(b))
    rng = np.random.default_rng(0)
    grads = [rng.normal(0, 0.01, size=x.shape).astype(F32) for x in outs]
    s.push(ticket, grads)
    assert o.push(feats, grads) == 0
    w, m, v, u = s.read_state(1, [5, 7])
    st, upd = o.state(1)
    assert np.array_equal(bits(w), bits(st[[5, 7], 0])) and np.array_equal(u, upd[[5, 7]])


def test_device_inputs_async_push_matches_host_path(eps):
    torch = pytest.importorskip("torch")
    case = golden_cases.load("hot_segments")
    host, dev = make_store(eps, case.tables), make_store(eps, case.tables)
    for step in range(case.steps):
        t1, o1 = host.lookup(inputs(eps, case.features))
        dfeats = [eps.FeatureInput(f.table, f.feature, f.pooling,
                                   torch.from_numpy(f.keys.astype(np.int64)).cuda(),
                                   torch.from_numpy(f.offsets.astype(np.int64)).cuda())
                  for f in case.features]
        t2, o2 = dev.lookup(dfeats)
        for a, b in zip(o1, o2):
            assert np.array_equal(bits(a), bits(b.cpu().numpy()))
        host.push(t1, case.grads[step])
        dev.push(t2, [torch.from_numpy(g).cuda() for g in case.grads[step]], wait=False)
    dev.synchronize()
    keys = case.state[1][0]
    for a, b in zip(host.read_state(1, keys), dev.read_state(1, keys)):
        assert np.array_equal(a.view(np.uint32) if a.dtype == F32 else a,
                              b.view(np.uint32) if b.dtype == F32 else b)


def test_device_input_errors_are_deferred(eps):
    torch = pytest.importorskip("torch")
    s = make_store(eps, kat_tables())
    before = s.read_state(1, [1])
    f = [eps.FeatureInput(1, 0, SUM, torch.tensor([1, 99], device="cuda"),
                          torch.tensor([0, 2], device="cuda"))]
    ticket, _ = s.lookup(f)
    with pytest.raises(eps.EpsError) as e:
        s.push(ticket, [torch.zeros((1, 2), device="cuda")])
    assert "wrong shard or outside" in e.value.message
    after = s.read_state(1, [1])
    assert np.array_equal(before[0], after[0]) and s.stats()["live_tickets"] == 0


def test_two_live_tickets_any_order(eps):
    # reference summation order: this batch has a row with > 64 occurrences
    case = golden_cases.load("small_bounded")
    s = make_store(eps, case.tables, reference_order=True)
    o = Oracle(case.tables)
    t1, _ = s.lookup(inputs(eps, case.features))
    t2, _ = s.lookup(inputs(eps, case.features))
    s.push(t2, case.grads[0])
    s.push(t1, case.grads[1])
    assert o.push(case.features, case.grads[0]) == 0
    assert o.push(case.features, case.grads[1]) == 0
    keys = case.state[1][0]
    w, m, v, u = s.read_state(1, keys)
    st, upd = o.state(1)
    k = keys.astype(np.int64)
    assert np.array_equal(bits(w), bits(st[k, 0])) and np.array_equal(u, upd[k])


def test_sync_reduce_known_answers_and_oracle(eps):
    """SynchronousGradientCollector::Reduce on the device: the reference's known
    answers (tests/synchronous_gradients_tests.cpp:37-50), bit-exact agreement
    with the oracle on a larger round, input rejection, and the reduced rows
    applied like the reference's synchronous applier."""
    import torch
    dev = "cuda:0"
    t2 = [TableDef(id=1, dimension=2, rows=8)]
    s = make_store(eps, t2)
    W = [(torch.tensor([1, 4], device=dev), torch.tensor([[3., 6.], [9., 12.]], device=dev), 1),
         (torch.tensor([1, 2], device=dev), torch.tensor([[6., 9.], [12., 15.]], device=dev), 3),
         (torch.empty(0, dtype=torch.int64, device=dev), torch.empty((0, 2), device=dev), 2)]
    expected = {0: [9, 15, 12, 15, 9, 12], 1: [3, 5, 4, 5, 3, 4], 2: [3.5, 5.5, 6, 7.5, 1.5, 2]}
    for reduction, want in expected.items():
        keys, values = s.sync_reduce(1, W, reduction)
        assert keys.cpu().tolist() == [1, 2, 4]
        assert values.cpu().reshape(-1).tolist() == want
    # a larger round against the oracle (sample_mean, 7 workers, overlapping keys)
    t = [TableDef(id=1, dimension=48, learning_rate=0.01, init_min=-0.05, init_max=0.05, rows=5000)]
    s, o = make_store(eps, t), Oracle(t)
    rng = np.random.default_rng(5)
    workers = []
    for w in range(7):
        k = np.unique(rng.integers(0, 5000, size=int(rng.integers(0, 900)))).astype(np.uint64)
        v = rng.normal(0, 0.01, size=(len(k), 48)).astype(F32)
        workers.append((k, v, int(rng.integers(1, 50))))
    for reduction in (0, 1, 2):
        ok, ov = o.sync_reduce(48, workers, reduction)
        dk, dv = s.sync_reduce(1, [(torch.from_numpy(k.astype(np.int64)).to(dev),
                                    torch.from_numpy(v).to(dev), c) for k, v, c in workers],
                               reduction)
        assert np.array_equal(dk.cpu().numpy().astype(np.uint64), ok)
        assert np.array_equal(bits(dv.cpu().numpy()), bits(ov))
    # the reduced rows applied as one sequence lookup + push, as the reference applier does
    s.apply_reduced(1, dk, dv)
    feat = Feature(1, 0, SEQUENCE, ok, [0, len(ok)])
    o.lookup([feat])
    assert o.push([feat], [ov]) == 0
    w_, m_, v_, u_ = s.read_state(1, np.arange(5000, dtype=np.uint64))
    st, upd = o.state(1)
    assert np.array_equal(bits(w_), bits(st[:, 0])) and np.array_equal(bits(v_), bits(st[:, 2]))
    assert np.array_equal(u_, upd)
    # rejected inputs: unsorted keys, non-finite values
    bad = [(torch.tensor([3, 1], device=dev), torch.zeros((2, 48), device=dev), 1)]
    with pytest.raises(eps.EpsError):
        s.sync_reduce(1, bad, 0)
    nan = torch.zeros((1, 48), device=dev)
    nan[0, 5] = float("nan")
    with pytest.raises(eps.EpsError):
        s.sync_reduce(1, [(torch.tensor([7], device=dev), nan, 1)], 0)


def test_agent_apply_rows_and_compact(eps):
    """The GpuCacheAgent device contract: ApplyHost with an external optimizer
    context and ApplyCompact (CSR expanded in reference order), against the oracle;
    the table's own powers do not advance; rejections leave the state unchanged."""
    import torch
    t = [TableDef(id=1, dimension=40, learning_rate=0.02, init_min=-0.05, init_max=0.05, rows=600,
                  bounds=(-0.06, 0.06))]
    s, o = make_store(eps, t), Oracle(t)
    rng = np.random.default_rng(9)
    before = s.optimizer_state(1)
    ctx = (0.03, 0.5, 0.7)                       # lr, beta1_power, beta2_power of the caller
    keys = rng.choice(600, size=250, replace=False).astype(np.uint64)
    vals = rng.normal(0, 0.5, size=(250, 40)).astype(F32)
    s.apply_rows(1, keys, vals, *ctx)
    assert o.apply_host(1, *ctx, keys, vals) == 0
    # device values, another context
    keys2 = rng.choice(600, size=100, replace=False).astype(np.uint64)
    vals2 = rng.normal(0, 0.5, size=(100, 40)).astype(F32)
    s.apply_rows(1, keys2, torch.from_numpy(vals2).cuda(), 0.01, 0.81, 0.998)
    assert o.apply_host(1, 0.01, 0.81, 0.998, keys2, vals2) == 0
    # compact: 80 target rows referencing 30 source rows with scales
    tk = rng.choice(600, size=80, replace=False).astype(np.uint64)
    src = rng.normal(0, 0.3, size=(30, 40)).astype(F32)
    counts = rng.integers(0, 6, size=80)
    offs = np.concatenate([[0], np.cumsum(counts)]).astype(np.uint64)
    srows = rng.integers(0, 30, size=int(offs[-1])).astype(np.uint64)
    scales = rng.choice([1.0, 0.5, 1.0 / 3.0, 0.125], size=int(offs[-1])).astype(F32)
    s.apply_compact(1, tk, src, offs, srows, scales, *ctx)
    rc, expanded = o.expand_compact(40, 80, src, offs, srows, scales)
    assert rc == 0 and o.apply_host(1, *ctx, tk, expanded) == 0
    allk = np.arange(600, dtype=np.uint64)
    w, m, v, u = s.read_state(1, allk)
    st, upd = o.state(1)
    assert np.array_equal(bits(w), bits(st[:, 0])) and np.array_equal(bits(m), bits(st[:, 1]))
    assert np.array_equal(bits(v), bits(st[:, 2])) and np.array_equal(u, upd)
    assert s.optimizer_state(1) == before             # agents do not advance the powers
    # rejections: non-finite value, duplicate row, bad context; nothing changes
    bad = vals.copy()
    bad[3, 7] = np.inf
    for args in [(keys, bad, *ctx), (np.array([5, 5], np.uint64), vals[:2], *ctx),
                 (keys, vals, 0.03, 1.0, 0.7)]:
        with pytest.raises(eps.EpsError):
            s.apply_rows(1, *args)
    w2, m2, v2, u2 = s.read_state(1, allk)
    assert np.array_equal(bits(w2), bits(w)) and np.array_equal(u2, u)
