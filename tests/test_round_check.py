"""The full-round checker (tests/round_check.py) on CPU.

The C restatement (oracle/eps_oracle.c, which sums every row serially in
occurrence order like the reference) stands in for the GPU, so every check must
pass with zero error at 1 and 2 shards; then mistakes planted in the stand-in's
results (a pooled output, a short row, a long row beyond its error bound, a
counter) must each be caught.
"""
import numpy as np
import pytest

import round_check as rc
from oracle_lib import Oracle, reference_available

pytestmark = pytest.mark.skipif(not reference_available(), reason="oracle/_ref not built")


def _oracle_round(parts, world):
    feats, grads = rc.combined(parts)
    oracle = Oracle(rc.table_defs(parts[0]))
    outs = oracle.lookup(feats, shards=world)
    assert oracle.push(feats, grads) == 0
    return oracle, outs


def _reader(oracle, planted=None):
    def read(tid, keys):
        st, upd = oracle.state(tid)
        k = keys.astype(np.int64)
        w, m, v, u = st[k, 0].copy(), st[k, 1].copy(), st[k, 2].copy(), upd[k].copy()
        if planted:
            planted(tid, keys, w, m, v, u)
        return w, m, v, u
    return read


@pytest.mark.parametrize("world", [1, 2])
def test_checker_accepts_a_serial_round(workloads, world):
    parts = [workloads.hot(seed=11 + r, rows=700, n=6000) for r in range(world)]
    ref_result = rc.reference_round(parts)
    oracle, outs = _oracle_round(parts, world)
    F = len(parts[0].features)
    for rank in range(world):
        rep = rc.check_round(parts, rank, outs[rank * F:(rank + 1) * F], _reader(oracle),
                             ref_result=ref_result)
        assert rep["parity"], rep
        assert rep["long_rows"] > 0 and rep["rows_checked"] > rep["long_rows"]
        assert max(rep["long_max_norm_err"].values()) == 0.0


def test_checker_catches_planted_mistakes(workloads):
    parts = [workloads.hot(seed=21, rows=700, n=6000)]
    ref_result = rc.reference_round(parts)
    oracle, outs = _oracle_round(parts, 1)
    feats, _ = rc.combined(parts)
    keys = np.unique(np.concatenate([f.keys for f in feats]))
    counts = np.unique(np.concatenate([f.keys for f in feats]), return_counts=True)[1]
    long_key, short_key = keys[np.argmax(counts)], keys[np.argmin(counts)]
    assert counts.max() > rc.LONG_RUN

    def plant_long(tid, k, w, m, v, u):
        i = np.nonzero(k == long_key)[0][0]
        m[i, 0] *= np.float32(1.001)

    def plant_short(tid, k, w, m, v, u):
        i = np.nonzero(k == short_key)[0][0]
        w[i, 3] = np.nextafter(w[i, 3], np.float32(1))

    def plant_counter(tid, k, w, m, v, u):
        u[0] += 1

    for planted in (plant_long, plant_short, plant_counter):
        rep = rc.check_round(parts, 0, outs, _reader(oracle, planted), ref_result=ref_result)
        assert not rep["parity"], planted.__name__
    bad = [o.copy() for o in outs]
    bad[0].reshape(-1)[5] = np.nextafter(bad[0].reshape(-1)[5], np.float32(1))
    rep = rc.check_round(parts, 0, bad, _reader(oracle), ref_result=ref_result)
    assert not rep["parity"] and not rep["outputs_bitexact"]


def test_coalescing_rule_check(workloads):
    """check_coalesced accepts the rule's own lists and rejects a swapped pair
    of occurrences inside one row."""
    w = workloads.hot(seed=5, rows=300, n=3000)
    feats, _ = rc.combined([w])
    k, s, sc, fid = rc.occurrence_lists(feats, 1)
    uk, counts = np.unique(k, return_counts=True)
    got = {"tables": np.ones(len(uk), np.uint32), "keys": uk,
           "row_offsets": np.concatenate([[0], np.cumsum(counts)]).astype(np.uint64),
           "features": fid.copy(), "sources": s.astype(np.uint64), "scales": sc.copy()}
    assert rc.check_coalesced(got, feats)
    j = int(np.argmax(counts))
    lo = int(got["row_offsets"][j])
    a, b = lo, lo + 1
    while got["sources"][a] == got["sources"][b] and b < lo + counts[j] - 1:
        b += 1
    got["sources"][[a, b]] = got["sources"][[b, a]]
    got["features"][[a, b]] = got["features"][[b, a]]
    got["scales"][[a, b]] = got["scales"][[b, a]]
    assert not rc.check_coalesced(got, feats)
