"""Full-round parity check against the unmodified reference (test infrastructure).

One round -- a lookup and a push of every rank's batch from freshly initialised
tables -- is compared with the reference's own CPU parameter server
(oracle/_ref, compiled from the reference sources) serving the same job: every
rank's features as ONE combined request, rank-major (feature ids r * F + f),
through its DistributedClient over `world` CpuParameterService shards, i.e. with
the same shard count, so that pooled outputs merge the same shard partials in the
same order (src/client/distributed_client.cpp:173-188,227-232).

Bars (the path's parity target: gather and coalescing bit-exact, Adam within
the tolerance of a different summation order):
  * pooled / sequence outputs of this rank's features: bit-exact;
  * w, m, v and row_updates of every touched row this rank owns (key % world ==
    rank): bit-exact for rows whose occurrences in the combined request number
    at most 64 (summed serially in occurrence order on the GPU, as the reference
    does, src/access/batch_access.cpp:109-119), and for every row when the GPU
    store runs with EPS_B200_FLAG_REFERENCE_ORDER;
  * longer rows in the default mode: their gradient is summed in pieces of 64
    combined in a fixed tree, so it may differ from the reference's serial fp32
    sum.  The bar is the north star's 1e-6 relative, taken against the sum's
    condition: |g_gpu - g_ref| <= 1e-6 * sum|terms| per element (a sum with
    cancellation cannot be held to 1e-6 of its own value by ANY change of order;
    the rounding errors of either order are about 2^-24 * sqrt(L) * rms(partial
    sums), some 20x below this bar for random gradients).  w, m and v must lie
    within the bounds that difference implies through LazyAdam
    (src/update/lazy_adam.cpp:24-42), plus 2 ulp of the final roundings; the
    report gives the largest |difference| / bound (must be <= 1), the largest
    relative difference of each quantity and how many elements exceed 1e-6
    relative of their own value.

Also the coalescing itself (single GPU): the ticket's coalesced rows
(eps_b200_ticket_coalesced, the CompactGradients CSR) against the reference's
rule -- per unique row, its occurrences in (feature, bag, position) order with
their gradient row and scale -- restated with a stable numpy sort.
"""
from __future__ import annotations

import numpy as np

from oracle_lib import MEAN, SEQUENCE, Feature, Reference, TableDef

U = 2.0 ** -24
LONG_RUN = 64


def table_defs(workload):
    """The tables as the GPU store creates them (eps TableDefinition defaults)."""
    return [TableDef(id=t.id, dimension=t.dimension, learning_rate=1e-3, init_min=-0.05,
                     init_max=0.05, init_seed=42, rows=t.rows) for t in workload.tables]


def combined(parts):
    """Every rank's features as one request, rank-major (ids r * F + f)."""
    F = len(parts[0].features)
    feats, grads = [], []
    for r, p in enumerate(parts):
        for f, g in zip(p.features, p.gradients):
            feats.append(Feature(f.table, r * F + f.feature, f.pooling, f.keys, f.offsets))
            grads.append(g)
    return feats, grads


def reference_round(parts, state_bytes=64 << 30):
    """One lookup + push of the combined request on the reference with
    len(parts) shards.  Returns (reference, outputs, features, gradients)."""
    world = len(parts)
    feats, grads = combined(parts)
    ref = Reference(table_defs(parts[0]), shards=world, state_bytes=state_bytes)
    batch, outs = ref.lookup(feats)
    ref.push(batch, feats, grads)
    return ref, outs, feats, grads


def _scales(f):
    """Per-occurrence gradient source row and scale of a feature (fp32)."""
    n = len(f.keys)
    if f.pooling == SEQUENCE:
        return np.arange(n, dtype=np.int64), np.ones(n, np.float32)
    lengths = np.diff(f.offsets.astype(np.int64))
    bag = np.repeat(np.arange(len(lengths), dtype=np.int64), lengths)
    if f.pooling == MEAN:
        with np.errstate(divide="ignore"):
            per_bag = np.where(lengths > 0, np.float32(1.0) / lengths.astype(np.float32),
                               np.float32(1.0)).astype(np.float32)
    else:
        per_bag = np.ones(len(lengths), np.float32)
    return bag, per_bag[bag]


def occurrence_lists(feats, table):
    """The reference's coalescing of one table: occurrences in (feature, bag,
    position) order, stably sorted by key.  Returns keys, sources, scales,
    feature ids of the occurrences in that order."""
    keys, srcs, scales, fids = [], [], [], []
    for f in feats:
        if f.table != table:
            continue
        s, sc = _scales(f)
        keys.append(f.keys.astype(np.uint64))
        srcs.append(s)
        scales.append(sc)
        fids.append(np.full(len(f.keys), f.feature, np.uint32))
    if not keys:
        return (np.zeros(0, np.uint64), np.zeros(0, np.int64), np.zeros(0, np.float32),
                np.zeros(0, np.uint32))
    k = np.concatenate(keys)
    order = np.argsort(k, kind="stable")
    return k[order], np.concatenate(srcs)[order], np.concatenate(scales)[order], \
        np.concatenate(fids)[order]


def check_coalesced(got, feats):
    """Bit-exact comparison of eps_b200_ticket_coalesced output with the rule."""
    ok = True
    for table in sorted(set(int(t) for t in got["tables"])):
        sel = np.nonzero(got["tables"] == table)[0]
        k, s, sc, fid = occurrence_lists(feats, table)
        uk, first, counts = np.unique(k, return_index=True, return_counts=True)
        gk = got["keys"][sel]
        if not np.array_equal(gk, uk):
            return False
        ro = got["row_offsets"]
        lo, hi = int(ro[sel[0]]), int(ro[sel[-1] + 1])
        if not np.array_equal(np.diff(ro[sel[0]:sel[-1] + 2]).astype(np.int64), counts):
            return False
        ok &= np.array_equal(got["features"][lo:hi], fid)
        ok &= np.array_equal(got["sources"][lo:hi].astype(np.int64), s)
        ok &= np.array_equal(got["scales"][lo:hi].view(np.uint32), sc.view(np.uint32))
    return bool(ok)


def _ulp(x):
    return np.spacing(np.abs(x).astype(np.float32)).astype(np.float64)


def _abs_term_sums(feats, grads, table, keys_sel, dim, chunk=1 << 20):
    """sum_i |grad[src_i] * scale_i| per (selected key, dim), float64."""
    k, s, sc, fid = occurrence_lists(feats, table)
    by_id = {f.feature: g for f, g in zip(feats, grads)}
    out = np.zeros((len(keys_sel), dim), np.float64)
    if not len(keys_sel):
        return out
    pos = np.minimum(np.searchsorted(keys_sel, k), len(keys_sel) - 1)
    idx = np.nonzero(keys_sel[pos] == k)[0]
    for a in range(0, len(idx), chunk):
        part = idx[a:a + chunk]
        terms = np.empty((len(part), dim), np.float32)
        for f in np.unique(fid[part]):
            m = fid[part] == f
            terms[m] = by_id[int(f)][s[part][m]] * sc[part][m][:, None]
        np.add.at(out, pos[part], np.abs(terms.astype(np.float64)))
    return out


def check_round(parts, rank, gpu_outputs, read_gpu_state, reference_order=False, ref_result=None,
                table_lr=1e-3, b1=0.9, b2=0.999, eps=1e-8, b1p=0.9, b2p=0.999):
    """Compares one GPU round (outputs of rank `rank`'s features, state of its
    owned rows through read_gpu_state(table, keys) -> (w, m, v, updates)) with
    the reference.  Returns a report dict; report['parity'] is the verdict."""
    world = len(parts)
    ref, outs, feats, grads = ref_result if ref_result is not None else reference_round(parts)
    F = len(parts[0].features)
    rep = {"world": world, "rank": rank, "reference_order": bool(reference_order)}
    mine = outs[rank * F:(rank + 1) * F]
    rep["outputs_bitexact"] = bool(all(
        np.array_equal(np.asarray(g, np.float32).view(np.uint32), w.view(np.uint32))
        for g, w in zip(gpu_outputs, mine)))
    lr_t = np.float64(np.float32(table_lr) * np.float32(np.sqrt(np.float32(1.0) - np.float32(b2p))) /
                      np.float32(np.float32(1.0) - np.float32(b1p))) * (1 + 1e-6)
    exact_ok, rows_checked, long_rows = True, 0, 0
    norm = {"w": 0.0, "m": 0.0, "v": 0.0}
    rel = {"w": 0.0, "m": 0.0, "v": 0.0}
    over = {"w": 0, "m": 0, "v": 0}
    updates_ok = True
    for t in parts[0].tables:
        ks = [f.keys for f in feats if f.table == t.id]
        if not ks:
            continue
        uk, counts = np.unique(np.concatenate(ks), return_counts=True)
        own = (uk % np.uint64(world)) == np.uint64(rank)
        uk, counts = uk[own], counts[own]
        if not len(uk):
            continue
        gw, gm, gv, gu = read_gpu_state(t.id, uk)
        rw, rm, rv, ru = ref.read_many(t.id, uk)
        rows_checked += len(uk)
        updates_ok &= bool(np.array_equal(np.asarray(gu, np.uint64), ru))
        long_sel = (counts > LONG_RUN) if not reference_order else np.zeros(len(uk), bool)
        ex = ~long_sel
        for g_, r_ in ((gw, rw), (gm, rm), (gv, rv)):
            exact_ok &= bool(np.array_equal(np.asarray(g_, np.float32)[ex].view(np.uint32),
                                            r_[ex].view(np.uint32)))
        if not long_sel.any():
            continue
        long_rows += int(long_sel.sum())
        lk = uk[long_sel]
        S = _abs_term_sums(feats, grads, t.id, lk, t.dimension)
        bg = 1e-6 * S
        rm_l, rv_l, rw_l = (x[long_sel].astype(np.float64) for x in (rm, rv, rw))
        gm_l, gv_l, gw_l = (np.asarray(x, np.float32)[long_sel].astype(np.float64)
                            for x in (gm, gv, gw))
        bm = (1 - b1) * bg * (1 + 4 * U) + 2 * _ulp(rm_l)
        bv = (1 - b2) * (2 * S + bg) * bg * (1 + 6 * U) + 2 * _ulp(rv_l)
        vmin = np.maximum(rv_l - bv, 0.0)
        den = np.sqrt(vmin) + eps
        dsq = bv / (np.sqrt(rv_l) + np.sqrt(vmin) + 1e-300)
        bw = lr_t * (bm / den + (np.abs(rm_l) + bm) * dsq / den ** 2) * (1 + 8 * U) + \
            2 * _ulp(rw_l)
        for name, g_, r_, b_ in (("w", gw_l, rw_l, bw), ("m", gm_l, rm_l, bm), ("v", gv_l, rv_l, bv)):
            d = np.abs(g_ - r_)
            norm[name] = max(norm[name], float((d / b_).max()))
            rr = d / np.maximum(np.abs(r_), 1e-30)
            rel[name] = max(rel[name], float(rr.max()))
            over[name] += int((rr > 1e-6).sum())
    rep.update({"rows_checked": rows_checked, "long_rows": long_rows,
                "rows_bitexact": bool(exact_ok), "row_updates_equal": bool(updates_ok),
                "long_max_norm_err": norm, "long_max_rel_err": rel,
                "long_elems_over_1e-6_rel": over})
    rep["parity"] = bool(rep["outputs_bitexact"] and exact_ok and updates_ok and
                         all(v <= 1.0 for v in norm.values()))
    return rep
