"""Test infrastructure for the multi-GPU round (distributed.ShardedClient).

* ``make_batch``        -- seeded per-rank batches with one shared feature schema
                           (sum / mean / sequence, empty bags, duplicate keys);
* ``FakeShardStore``    -- a CPU stand-in for ParameterStore used by the gloo
                           tests: a numpy restatement of the route layouts
                           (partition, payload, merge, gather) written from the
                           C-ABI contract in include/eps_b200.h, shard partials
                           computed from a fixed weight table, pushes recorded;
* ``reduce_gradients``  -- numpy ReduceGradients (src/access/batch_access.cpp:54-97)
                           with explicit valid lengths, to check what each owner
                           was pushed;
* ``concat``            -- the single combined request that one round of n ranks
                           is equivalent to (features of every rank, rank-major).

Nothing here is part of the product path.
"""
from __future__ import annotations

import numpy as np

from oracle_lib import Feature, TableDef, SUM, MEAN, SEQUENCE

TABLES = [TableDef(id=1, dimension=8, learning_rate=0.01, init_min=-0.05, init_max=0.05,
                   rows=61),
          TableDef(id=2, dimension=4, learning_rate=0.02, init_min=-0.05, init_max=0.05,
                   rows=37)]
SCHEMA = [(1, SUM), (1, MEAN), (2, SEQUENCE), (2, SUM)]


def make_batch(rank: int, step: int, bags: int = 9, onehot: bool = False):
    """Features of one rank (ids 0..F-1) and matching gradients.  With
    `onehot`, the first two features (sum, mean) hold one key per bag over many
    duplicate keys: the groups the multi-GPU round returns distinct rows for."""
    rng = np.random.default_rng(1000 * rank + step + (500 if onehot else 0))
    rows = {t.id: t.rows for t in TABLES}
    dims = {t.id: t.dimension for t in TABLES}
    feats, grads = [], []
    for fi, (tid, pool) in enumerate(SCHEMA):
        if onehot and fi < 2:
            lens = np.ones(4 * bags, np.int64)
        else:
            lens = rng.integers(0, 6, size=bags)
            lens[rng.integers(0, bags)] = 0                   # at least one empty bag
        offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.uint64)
        hot = rng.integers(0, rows[tid], size=3)
        keys = np.where(rng.random(int(offs[-1])) < 0.4,
                        rng.choice(hot, size=int(offs[-1])),
                        rng.integers(0, rows[tid], size=int(offs[-1]))).astype(np.uint64)
        f = Feature(tid, fi, pool, keys, offs)
        feats.append(f)
        grads.append(rng.normal(0, 0.01, size=(f.output_rows, dims[tid])).astype(np.float32))
    return feats, grads


def concat(per_rank):
    """[(feats, grads)] per rank -> the combined request (ids r * F + f)."""
    feats, grads = [], []
    for r, (fs, gs) in enumerate(per_rank):
        F = len(fs)
        for f, g in zip(fs, gs):
            feats.append(Feature(f.table, r * F + f.feature, f.pooling, f.keys, f.offsets))
            grads.append(g)
    return feats, grads


def reduce_gradients(features, grads, dims):
    """{(table, key): float32[D]} summed in (feature, bag, position) order.

    features: list of (table, pooling, keys, offsets, valid_lengths)."""
    out = {}
    for (tid, pool, keys, offs, lens), g in zip(features, grads):
        for b in range(len(offs) - 1):
            scale = np.float32(1.0) / np.float32(lens[b]) if pool == MEAN and lens[b] else np.float32(1.0)
            for i in range(int(offs[b]), int(offs[b + 1])):
                src = g[i if pool == SEQUENCE else b]
                k = (tid, int(keys[i]))
                acc = out.setdefault(k, np.zeros(dims[tid], np.float32))
                acc += (src * scale).astype(np.float32)
    return out


class FakeShardStore:
    """CPU stand-in for ParameterStore(shard_id=rank, shard_count=n)."""

    def __init__(self, rank, n, weights):
        self.rank, self.n = rank, n
        self.device = -1
        self.weights = weights                      # {table: float32[key_space, D]}
        self.routes, self.tickets, self.pushed = {}, {}, []
        self._next = 1

    def dimension(self, table):
        return self.weights[table].shape[1]

    # ---- route: PrepareLookupInputs with the bags that have keys on each shard
    def route(self, feats, n, counts, stream=None):
        """Writes the count rows [n][5F + 1] into `counts` (tables, poolings,
        distinct keys -- always 0: this stand-in deduplicates no group --
        input-error bits last) and keeps the partition."""
        F = len(feats)
        rows = np.zeros((n, 5 * F + 1), np.int64)
        rows[:, 2 * F:3 * F] = [f.table for f in feats]
        rows[:, 3 * F:4 * F] = [f.pooling for f in feats]
        parts, bits = [], 0
        for fi, f in enumerate(feats):
            keys = f.keys.numpy().astype(np.uint64)
            offs = f.offsets.numpy().astype(np.uint64)
            space = self.weights[f.table].shape[0]
            if offs[0] != 0 or offs[-1] != len(keys) or np.any(np.diff(offs.astype(np.int64)) < 0):
                bits |= 1
            if np.any(keys >= space):
                bits |= 2
            per = [dict(keys=[], pos=[], kept=[], kept_len=[], kept_end=[]) for _ in range(n)]
            if not bits:
                for b in range(len(offs) - 1):
                    for i in range(int(offs[b]), int(offs[b + 1])):
                        o = int(keys[i] % n)
                        per[o]["keys"].append(int(keys[i]))
                        per[o]["pos"].append(i)
                    for o in range(n):
                        got = len(per[o]["keys"]) - (per[o]["kept_end"][-1] if per[o]["kept_end"] else 0)
                        if got:
                            per[o]["kept"].append(b)
                            per[o]["kept_len"].append(int(offs[b + 1] - offs[b]))
                            per[o]["kept_end"].append(len(per[o]["keys"]))
            for o in range(n):
                rows[o, 2 * fi] = len(per[o]["keys"])
                rows[o, 2 * fi + 1] = len(per[o]["kept"])
            parts.append(per)
        rows[:, 5 * F] = bits
        counts.copy_(__import__("torch").from_numpy(rows))
        rid = self._next
        self._next += 1
        self.routes[rid] = dict(feats=feats, parts=parts, n=n)
        return rid

    def route_scatter(self, rid, payload, stream=None):
        r = self.routes[rid]
        words = []
        for o in range(r["n"]):
            per = [p[o] for p in r["parts"]]
            for p in per:
                words += p["keys"]
            for p in per:
                words += [0] + p["kept_end"]
            for p in per:
                words += p["kept_len"]
        payload.copy_(__import__("torch").tensor(words, dtype=payload.dtype))

    def _row_blocks(self, r):
        """[(o, f, rows)] in shard-major, feature-minor order."""
        out = []
        for o in range(r["n"]):
            for fi, f in enumerate(r["feats"]):
                p = r["parts"][fi][o]
                out.append((o, fi, len(p["keys"]) if f.pooling == SEQUENCE else len(p["kept"])))
        return out

    def route_merge(self, rid, partials, outputs, stream=None):
        r = self.routes[rid]
        part = partials.numpy()
        at = 0
        blocks = {}
        for o, fi, rows in self._row_blocks(r):
            D = self.dimension(r["feats"][fi].table)
            blocks[(o, fi)] = part[at:at + rows * D].reshape(rows, D)
            at += rows * D
        for fi, f in enumerate(r["feats"]):
            out = outputs[fi].numpy()
            D = out.shape[1]
            if f.pooling == SEQUENCE:
                for o in range(r["n"]):
                    for j, pos in enumerate(r["parts"][fi][o]["pos"]):
                        out[pos] = blocks[(o, fi)][j]
                continue
            offs = f.offsets.numpy()
            for b in range(len(offs) - 1):
                acc = np.zeros(D, np.float32)
                for o in range(r["n"]):
                    kept = r["parts"][fi][o]["kept"]
                    if b in kept:
                        acc = acc + blocks[(o, fi)][kept.index(b)]
                length = int(offs[b + 1] - offs[b])
                if f.pooling == MEAN and length:
                    acc = acc / np.float32(length)
                out[b] = acc

    def route_gather(self, rid, grads, send, flag=None, stream=None):
        r = self.routes[rid]
        rows_out = []
        for o, fi, rows in self._row_blocks(r):
            g = grads[fi].numpy()
            p = r["parts"][fi][o]
            idx = p["pos"] if r["feats"][fi].pooling == SEQUENCE else p["kept"]
            rows_out.append(g[idx].reshape(-1))
        flat = np.concatenate(rows_out) if rows_out else np.zeros(0, np.float32)
        send.copy_(__import__("torch").from_numpy(flat.astype(np.float32)))
        if flag is not None:
            flag[0] = int(any(not np.all(np.isfinite(g.numpy())) for g in grads))

    def route_release(self, rid):
        del self.routes[rid]

    # ---- shard side
    def lookup(self, feats, read_only=False, shard_partial=False, outputs=None, stream=None):
        assert shard_partial
        rec = []
        for f, out in zip(feats, outputs):
            keys = f.keys.numpy().astype(np.uint64)
            offs = f.offsets.numpy().astype(np.uint64)
            lens = f.valid_lengths.numpy().astype(np.uint64)
            assert np.all(keys % self.n == self.rank), "key routed to the wrong shard"
            w = self.weights[f.table]
            o = out.numpy()
            if f.pooling == SEQUENCE:
                for i, k in enumerate(keys):
                    o[i] = np.float32(0) + w[int(k)]
            else:
                for b in range(len(offs) - 1):
                    acc = np.zeros(w.shape[1], np.float32)
                    for i in range(int(offs[b]), int(offs[b + 1])):
                        acc = acc + w[int(keys[i])]
                    o[b] = acc
            rec.append((f.table, f.pooling, keys, offs, lens, f.feature))
        if read_only:
            return None, outputs
        t = self._next
        self._next += 1
        self.tickets[t] = rec
        return t, outputs

    def push(self, ticket, grads, features=None, wait=True, stream=None):
        rec = self.tickets.pop(ticket)
        by_id = dict(zip(features, grads))
        feats = [(tid, pool, keys, offs, lens) for tid, pool, keys, offs, lens, _ in rec]
        gs = [by_id[fid].numpy().copy() for *_, fid in rec]
        self.pushed.append((feats, gs))

    def serve(self, payload, peer_counts, tables, poolings, partials, read_only=False,
              stream=None):
        """Owner side: parse every requester's payload region and run the shard
        lookup (ids r * F + f) into `partials`, requester-major."""
        import torch
        pay = payload.numpy()
        n, F = peer_counts.shape[0], len(tables)
        feats, outs, base, at = [], [], 0, 0
        for r in range(n):
            nk = [int(peer_counts[r, f, 0]) for f in range(F)]
            kb = [int(peer_counts[r, f, 1]) for f in range(F)]
            k0, o0, l0 = base, base + sum(nk), base + sum(nk) + sum(kb) + F
            for f in range(F):
                keys = pay[k0:k0 + nk[f]]
                offs = pay[o0:o0 + kb[f] + 1]
                lens = pay[l0:l0 + kb[f]]
                k0 += nk[f]; o0 += kb[f] + 1; l0 += kb[f]
                feats.append(type("F", (), dict(table=tables[f], pooling=poolings[f],
                                                feature=r * F + f,
                                                keys=torch.from_numpy(keys.copy()),
                                                offsets=torch.from_numpy(offs.copy()),
                                                valid_lengths=torch.from_numpy(lens.copy()))))
                rows = nk[f] if poolings[f] == SEQUENCE else kb[f]
                D = self.dimension(tables[f])
                outs.append(partials[at:at + rows * D].view(rows, D))
                at += rows * D
            base += sum(nk) + 2 * sum(kb) + F
        ticket, _ = self.lookup(feats, read_only=read_only, shard_partial=True, outputs=outs)
        return ticket

    def serve_push(self, ticket, gradients, peer_counts, tables, poolings, reject=None,
                   stream=None, wait=False):
        from eps_b200 import EpsError
        n, F = peer_counts.shape[0], len(tables)
        if reject is not None and int(reject[0]):
            if wait:
                raise EpsError(1, "non-finite gradient")
            return
        views, ids, at = [], [], 0
        for r in range(n):
            for f in range(F):
                rows = int(peer_counts[r, f, 0] if poolings[f] == SEQUENCE else peer_counts[r, f, 1])
                D = self.dimension(tables[f])
                views.append(gradients[at:at + rows * D].view(rows, D))
                ids.append(r * F + f)
                at += rows * D
        self.push(ticket, views, features=ids)

    def release(self, ticket):
        self.tickets.pop(ticket, None)


class ThreadComm:
    """In-process stand-in for torch.distributed among n threads (one per
    emulated rank, all on one GPU): every collective synchronises the calling
    thread's device work first, then exchanges tensors under a barrier.  No
    kernel ever waits on another rank's kernel."""

    class ReduceOp:
        MAX = "max"

    def __init__(self, n):
        import threading
        self.n = n
        self.barrier = threading.Barrier(n, timeout=120)
        self.slots = [None] * n
        self.local = threading.local()

    def bind(self, rank):
        self.local.rank = rank

    def get_rank(self, group=None):
        return self.local.rank

    def get_world_size(self, group=None):
        return self.n

    def _sync(self, t):
        import torch
        if t.is_cuda:
            torch.cuda.synchronize(t.device)

    def all_to_all_single(self, out, inp, output_split_sizes=None, input_split_sizes=None,
                          group=None):
        import torch
        r, n = self.local.rank, self.n
        ins = input_split_sizes or [inp.shape[0] // n] * n
        outs = output_split_sizes or [out.shape[0] // n] * n
        self._sync(inp)
        self.slots[r] = (inp, list(ins))
        self.barrier.wait()
        at = 0
        for src in range(n):
            t, splits = self.slots[src]
            start = sum(splits[:r])
            assert splits[r] == outs[src], "split sizes disagree"
            out[at:at + outs[src]].copy_(t[start:start + splits[r]])
            at += outs[src]
        self._sync(out)
        self.barrier.wait()

    def all_reduce(self, t, op=None, group=None):
        import torch
        r = self.local.rank
        self._sync(t)
        self.slots[r] = t.clone()
        self.barrier.wait()
        m = self.slots[0]
        for x in self.slots[1:]:
            m = torch.maximum(m, x)
        self.barrier.wait()
        t.copy_(m)
        self._sync(t)
