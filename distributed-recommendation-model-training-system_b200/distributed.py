"""Multi-GPU round: one ParameterStore shard per rank, rows sharded by key % n.

Mirrors the reference's DistributedClient over n shards
(include/eps/distributed_client.hpp:32-70, src/client/distributed_client.cpp),
with every rank acting both as a client (its own data-parallel batch) and as
the shard that owns keys k with k % n == rank:

  lookup  1. route      keys bucketed by owner on the device (eps_b200_route:
                        PrepareLookupInputs, src/access/prepared_lookup.cpp:47-83)
          2. counts     all-to-all of (keys, kept bags) per (owner, feature)
          3. payload    all-to-all of keys / bag offsets / valid lengths
          4. shard      one eps_b200_lookup(shard_partial=1) per rank over the
                        features of ALL requesters (requester-major), which is
                        the reference shard's Lookup of that combined request
          5. partials   all-to-all back; eps_b200_route_merge adds them in shard
                        order and divides mean bags (distributed_client.cpp:173-188,227-232)
  push    6. gather     eps_b200_route_gather: the gradient rows each owner needs
                        (distributed_client.cpp:252-265)
          7. gradients  all-to-all; each owner runs ONE eps_b200_push over all
                        requesters' rows: ReduceGradients in (requester, feature,
                        bag, position) order + LazyAdam, beta powers advanced once
                        per round per table.

Per round every owner therefore applies exactly what a reference shard applies
for one DistributedClient lookup + push whose features are the concatenation
of every rank's features in rank order; tests pin that bit for bit.

Every rank must issue the same sequence of rounds with the same feature schema
(tables and poolings in the same order).  Input errors are agreed on by all
ranks through the count exchange before any data moves, so a bad input raises
EpsError on every rank instead of leaving peers waiting in a collective.
The exchange runs through torch.distributed (NCCL on GPUs, gloo in CPU tests)
on the caller's current stream.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import numpy as np

from . import EpsError, FeatureInput, INVALID_ARGUMENT, SEQUENCE


@dataclass
class RoundHandle:
    """State of one sharded lookup until its push (DistributedBatch)."""
    route: int | None
    ticket: int | None
    counts: np.ndarray        # [owner, feature, (keys, kept)] of this rank's batch
    peer_counts: np.ndarray   # [requester, feature, (keys, kept)] received by this shard
    dims: list
    poolings: list
    read_only: bool


def _rows(counts: np.ndarray, poolings) -> np.ndarray:
    """Rows exchanged per (shard, feature): keys for sequence, kept bags otherwise."""
    seq = np.array([p == SEQUENCE for p in poolings])
    return np.where(seq[None, :], counts[:, :, 0], counts[:, :, 1]).astype(np.int64)


def payload_layout(counts_row: np.ndarray):
    """Word offsets of one shard's payload: (keys_at[f], offsets_at[f], lengths_at[f], total)."""
    nk = counts_row[:, 0].astype(np.int64)
    kb = counts_row[:, 1].astype(np.int64)
    F = len(nk)
    keys_at = np.concatenate([[0], np.cumsum(nk)[:-1]]) if F else np.zeros(0, np.int64)
    NK = int(nk.sum())
    off_at = NK + np.concatenate([[0], np.cumsum(kb + 1)[:-1]])
    KB = int(kb.sum())
    len_at = NK + KB + F + np.concatenate([[0], np.cumsum(kb)[:-1]])
    return keys_at, off_at, len_at, NK + 2 * KB + F


class ShardedClient:
    """DistributedClient over one shard per rank; see the module docstring.

    `store` is this rank's ParameterStore(shard_id=rank, shard_count=world) with
    every table created on every rank.  `group` is a torch.distributed process
    group (default: the world).  `comm` replaces torch.distributed by an object
    with the same get_rank / get_world_size / all_to_all_single / all_reduce /
    ReduceOp API (in-process ranks in tests)."""

    def __init__(self, store, group=None, device=None, comm=None):
        import torch
        if comm is None:
            import torch.distributed as comm
        self.torch = torch
        self.dist = comm                 # torch.distributed, or a stand-in with its API
        dist = comm
        self.store = store
        self.group = group
        self.rank = dist.get_rank(group)
        self.n = dist.get_world_size(group)
        if device is None:
            device = torch.device(f"cuda:{store.device}")
        self.device = torch.device(device)

    # ------------------------------------------------------------ helpers
    def _stream(self):
        if self.device.type == "cuda":
            return self.torch.cuda.current_stream(self.device)
        return None

    def _a2a(self, out, inp, out_splits=None, in_splits=None):
        self.dist.all_to_all_single(out, inp, output_split_sizes=out_splits,
                                    input_split_sizes=in_splits, group=self.group)

    # ------------------------------------------------------------- lookup
    def lookup(self, feats: Sequence[FeatureInput], outputs=None, read_only: bool = False):
        """Sharded pull of this rank's features.  Returns (handle, outputs)."""
        torch, n, F = self.torch, self.n, len(feats)
        stream = self._stream()
        dims = [self.store.dimension(f.table) for f in feats]
        pools = [int(f.pooling) for f in feats]
        err, route = None, None
        counts = np.zeros((n, F, 2), np.uint64)
        try:
            route, counts = self.store.route(feats, n, stream)
        except EpsError as e:
            err = e
        # ---- 2. counts + schema + error flag, one row per peer
        width = 4 * F + 1
        send = np.zeros((n, width), np.int64)
        send[:, :2 * F] = counts.reshape(n, 2 * F).astype(np.int64)
        send[:, 2 * F:3 * F] = [f.table for f in feats]
        send[:, 3 * F:4 * F] = pools
        send[:, 4 * F] = 1 if err else 0
        send_t = torch.from_numpy(send).to(self.device)
        recv_t = torch.empty_like(send_t)
        self._a2a(recv_t, send_t)
        recv = recv_t.cpu().numpy()
        bad_schema = (recv[:, 2 * F:4 * F] != send[0, 2 * F:4 * F][None, :]).any()
        if err is not None or recv[:, 4 * F].any() or bad_schema:
            if route is not None:
                self.store.route_release(route)
            if err is not None:
                raise err
            raise EpsError(INVALID_ARGUMENT, "a peer rank rejected its lookup inputs"
                           if not bad_schema else "ranks disagree on the feature schema")
        peer = recv[:, :2 * F].reshape(n, F, 2).astype(np.uint64)   # [requester, f, (k, b)]

        # ---- 3. payload: keys / offsets / valid lengths per owner
        send_words = [payload_layout(counts[o])[3] for o in range(n)]
        recv_lay = [payload_layout(peer[r]) for r in range(n)]
        recv_words = [lay[3] for lay in recv_lay]
        payload = torch.empty(sum(send_words), dtype=torch.int64, device=self.device)
        self.store.route_scatter(route, payload, stream)
        rpay = torch.empty(sum(recv_words), dtype=torch.int64, device=self.device)
        self._a2a(rpay, payload, recv_words, send_words)

        # ---- 4. this shard's lookup over every requester's part
        prow = _rows(peer, pools)                 # [requester, f]
        own_feats, part_views = [], []
        part_send = torch.empty(int((prow * np.array(dims)[None, :]).sum()),
                                dtype=torch.float32, device=self.device)
        base, fo = 0, 0
        for r in range(n):
            keys_at, off_at, len_at, words = recv_lay[r]
            for f in range(F):
                nk, kb = int(peer[r, f, 0]), int(peer[r, f, 1])
                k0, o0, l0 = base + int(keys_at[f]), base + int(off_at[f]), base + int(len_at[f])
                own_feats.append(FeatureInput(feats[f].table, r * F + f, pools[f],
                                              rpay[k0:k0 + nk], rpay[o0:o0 + kb + 1],
                                              rpay[l0:l0 + kb]))
                rows = int(prow[r, f])
                part_views.append(part_send[fo:fo + rows * dims[f]].view(rows, dims[f]))
                fo += rows * dims[f]
            base += words
        ticket, _ = self.store.lookup(own_feats, read_only=read_only, shard_partial=True,
                                      outputs=part_views, stream=stream)

        # ---- 5. partials back to their requesters, merged in shard order
        mrow = _rows(counts, pools)               # [owner, f]
        send_f = [int((prow[r] * np.array(dims)).sum()) for r in range(n)]
        recv_f = [int((mrow[o] * np.array(dims)).sum()) for o in range(n)]
        part_recv = torch.empty(sum(recv_f), dtype=torch.float32, device=self.device)
        self._a2a(part_recv, part_send, recv_f, send_f)
        if outputs is None:
            outputs = [torch.empty((f.output_rows, d), dtype=torch.float32, device=self.device)
                       for f, d in zip(feats, dims)]
        self.store.route_merge(route, part_recv, outputs, stream)
        handle = RoundHandle(route, ticket, counts, peer, dims, pools, read_only)
        if read_only:
            self.store.route_release(route)
        return handle, outputs

    # --------------------------------------------------------------- push
    def push(self, handle: RoundHandle, gradients, wait: bool = False):
        """Sharded push of this rank's feature gradients (one tensor per feature,
        shaped like the lookup outputs).  Every rank must call it."""
        if handle.read_only:
            raise EpsError(INVALID_ARGUMENT, "read-only lookups cannot be pushed")
        torch, n = self.torch, self.n
        F = len(handle.dims)
        stream = self._stream()
        dims = np.array(handle.dims)
        mrow = _rows(handle.counts, handle.poolings)
        prow = _rows(handle.peer_counts, handle.poolings)
        send_f = [int((mrow[o] * dims).sum()) for o in range(n)]
        recv_f = [int((prow[r] * dims).sum()) for r in range(n)]
        send = torch.empty(sum(send_f), dtype=torch.float32, device=self.device)
        flag = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.store.route_gather(handle.route, gradients, send, flag, stream)
        # the client-side finiteness check (distributed_client.cpp:249), agreed by
        # every rank before any shard applies anything: a rejected push leaves the
        # round pushable (retry) or releasable, as in the reference
        self.dist.all_reduce(flag, op=self.dist.ReduceOp.MAX, group=self.group)
        if int(flag.item()):
            raise EpsError(INVALID_ARGUMENT, "non-finite gradient")
        self.store.route_release(handle.route)
        handle.route = None
        recv = torch.empty(sum(recv_f), dtype=torch.float32, device=self.device)
        self._a2a(recv, send, recv_f, send_f)
        views, ids, fo = [], [], 0
        for r in range(n):
            for f in range(F):
                rows = int(prow[r, f])
                views.append(recv[fo:fo + rows * int(dims[f])].view(rows, int(dims[f])))
                ids.append(r * F + f)
                fo += rows * int(dims[f])
        self.store.push(handle.ticket, views, features=ids, wait=wait, stream=stream)
        handle.ticket = None

    def release(self, handle: RoundHandle):
        """Abandons a round: frees its route and this shard's ticket (Release)."""
        if handle.route is not None:
            self.store.route_release(handle.route)
            handle.route = None
        if handle.ticket is not None:
            self.store.release(handle.ticket)
            handle.ticket = None
