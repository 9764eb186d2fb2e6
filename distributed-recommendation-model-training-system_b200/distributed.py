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

from . import EpsError, FeatureInput, INVALID_ARGUMENT, SEQUENCE  # noqa: F401


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
    tables: list


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

    def _on(self, stream):
        if stream is None:
            import contextlib
            return contextlib.nullcontext()
        return self.torch.cuda.stream(stream)

    def _a2a(self, out, inp, out_splits=None, in_splits=None):
        self.dist.all_to_all_single(out, inp, output_split_sizes=out_splits,
                                    input_split_sizes=in_splits, group=self.group)

    # ------------------------------------------------------------- lookup
    def lookup(self, feats: Sequence[FeatureInput], outputs=None, read_only: bool = False,
               input_stream=None):
        """Sharded pull of this rank's features.  Returns (handle, outputs).

        The partition and the key exchange run on `input_stream` (a stream on
        which the inputs are ready; default: the current stream), so that they
        can overlap the previous round's push; the shard lookup and the merge run
        on the current stream.  The call waits for the partition counts (they
        size the exchange)."""
        torch, n, F = self.torch, self.n, len(feats)
        main = self._stream()
        side = input_stream if (input_stream is not None and main is not None) else main
        dims = [self.store.dimension(f.table) for f in feats]
        pools = [int(f.pooling) for f in feats]
        tables = [int(f.table) for f in feats]
        with self._on(side):
            err, route = None, None
            counts = np.zeros((n, F, 2), np.uint64)
            try:
                route, counts = self.store.route(feats, n, side)
            except EpsError as e:
                err = e
            # ---- 2. counts + schema + error flag, one row per peer
            width = 4 * F + 1
            send = np.zeros((n, width), np.int64)
            send[:, :2 * F] = counts.reshape(n, 2 * F).astype(np.int64)
            send[:, 2 * F:3 * F] = tables
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
            recv_words = [payload_layout(peer[r])[3] for r in range(n)]
            payload = torch.empty(sum(send_words), dtype=torch.int64, device=self.device)
            self.store.route_scatter(route, payload, side)
            rpay = torch.empty(sum(recv_words), dtype=torch.int64, device=self.device)
            self._a2a(rpay, payload, recv_words, send_words)
        if side is not main:
            main.wait_stream(side)
            rpay.record_stream(main)
        # ---- 4. this shard's lookup over every requester's part (C++ layout)
        dim_arr = np.array(dims)
        prow = _rows(peer, pools)                 # [requester, f]
        part_send = torch.empty(max(1, int((prow * dim_arr[None, :]).sum())),
                                dtype=torch.float32, device=self.device)
        ticket = self.store.serve(rpay, peer, tables, pools, part_send, read_only=read_only,
                                  stream=main)
        # ---- 5. partials back to their requesters, merged in shard order
        mrow = _rows(counts, pools)               # [owner, f]
        send_f = [int((prow[r] * dim_arr).sum()) for r in range(n)]
        recv_f = [int((mrow[o] * dim_arr).sum()) for o in range(n)]
        part_recv = torch.empty(max(1, sum(recv_f)), dtype=torch.float32, device=self.device)
        self._a2a(part_recv[:sum(recv_f)], part_send[:sum(send_f)], recv_f, send_f)
        if outputs is None:
            outputs = [torch.empty((f.output_rows, d), dtype=torch.float32, device=self.device)
                       for f, d in zip(feats, dims)]
        self.store.route_merge(route, part_recv, outputs, main)
        handle = RoundHandle(route, ticket, counts, peer, dims, pools, read_only, tables)
        if read_only:
            self.store.route_release(route)
            handle.route = None
        return handle, outputs

    # --------------------------------------------------------------- push
    def push(self, handle: RoundHandle, gradients, wait: bool = False):
        """Sharded push of this rank's feature gradients (one tensor per feature,
        shaped like the lookup outputs).  Every rank must call it.

        The client-side finiteness check (distributed_client.cpp:249) is agreed
        by every rank on the device (all-reduce of a flag) and consumed by every
        owner's push on the device, so a non-finite value anywhere rejects the
        push on every shard (state unchanged, round pushable again or
        releasable) without a host round trip; with wait=False the rejection is
        reported by the store's synchronize()."""
        if handle.read_only:
            raise EpsError(INVALID_ARGUMENT, "read-only lookups cannot be pushed")
        torch, n = self.torch, self.n
        main = self._stream()
        dims = np.array(handle.dims)
        mrow = _rows(handle.counts, handle.poolings)
        prow = _rows(handle.peer_counts, handle.poolings)
        send_f = [int((mrow[o] * dims).sum()) for o in range(n)]
        recv_f = [int((prow[r] * dims).sum()) for r in range(n)]
        send = torch.empty(max(1, sum(send_f)), dtype=torch.float32, device=self.device)
        flag = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.store.route_gather(handle.route, gradients, send, flag, main)
        self.dist.all_reduce(flag, op=self.dist.ReduceOp.MAX, group=self.group)
        recv = torch.empty(max(1, sum(recv_f)), dtype=torch.float32, device=self.device)
        self._a2a(recv[:sum(recv_f)], send[:sum(send_f)], recv_f, send_f)
        # a rejected push with wait=True raises here and keeps the route and the
        # ticket (push again, or release); an enqueued push releases the route
        self.store.serve_push(handle.ticket, recv, handle.peer_counts, handle.tables,
                              handle.poolings, reject=flag, stream=main, wait=wait)
        self.store.route_release(handle.route)
        handle.route = None

    def release(self, handle: RoundHandle):
        """Abandons a round: frees its route and this shard's ticket (Release)."""
        if handle.route is not None:
            self.store.route_release(handle.route)
            handle.route = None
        if handle.ticket is not None:
            self.store.release(handle.ticket)
            handle.ticket = None
