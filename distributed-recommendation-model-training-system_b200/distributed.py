"""Multi-GPU round: one ParameterStore shard per rank, rows sharded by key % n.

Mirrors the reference's DistributedClient over n shards
(include/eps/distributed_client.hpp:32-70, src/client/distributed_client.cpp),
with every rank acting both as a client (its own data-parallel batch) and as
the shard that owns keys k with k % n == rank:

  lookup  1. route      keys bucketed by owner on the device (eps_b200_route:
                        PrepareLookupInputs, src/access/prepared_lookup.cpp:47-83)
          2. counts     all-to-all of (keys, kept bags, distinct keys) per
                        (owner, feature)
          3. payload    all-to-all of keys / bag offsets / valid lengths, and the
                        distinct keys of deduplicated groups
          4. shard      one eps_b200_lookup(shard_partial=1) per rank over the
                        features of ALL requesters (requester-major), which is
                        the reference shard's Lookup of that combined request
          5. partials   all-to-all back (a deduplicated group -- one key per kept
                        bag, dense table -- returns each distinct row once);
                        eps_b200_route_merge adds them in shard order and divides
                        mean bags (distributed_client.cpp:173-188,227-232)
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

import ctypes as C

from . import EpsError, FeatureInput, INVALID_ARGUMENT, SEQUENCE, Status, _check, load_library  # noqa: F401


@dataclass
class RoundHandle:
    """State of one sharded lookup until its push (DistributedBatch)."""
    route: int | None
    ticket: int | None
    counts: np.ndarray        # [owner, feature, (keys, kept, distinct)] of this rank's batch
    peer_counts: np.ndarray   # [requester, feature, (keys, kept, distinct)] received here
    dims: list
    poolings: list
    read_only: bool
    tables: list
    send_f: np.ndarray = None   # floats of partials sent to each requester
    recv_f: np.ndarray = None   # floats of partials received from each owner
    gsend_f: np.ndarray = None  # floats of gradients sent to each owner
    grecv_f: np.ndarray = None  # floats of gradients received from each requester
    mrow: np.ndarray = None
    prow: np.ndarray = None


@dataclass
class PreparedRound:
    """A partitioned batch whose keys have reached their owners (PreparedLookup)."""
    route: int | None
    counts: np.ndarray
    peer: np.ndarray
    dims: np.ndarray
    pools: list
    tables: list
    payload: object
    side: object
    ready: object
    output_rows: list
    inputs: list


def _rows(counts: np.ndarray, poolings) -> np.ndarray:
    """Rows exchanged per (shard, feature): keys for sequence, kept bags otherwise."""
    seq = np.array([p == SEQUENCE for p in poolings])
    return np.where(seq[None, :], counts[:, :, 0], counts[:, :, 1]).astype(np.int64)


def _device_inputs(feats):
    """The device tensors of a batch (keys, offsets, valid lengths)."""
    out = []
    for f in feats:
        for t in (f.keys, f.offsets, f.valid_lengths):
            if t is not None and hasattr(t, "record_stream") and getattr(t, "is_cuda", False):
                out.append(t)
    return out


def _input_message(bits: int) -> str:
    parts = []
    if bits & 1:
        parts.append("bag offsets must rise from 0 to the key count")
    if bits & 4:
        parts.append("valid lengths must equal the bag sizes")
    if bits & 2:
        parts.append("key outside the table's key space")
    return "invalid lookup inputs: " + "; ".join(parts or [f"error bits {bits}"])


def payload_layout(counts_row: np.ndarray):
    """Word offsets of one shard's payload: (keys_at[f], offsets_at[f],
    lengths_at[f], uniq_at[f], total).  counts_row[f] = (keys, kept bags,
    distinct keys); a deduplicated group (distinct > 0) ends the payload with
    [0, U, U distinct keys] at uniq_at[f]."""
    nk = counts_row[:, 0].astype(np.int64)
    kb = counts_row[:, 1].astype(np.int64)
    uw = np.where(counts_row[:, 2] > 0, counts_row[:, 2].astype(np.int64) + 2, 0)
    F = len(nk)
    keys_at = np.concatenate([[0], np.cumsum(nk)[:-1]]) if F else np.zeros(0, np.int64)
    NK = int(nk.sum())
    off_at = NK + np.concatenate([[0], np.cumsum(kb + 1)[:-1]])
    KB = int(kb.sum())
    len_at = NK + KB + F + np.concatenate([[0], np.cumsum(kb)[:-1]])
    uniq_at = NK + 2 * KB + F + np.concatenate([[0], np.cumsum(uw)[:-1]])
    return keys_at, off_at, len_at, uniq_at, NK + 2 * KB + F + int(uw.sum())


def _words(counts: np.ndarray) -> np.ndarray:
    """Payload words per owner (or requester) of counts [n, F, (keys, kept, distinct)]."""
    uw = np.where(counts[:, :, 2] > 0, counts[:, :, 2] + 2, 0)
    return (counts[:, :, 0] + 2 * counts[:, :, 1] + 1 + uw).sum(axis=1)


class ShardedClient:
    """DistributedClient over one shard per rank; see the module docstring.

    `store` is this rank's ParameterStore(shard_id=rank, shard_count=world) with
    every table created on every rank.  `group` is a torch.distributed process
    group (default: the world).  `comm` replaces torch.distributed by an object
    with the same get_rank / get_world_size / all_to_all_single / all_reduce /
    ReduceOp API (in-process ranks in tests)."""

    def __init__(self, store, group=None, device=None, comm=None, input_comm=None):
        import torch
        if comm is None:
            import torch.distributed as comm
        self.torch = torch
        self.dist = comm                 # torch.distributed, or a stand-in with its API
        # the prepare phase's exchanges (input stream) may use their own
        # communicator, so that they are not queued behind this round's
        # partial / gradient exchanges on the current stream
        self.input_dist = input_comm if input_comm is not None else comm
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

    def _a2a(self, out, inp, out_splits=None, in_splits=None, comm=None):
        (comm or self.dist).all_to_all_single(out, inp, output_split_sizes=out_splits,
                                              input_split_sizes=in_splits, group=self.group)

    # ------------------------------------------------------------- lookup
    def prepare(self, feats: Sequence[FeatureInput], input_stream=None) -> "PreparedRound":
        """Partition + key exchange of a batch (PrepareLookupInputs and the ids'
        all-to-all), before its lookup.  Runs on `input_stream` (a stream on which
        the inputs are ready; default: the current stream) and touches no table
        state, so the next batch can be prepared while this round's push runs.
        Waits only for the partition counts, which size the exchange."""
        torch, n, F = self.torch, self.n, len(feats)
        main = self._stream()
        side = input_stream if (input_stream is not None and main is not None) else main
        dims = np.array([self.store.dimension(f.table) for f in feats], np.int64)
        pools = [int(f.pooling) for f in feats]
        tables = [int(f.table) for f in feats]
        with self._on(side):
            # ---- 1./2. partition (asynchronous) and the count rows, one per peer
            width = 5 * F + 1
            send_t = torch.empty((n, width), dtype=torch.int64, device=self.device)
            err, route = None, None
            try:
                route = self.store.route(feats, n, send_t, side)
            except EpsError as e:                  # host-side shape error: still exchange
                err = e
                host = np.zeros((n, width), np.int64)
                host[:, 2 * F:3 * F] = tables
                host[:, 3 * F:4 * F] = pools
                host[:, 5 * F] = -1
                send_t.copy_(torch.from_numpy(host))
            recv_t = torch.empty_like(send_t)
            self._a2a(recv_t, send_t, comm=self.input_dist)
            both = torch.stack([send_t, recv_t]).cpu().numpy()     # the one wait of a round
            mine, recv = both[0], both[1]
            schema = np.array(tables + pools, np.int64)
            bad_schema = bool((recv[:, 2 * F:4 * F] != schema[None, :]).any())
            own_bits = int(mine[0, 5 * F])
            if err is not None or own_bits or recv[:, 5 * F].any() or bad_schema:
                if route is not None:
                    self.store.route_release(route)
                if err is not None:
                    raise err
                if own_bits:
                    raise EpsError(INVALID_ARGUMENT, _input_message(own_bits))
                raise EpsError(INVALID_ARGUMENT, "a peer rank rejected its lookup inputs"
                               if not bad_schema else "ranks disagree on the feature schema")
            # [owner, f, (keys, kept, distinct)] / [requester, f, (...)]
            counts = np.concatenate([mine[:, :2 * F].reshape(n, F, 2),
                                     mine[:, 4 * F:5 * F].reshape(n, F, 1)], axis=2)
            peer = np.concatenate([recv[:, :2 * F].reshape(n, F, 2),
                                   recv[:, 4 * F:5 * F].reshape(n, F, 1)], axis=2)
            # ---- 3. payload: keys / offsets / valid lengths (/ distinct keys) per owner
            send_words = _words(counts)
            recv_words = _words(peer)
            payload = torch.empty(int(send_words.sum()), dtype=torch.int64, device=self.device)
            self.store.route_scatter(route, payload, side)
            rpay = torch.empty(int(recv_words.sum()), dtype=torch.int64, device=self.device)
            self._a2a(rpay, payload, recv_words.tolist(), send_words.tolist(), comm=self.input_dist)
            ready = torch.cuda.Event() if main is not None else None
            if ready is not None:
                ready.record(side)
        return PreparedRound(route, counts.astype(np.uint64), peer.astype(np.uint64), dims, pools,
                             tables, rpay, side, ready, [f.output_rows for f in feats],
                             _device_inputs(feats))

    def lookup_prepared(self, prep: "PreparedRound", outputs=None, read_only: bool = False):
        """Shard lookup + partial exchange + shard-ordered merge of a prepared
        batch (DistributedClient::LookupPrepared), on the current stream.
        Returns (handle, outputs)."""
        torch, n = self.torch, self.n
        main = self._stream()
        if prep.ready is not None and prep.side is not main:
            main.wait_event(prep.ready)
            prep.payload.record_stream(main)
            for t in prep.inputs:            # the merge reads the bag offsets on `main`
                t.record_stream(main)
        dims, pools = prep.dims, prep.pools
        seq = np.array([p == SEQUENCE for p in pools])
        prow = np.where(seq[None, :], prep.peer[:, :, 0], prep.peer[:, :, 1]).astype(np.int64)
        mrow = np.where(seq[None, :], prep.counts[:, :, 0], prep.counts[:, :, 1]).astype(np.int64)
        # partial rows: a deduplicated group returns its distinct rows
        pprow = np.where(prep.peer[:, :, 2] > 0, prep.peer[:, :, 2], prow).astype(np.int64)
        pmrow = np.where(prep.counts[:, :, 2] > 0, prep.counts[:, :, 2], mrow).astype(np.int64)
        send_f = (pprow * dims[None, :]).sum(axis=1)
        recv_f = (pmrow * dims[None, :]).sum(axis=1)
        # ---- 4. this shard's lookup over every requester's part (C++ layout)
        part_send = torch.empty(max(1, int(send_f.sum())), dtype=torch.float32, device=self.device)
        ticket = self.store.serve(prep.payload, prep.peer, prep.tables, pools, part_send,
                                  read_only=read_only, stream=main)
        # ---- 5. partials back to their requesters, merged in shard order
        part_recv = torch.empty(max(1, int(recv_f.sum())), dtype=torch.float32, device=self.device)
        self._a2a(part_recv[:int(recv_f.sum())], part_send[:int(send_f.sum())], recv_f.tolist(),
                  send_f.tolist())
        if outputs is None:
            outputs = [torch.empty((r, int(d)), dtype=torch.float32, device=self.device)
                       for r, d in zip(prep.output_rows, dims)]
        self.store.route_merge(prep.route, part_recv, outputs, main)
        handle = RoundHandle(prep.route, ticket, prep.counts, prep.peer, list(dims), pools,
                             read_only, prep.tables, send_f, recv_f,
                             (mrow * dims[None, :]).sum(axis=1), (prow * dims[None, :]).sum(axis=1),
                             mrow, prow)
        prep.route = None
        if read_only:
            self.store.route_release(handle.route)
            handle.route = None
        return handle, outputs

    def lookup(self, feats: Sequence[FeatureInput], outputs=None, read_only: bool = False,
               input_stream=None):
        """Sharded pull of this rank's features: prepare + lookup_prepared.
        Returns (handle, outputs)."""
        return self.lookup_prepared(self.prepare(feats, input_stream), outputs, read_only)

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
        torch = self.torch
        main = self._stream()
        # one gradient row per kept bag (or key) of every (shard, feature) block
        send_f, recv_f = handle.gsend_f, handle.grecv_f
        send = torch.empty(max(1, int(send_f.sum())), dtype=torch.float32, device=self.device)
        flag = torch.zeros(2, dtype=torch.int32, device=self.device)   # non-finite, max |g| bits
        self.store.route_gather(handle.route, gradients, send, flag, main)
        self.dist.all_reduce(flag, op=self.dist.ReduceOp.MAX, group=self.group)
        recv = torch.empty(max(1, int(recv_f.sum())), dtype=torch.float32, device=self.device)
        self._a2a(recv[:int(recv_f.sum())], send[:int(send_f.sum())], recv_f.tolist(),
                  send_f.tolist())
        # a rejected push with wait=True raises here and keeps the route and the
        # ticket (push again, or release); an enqueued push releases the route
        self.store.serve_push(handle.ticket, recv, handle.peer_counts, handle.tables,
                              handle.poolings, reject=flag, stream=main, wait=wait)
        self.store.route_release(handle.route)
        handle.route = None

    def discard(self, prep: PreparedRound):
        """Drops a prepared batch that will not be looked up (local; no exchange)."""
        if prep.route is not None:
            self.store.route_release(prep.route)
            prep.route = None

    def release(self, handle: RoundHandle):
        """Abandons a round: frees its route and this shard's ticket (Release)."""
        if handle.route is not None:
            self.store.route_release(handle.route)
            handle.route = None
        if handle.ticket is not None:
            self.store.release(handle.ticket)
            handle.ticket = None


class NcclComm:
    """The round's exchange over the library's NCCL communicator
    (eps_b200_comm_*), with the part of the torch.distributed API that
    ShardedClient uses.  Calls enqueue NCCL work on the caller's current
    stream; no extra streams or events are involved."""

    class ReduceOp:
        MAX = "max"

    def __init__(self, device: int, rank: int, world: int, unique_id: bytes):
        import torch
        self.torch = torch
        self.lib = load_library()
        self.device, self.rank, self.world = device, rank, world
        h = C.c_void_p()
        st = Status()
        uid = (C.c_uint8 * 128).from_buffer_copy(unique_id)
        _check(self.lib.eps_b200_comm_create(device, rank, world, uid, C.byref(h), C.byref(st)), st)
        self._h = h

    @staticmethod
    def unique_id() -> bytes:
        lib = load_library()
        buf = (C.c_uint8 * 128)()
        st = Status()
        _check(lib.eps_b200_comm_unique_id(buf, C.byref(st)), st)
        return bytes(buf)

    @classmethod
    def from_process_group(cls, device: int, group=None):
        """Bootstraps over an existing torch.distributed group (rank 0 makes the id)."""
        import torch.distributed as dist
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        box = [cls.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0, group=group)
        return cls(device, rank, world, box[0])

    def close(self):
        if getattr(self, "_h", None):
            self.lib.eps_b200_comm_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def get_rank(self, group=None):
        return self.rank

    def get_world_size(self, group=None):
        return self.world

    def _stream(self):
        return self.torch.cuda.current_stream(self.device).cuda_stream

    def all_to_all_single(self, out, inp, output_split_sizes=None, input_split_sizes=None,
                          group=None):
        n = self.world
        ins = input_split_sizes if input_split_sizes is not None else [inp.shape[0] // n] * n
        outs = output_split_sizes if output_split_sizes is not None else [out.shape[0] // n] * n
        rest_in = int(np.prod(inp.shape[1:])) if inp.dim() > 1 else 1
        rest_out = int(np.prod(out.shape[1:])) if out.dim() > 1 else 1
        sc = np.asarray(ins, np.uint64) * np.uint64(rest_in)
        rc = np.asarray(outs, np.uint64) * np.uint64(rest_out)
        st = Status()
        _check(self.lib.eps_b200_comm_alltoallv(self._h, inp.data_ptr(), sc.ctypes.data,
                                                out.data_ptr(), rc.ctypes.data,
                                                inp.element_size(), self._stream(),
                                                C.byref(st)), st)

    def all_reduce(self, t, op=None, group=None):
        if t.element_size() != 4:
            raise EpsError(INVALID_ARGUMENT, "all_reduce supports 32-bit flags only")
        st = Status()
        _check(self.lib.eps_b200_comm_allreduce_max(self._h, t.data_ptr(), t.numel(),
                                                    self._stream(), C.byref(st)), st)


class NativeClient:
    """The round's host side in C++ (eps_b200_client_*): the same protocol as
    ShardedClient, one library call per phase, NCCL on the caller's streams.
    This is the path the benchmark measures."""

    def __init__(self, store, comm: NcclComm, input_comm: NcclComm | None = None):
        import torch
        self.torch = torch
        self.store = store
        self.lib = load_library()
        self._comms = (comm, input_comm)          # keep the communicators alive
        h = C.c_void_p()
        st = Status()
        _check(self.lib.eps_b200_client_create(store._h, comm._h,
                                               input_comm._h if input_comm else None,
                                               C.byref(h), C.byref(st)), st)
        self._h = h
        self._keep = {}

    def close(self):
        if getattr(self, "_h", None):
            self.lib.eps_b200_client_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _stream(self, stream):
        if stream is None:
            stream = self.torch.cuda.current_stream(self.store.device)
        return stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)

    def prepare(self, feats: Sequence[FeatureInput], input_stream=None) -> int:
        arr, on_device, keep = self.store._features(feats)
        if not on_device:
            raise EpsError(INVALID_ARGUMENT, "a sharded round needs device inputs")
        pid = C.c_uint64(0)
        st = Status()
        _check(self.lib.eps_b200_client_prepare(self._h, arr, len(feats),
                                                self._stream(input_stream), C.byref(pid),
                                                C.byref(st)), st)
        self._keep[pid.value] = (keep, [f.output_rows for f in feats],
                                 [self.store.dimension(f.table) for f in feats],
                                 _device_inputs(feats))
        return pid.value

    def lookup_prepared(self, prepared: int, outputs=None, read_only: bool = False, stream=None):
        keep, rows, dims, inputs = self._keep.pop(prepared)
        main = stream if stream is not None else self.torch.cuda.current_stream(self.store.device)
        for t in inputs:                     # the merge reads the bag offsets on `main`
            t.record_stream(main)
        if outputs is None:
            outputs = [self.torch.empty((r, d), dtype=self.torch.float32,
                                        device=f"cuda:{self.store.device}")
                       for r, d in zip(rows, dims)]
        bufs = self.store._buffers(outputs)
        rid = C.c_uint64(0)
        st = Status()
        _check(self.lib.eps_b200_client_lookup(self._h, prepared, bufs, int(read_only),
                                               self._stream(stream), C.byref(rid), C.byref(st)),
               st)
        return (None if read_only else rid.value), outputs

    def lookup(self, feats: Sequence[FeatureInput], outputs=None, read_only: bool = False,
               input_stream=None):
        return self.lookup_prepared(self.prepare(feats, input_stream), outputs, read_only)

    def push(self, round_id: int, gradients, wait: bool = False, stream=None):
        st = Status()
        _check(self.lib.eps_b200_client_push(self._h, round_id, self.store._buffers(gradients),
                                             self._stream(stream), int(wait), C.byref(st)), st)

    EXCHANGES = ("counts", "keys", "partials", "gradients")

    def profile(self, mode: int = -1) -> dict:
        """eps_b200_client_profile: per exchange {ms, bytes, calls} (mode 1
        resets and starts timing, 0 stops)."""
        ms = (C.c_double * 4)()
        by = (C.c_uint64 * 4)()
        ca = (C.c_uint64 * 4)()
        st = Status()
        _check(self.lib.eps_b200_client_profile(self._h, mode, ms, by, ca, C.byref(st)), st)
        return {k: {"ms": ms[i], "bytes": by[i], "calls": ca[i]} for i, k in enumerate(self.EXCHANGES)}

    def release(self, handle: int):
        """Drops a prepared batch or an unpushed round."""
        self._keep.pop(handle, None)
        st = Status()
        _check(self.lib.eps_b200_client_release(self._h, handle, C.byref(st)), st)

    discard = release
