"""Python binding of the B200 embedding parameter store (libeps_b200.so).

Mirrors the reference parameter server's shard/client interface
(include/eps/parameter_service.hpp, include/eps/distributed_client.hpp):

    store = ParameterStore(device=0)
    store.create_table(TableDefinition(id=1, dimension=64, ...))
    ticket, outputs = store.lookup([FeatureInput(table=1, feature=0, pooling=SUM,
                                                 keys=..., offsets=...)])
    store.push(ticket, gradients)          # coalesce + segment-sum + LazyAdam
    store.release(ticket)                  # for an abandoned lookup

Host (numpy) and device (torch CUDA tensor) inputs are both accepted; the
library itself runs only the hand-written sm_100a kernels.  There is no CPU
fallback: importing this package fails loudly if the native library is missing,
and every call fails with the library's own error when no GPU is present.
Errors raise ``EpsError`` whose ``code`` is eps::Error::Code + 1
(include/eps/types.hpp:17-25).
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass
from typing import Sequence

import numpy as np

__all__ = ["ParameterStore", "TableDefinition", "FeatureInput", "EpsError", "SUM", "MEAN",
           "SEQUENCE", "library_path", "load_library"]

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(HERE, "libeps_b200.so")

SUM, MEAN, SEQUENCE = 0, 1, 2
INVALID_ARGUMENT, UNAVAILABLE, STALE_GENERATION, RETIRED_REQUEST, CAPACITY_EXCEEDED, RUN_FAILED = range(1, 7)


def library_path() -> str:
    return _LIB_PATH


class EpsError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code
        self.message = message


# ------------------------------------------------------------------ C structs
class Status(C.Structure):
    _fields_ = [("code", C.c_int32), ("message", C.c_char * 1024)]


class Options(C.Structure):
    _fields_ = [("device", C.c_int32), ("shard_id", C.c_uint32), ("shard_count", C.c_uint32),
                ("max_live_tickets", C.c_uint32), ("partition_epoch", C.c_uint64),
                ("state_bytes", C.c_uint64), ("flags", C.c_uint32),
                ("max_enqueued_pushes", C.c_uint32)]


FLAG_REFERENCE_ORDER = 1
FLAG_REGISTER_ROWS = 2


class Table(C.Structure):
    _fields_ = [("id", C.c_uint32), ("dimension", C.c_uint32), ("shard_count", C.c_uint32),
                ("has_weight_bounds", C.c_int32), ("partition_epoch", C.c_uint64),
                ("learning_rate", C.c_float), ("beta1", C.c_float), ("beta2", C.c_float),
                ("epsilon", C.c_float), ("initial_beta1_power", C.c_float),
                ("initial_beta2_power", C.c_float), ("weight_min", C.c_float),
                ("weight_max", C.c_float), ("initialization_min", C.c_float),
                ("initialization_max", C.c_float), ("initialization_seed", C.c_uint64),
                ("key_space", C.c_uint64), ("capacity", C.c_uint64)]


class Feature(C.Structure):
    _fields_ = [("table", C.c_uint32), ("feature", C.c_uint32), ("pooling", C.c_uint32),
                ("has_padding", C.c_uint32), ("keys", C.c_void_p), ("key_count", C.c_uint64),
                ("offsets", C.c_void_p), ("offset_count", C.c_uint64),
                ("valid_lengths", C.c_void_p), ("padding_key", C.c_uint64)]


class Buffer(C.Structure):
    _fields_ = [("feature", C.c_uint32), ("reserved", C.c_uint32), ("rows", C.c_uint64),
                ("columns", C.c_uint64), ("data", C.c_void_p), ("device", C.c_int32),
                ("reserved2", C.c_int32)]


class WorkerGradients(C.Structure):
    _fields_ = [("keys", C.c_void_p), ("values", C.c_void_p), ("rows", C.c_uint64),
                ("sample_count", C.c_uint64)]


REDUCE_SUM, REDUCE_WORKER_MEAN, REDUCE_SAMPLE_MEAN = 0, 1, 2


class UpdateContext(C.Structure):
    _fields_ = [("table", C.c_uint32), ("learning_rate", C.c_float), ("beta1_power", C.c_float),
                ("beta2_power", C.c_float), ("optimizer_sequence", C.c_uint64)]


class CompactGradients(C.Structure):
    _fields_ = [("keys", C.c_void_p), ("rows", C.c_uint64), ("dimension", C.c_uint32),
                ("source_values", C.c_void_p), ("sources", C.c_uint64),
                ("row_offsets", C.c_void_p), ("source_rows", C.c_void_p), ("scales", C.c_void_p),
                ("refs", C.c_uint64)]


class SnapshotInfo(C.Structure):
    _fields_ = [("format", C.c_uint32), ("run", C.c_char * 1025), ("shard", C.c_uint64),
                ("shard_count", C.c_uint64), ("partition_epoch", C.c_uint64),
                ("checksum", C.c_uint64), ("tables", C.c_uint64)]


class Stats(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in ("lookups", "updates", "rejected_updates",
                                          "duplicate_requests", "live_tickets", "state_bytes",
                                          "rows", "tables", "kernel_launches")]


PHASES = ("lookup", "sort", "prescan", "apply", "finalize", "emit", "pieces", "long")


_lib = None

class SnapshotTable(C.Structure):
    _fields_ = [("definition", Table), ("optimizer_sequence", C.c_uint64),
                ("beta1_power", C.c_float), ("beta2_power", C.c_float), ("rows", C.c_uint64)]


ENTRY_POINTS = ("eps_b200_abi_version", "eps_b200_create", "eps_b200_destroy",
                "eps_b200_create_table", "eps_b200_lookup", "eps_b200_lookup_noalloc",
                "eps_b200_push", "eps_b200_release", "eps_b200_ticket_coalesced",
                "eps_b200_synchronize", "eps_b200_read_state", "eps_b200_load_state",
                "eps_b200_optimizer_state", "eps_b200_profile", "eps_b200_stats",
                "eps_b200_route", "eps_b200_route_scatter", "eps_b200_route_merge",
                "eps_b200_route_gather", "eps_b200_route_release", "eps_b200_serve",
                "eps_b200_serve_push", "eps_b200_comm_unique_id", "eps_b200_comm_create",
                "eps_b200_comm_destroy", "eps_b200_comm_alltoallv", "eps_b200_comm_allreduce_max",
                "eps_b200_client_create", "eps_b200_client_destroy", "eps_b200_client_prepare",
                "eps_b200_client_lookup", "eps_b200_client_push", "eps_b200_client_release",
                "eps_b200_client_profile",
                "eps_b200_sync_reduce", "eps_b200_apply_rows", "eps_b200_apply_compact",
                "eps_b200_snapshot_write", "eps_b200_snapshot_read", "eps_b200_snapshot_inspect",
                "eps_b200_snapshot_rows")


def load_library() -> C.CDLL:
    """Loads libeps_b200.so; raises if it has not been built (no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        raise ImportError(f"{_LIB_PATH} is missing: build it with `python build.py` "
                          "(there is no non-CUDA fallback)")
    lib = C.CDLL(_LIB_PATH)
    P = C.POINTER
    vp = C.c_void_p
    lib.eps_b200_abi_version.restype = C.c_uint32
    lib.eps_b200_create.argtypes = [P(Options), P(vp), P(Status)]
    lib.eps_b200_destroy.argtypes = [vp]
    lib.eps_b200_destroy.restype = None
    lib.eps_b200_create_table.argtypes = [vp, P(Table), P(Status)]
    lib.eps_b200_lookup.argtypes = [vp, P(Feature), C.c_uint64, C.c_int32, C.c_int32, C.c_int32,
                                    P(Buffer), vp, P(C.c_uint64), P(Status)]
    lib.eps_b200_lookup_noalloc.argtypes = [vp, P(Feature), C.c_uint64, P(Buffer), vp, P(Status)]
    lib.eps_b200_push.argtypes = [vp, C.c_uint64, P(Buffer), C.c_uint64, vp, C.c_int32, P(Status)]
    lib.eps_b200_release.argtypes = [vp, C.c_uint64, P(Status)]
    lib.eps_b200_ticket_coalesced.argtypes = [vp, C.c_uint64, vp, vp, vp, vp, vp, vp, C.c_uint64,
                                              C.c_uint64, P(C.c_uint64), P(C.c_uint64), P(Status)]
    lib.eps_b200_synchronize.argtypes = [vp, P(Status)]
    lib.eps_b200_read_state.argtypes = [vp, C.c_uint32, vp, C.c_uint64, vp, vp, vp, vp, P(Status)]
    lib.eps_b200_load_state.argtypes = [vp, C.c_uint32, vp, C.c_uint64, vp, vp, vp, vp, P(Status)]
    lib.eps_b200_optimizer_state.argtypes = [vp, C.c_uint32, P(C.c_uint64), P(C.c_float),
                                             P(C.c_float), P(Status)]
    lib.eps_b200_stats.argtypes = [vp, P(Stats), P(Status)]
    lib.eps_b200_profile.argtypes = [vp, C.c_int32, P(C.c_double), P(C.c_uint64), P(C.c_uint64),
                                     P(Status)]
    lib.eps_b200_route.argtypes = [vp, P(Feature), C.c_uint64, C.c_uint32, vp, P(C.c_uint64), vp,
                                   P(Status)]
    lib.eps_b200_route_scatter.argtypes = [vp, C.c_uint64, vp, vp, P(Status)]
    lib.eps_b200_route_merge.argtypes = [vp, C.c_uint64, vp, P(Buffer), vp, P(Status)]
    lib.eps_b200_route_gather.argtypes = [vp, C.c_uint64, P(Buffer), vp, vp, vp, P(Status)]
    lib.eps_b200_route_release.argtypes = [vp, C.c_uint64, P(Status)]
    lib.eps_b200_serve.argtypes = [vp, vp, vp, vp, vp, C.c_uint32, C.c_uint32, C.c_int32, vp, vp,
                                   P(C.c_uint64), P(Status)]
    lib.eps_b200_serve_push.argtypes = [vp, C.c_uint64, vp, vp, vp, vp, C.c_uint32, C.c_uint32, vp,
                                        vp, C.c_int32, P(Status)]
    lib.eps_b200_comm_unique_id.argtypes = [vp, P(Status)]
    lib.eps_b200_comm_create.argtypes = [C.c_int32, C.c_uint32, C.c_uint32, vp, P(vp), P(Status)]
    lib.eps_b200_comm_destroy.argtypes = [vp]
    lib.eps_b200_comm_destroy.restype = None
    lib.eps_b200_comm_alltoallv.argtypes = [vp, vp, vp, vp, vp, C.c_uint32, vp, P(Status)]
    lib.eps_b200_comm_allreduce_max.argtypes = [vp, vp, C.c_uint64, vp, P(Status)]
    lib.eps_b200_client_create.argtypes = [vp, vp, vp, P(vp), P(Status)]
    lib.eps_b200_client_destroy.argtypes = [vp]
    lib.eps_b200_client_destroy.restype = None
    lib.eps_b200_client_prepare.argtypes = [vp, P(Feature), C.c_uint64, vp, P(C.c_uint64), P(Status)]
    lib.eps_b200_client_lookup.argtypes = [vp, C.c_uint64, P(Buffer), C.c_int32, vp,
                                           P(C.c_uint64), P(Status)]
    lib.eps_b200_client_push.argtypes = [vp, C.c_uint64, P(Buffer), vp, C.c_int32, P(Status)]
    lib.eps_b200_client_release.argtypes = [vp, C.c_uint64, P(Status)]
    lib.eps_b200_client_profile.argtypes = [vp, C.c_int32, P(C.c_double), P(C.c_uint64),
                                            P(C.c_uint64), P(Status)]
    lib.eps_b200_sync_reduce.argtypes = [vp, C.c_uint32, vp, C.c_uint32, C.c_int32, vp, vp,
                                         C.c_uint64, P(C.c_uint64), vp, P(Status)]
    lib.eps_b200_apply_rows.argtypes = [vp, P(UpdateContext), vp, C.c_uint64, vp, C.c_int32, vp,
                                        P(Status)]
    lib.eps_b200_apply_compact.argtypes = [vp, P(UpdateContext), P(CompactGradients), vp, P(Status)]
    lib.eps_b200_snapshot_write.argtypes = [vp, C.c_char_p, C.c_char_p, C.c_int32, P(Status)]
    lib.eps_b200_snapshot_read.argtypes = [vp, C.c_char_p, C.c_char_p, P(Status)]
    lib.eps_b200_snapshot_inspect.argtypes = [C.c_char_p, P(SnapshotInfo), vp, C.c_uint64, P(Status)]
    lib.eps_b200_snapshot_rows.argtypes = [C.c_char_p, C.c_uint64, vp, vp, vp, C.c_uint64, P(Status)]
    for name in ENTRY_POINTS[1:]:
        if name not in ("eps_b200_destroy", "eps_b200_comm_destroy", "eps_b200_client_destroy"):
            getattr(lib, name).restype = C.c_int
    if lib.eps_b200_abi_version() != 3:
        raise ImportError("libeps_b200.so ABI version mismatch")
    _lib = lib
    return lib


load_library()


# ----------------------------------------------------------- python mirror
@dataclass
class TableDefinition:
    """eps::TableDefinition + OptimizerConfig (include/eps/types.hpp:76-97).

    key_space > 0: a dense table of keys [0, key_space).  key_space == 0: a hashed
    table -- any 64-bit key, rows created on first touch (ShardStore::Ensure,
    src/store/shard_store.cpp:76-115), at most `capacity` rows on this shard."""
    id: int
    dimension: int
    key_space: int
    learning_rate: float = 1e-3
    beta1: float = 0.9
    beta2: float = 0.999
    epsilon: float = 1e-8
    initial_beta1_power: float = 0.9
    initial_beta2_power: float = 0.999
    weight_bounds: tuple | None = None
    initialization_min: float = -0.05
    initialization_max: float = 0.05
    initialization_seed: int = 42
    shard_count: int = 1
    partition_epoch: int = 1
    capacity: int = 0


@dataclass
class FeatureInput:
    """eps::FeatureInput (include/eps/types.hpp:99-107).

    keys/offsets/valid_lengths are uint64 numpy arrays (host) or int64/uint64
    torch CUDA tensors (device).  valid_lengths=None means offset differences.
    padding_key: keys equal to it are dropped as in PrepareAdapterInput
    (src/access/prepare_queue.cpp:58-85); sequence positions holding it read 0.
    """
    table: int
    feature: int
    pooling: int
    keys: object
    offsets: object
    valid_lengths: object = None
    padding_key: int | None = None     # keys equal to it are dropped (adapter padding)

    @property
    def output_rows(self) -> int:
        return _length(self.keys) if self.pooling == SEQUENCE else _length(self.offsets) - 1


def _length(a) -> int:
    return int(a.shape[0]) if hasattr(a, "shape") else len(a)


def _is_device(a) -> bool:
    return hasattr(a, "is_cuda") and a.is_cuda


def _ptr(a):
    if a is None:
        return None
    if _is_device(a):
        return a.data_ptr()
    return a.ctypes.data


def _host_u64(a):
    return np.ascontiguousarray(a, dtype=np.uint64)


def _check(rc: int, status: Status):
    if rc:
        raise EpsError(rc, status.message.decode(errors="replace"))


class ParameterStore:
    """One shard of device-resident embedding tables (eps_b200_create)."""

    def __init__(self, device: int = 0, shard_id: int = 0, shard_count: int = 1,
                 state_bytes: int = 64 << 30, max_live_tickets: int = 1024,
                 partition_epoch: int = 1, reference_order: bool = False,
                 register_rows: bool = False, max_enqueued_pushes: int = 0):
        self.lib = load_library()
        self.device = device
        self.shard_count = shard_count
        self._tables: dict[int, TableDefinition] = {}
        opt = Options(device, shard_id, shard_count, max_live_tickets, partition_epoch, state_bytes,
                      (FLAG_REFERENCE_ORDER if reference_order else 0) |
                      (FLAG_REGISTER_ROWS if register_rows else 0), max_enqueued_pushes)
        st = Status()
        h = C.c_void_p()
        _check(self.lib.eps_b200_create(C.byref(opt), C.byref(h), C.byref(st)), st)
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            self.lib.eps_b200_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # ParameterService::CreateTable (include/eps/parameter_service.hpp:16)
    def create_table(self, t: TableDefinition):
        b = t.weight_bounds
        ct = Table(t.id, t.dimension, t.shard_count, 1 if b else 0, t.partition_epoch,
                   t.learning_rate, t.beta1, t.beta2, t.epsilon, t.initial_beta1_power,
                   t.initial_beta2_power, *(b if b else (0.0, 0.0)), t.initialization_min,
                   t.initialization_max, t.initialization_seed, t.key_space, t.capacity)
        st = Status()
        _check(self.lib.eps_b200_create_table(self._h, C.byref(ct), C.byref(st)), st)
        self._tables[t.id] = t

    def _features(self, feats: Sequence[FeatureInput]):
        on_device = None
        keep = []
        arr = (Feature * len(feats))()
        for i, f in enumerate(feats):
            dev = _is_device(f.keys)
            if on_device is None:
                on_device = dev
            if dev != on_device or _is_device(f.offsets) != dev:
                raise EpsError(INVALID_ARGUMENT, "mixed host/device lookup inputs")
            keys, offs, lens = f.keys, f.offsets, f.valid_lengths
            if not dev:
                keys, offs = _host_u64(keys), _host_u64(offs)
                lens = None if lens is None else _host_u64(lens)
            keep += [keys, offs, lens]
            pad = getattr(f, "padding_key", None)
            arr[i] = Feature(f.table, f.feature, f.pooling, 0 if pad is None else 1, _ptr(keys),
                             _length(keys), _ptr(offs), _length(offs), _ptr(lens),
                             0 if pad is None else int(pad))
        return arr, bool(on_device), keep

    def lookup(self, feats: Sequence[FeatureInput], read_only: bool = False,
               shard_partial: bool = False, outputs=None, stream=None, host_outputs=None):
        """Pull.  Returns (ticket or None, outputs).  Device inputs give torch
        CUDA outputs unless `outputs` is supplied; host inputs give numpy."""
        arr, on_device, keep = self._features(feats)
        if host_outputs is None:
            host_outputs = not on_device
        if outputs is None:
            outputs = []
            for f in feats:
                if f.table not in self._tables:
                    raise EpsError(INVALID_ARGUMENT, "unknown table")
                shape = (f.output_rows, self._tables[f.table].dimension)
                if host_outputs:
                    outputs.append(np.empty(shape, np.float32))
                else:
                    import torch
                    outputs.append(torch.empty(shape, dtype=torch.float32,
                                               device=f"cuda:{self.device}"))
        bufs = (Buffer * len(feats))()
        for i, (f, o) in enumerate(zip(feats, outputs)):
            dev = _is_device(o)
            bufs[i] = Buffer(f.feature, 0, int(o.shape[0]), int(o.shape[1]), _ptr(o),
                             self.device if dev else -1, 0)
        ticket = C.c_uint64(0)
        st = Status()
        rc = self.lib.eps_b200_lookup(self._h, arr, len(feats), int(on_device), int(read_only),
                                      int(shard_partial), bufs, _stream_ptr(stream),
                                      C.byref(ticket), C.byref(st))
        _check(rc, st)
        del keep
        return (None if read_only else ticket.value), outputs

    def lookup_noalloc(self, feats: Sequence[FeatureInput], outputs, stream=None):
        """Read-only pooled lookup through eps_b200_lookup_noalloc: writes the
        given device output tensors and allocates no device memory (for callers
        whose serving path may not allocate; at most 256 features per call).
        Input errors surface at the next synchronize()."""
        arr, on_device, keep = self._features(feats)
        if not on_device:
            raise EpsError(INVALID_ARGUMENT, "the allocation-free lookup needs device inputs")
        bufs = (Buffer * len(feats))()
        for i, (f, o) in enumerate(zip(feats, outputs)):
            bufs[i] = Buffer(f.feature, 0, int(o.shape[0]), int(o.shape[1]), _ptr(o),
                             self.device if _is_device(o) else -1, 0)
        st = Status()
        rc = self.lib.eps_b200_lookup_noalloc(self._h, arr, len(feats), bufs,
                                              _stream_ptr(stream), C.byref(st))
        _check(rc, st)
        del keep
        return outputs

    def prepare_lookup(self, feats: Sequence[FeatureInput], outputs, read_only=False,
                       shard_partial=False):
        """Binds inputs/outputs once; the returned callable runs eps_b200_lookup
        with no per-call Python marshalling (for steady-state loops).
        outputs=None binds a push-only lookup (occurrence list and coalescing
        sort, no gather)."""
        arr, on_device, keep = self._features(feats)
        bufs = None
        if outputs is not None:
            bufs = (Buffer * len(feats))()
            for i, (f, o) in enumerate(zip(feats, outputs)):
                dev = _is_device(o)
                bufs[i] = Buffer(f.feature, 0, int(o.shape[0]), int(o.shape[1]), _ptr(o),
                                 self.device if dev else -1, 0)
        ticket = C.c_uint64(0)
        st = Status()
        lib, h, n = self.lib, self._h, len(feats)
        ro, sp, od = int(read_only), int(shard_partial), int(on_device)

        def run(stream=None):
            rc = lib.eps_b200_lookup(h, arr, n, od, ro, sp, bufs, _stream_ptr(stream),
                                     C.byref(ticket), C.byref(st))
            _check(rc, st)
            return ticket.value

        run._keep = (arr, bufs, keep, outputs)
        return run

    def prepare_push(self, gradients, features: Sequence[int] | None = None):
        """Binds gradient buffers once; returns push(ticket, stream=None, wait=False)."""
        n = len(gradients)
        bufs = (Buffer * n)()
        keep = []
        for i, g in enumerate(gradients):
            dev = _is_device(g)
            if not dev:
                g = np.ascontiguousarray(g, dtype=np.float32)
            keep.append(g)
            fid = features[i] if features is not None else i
            bufs[i] = Buffer(fid, 0, int(g.shape[0]), int(g.shape[1]), _ptr(g),
                             self.device if dev else -1, 0)
        st = Status()
        lib, h = self.lib, self._h

        def run(ticket, stream=None, wait=False):
            _check(lib.eps_b200_push(h, ticket, bufs, n, _stream_ptr(stream), int(wait),
                                     C.byref(st)), st)

        run._keep = (bufs, keep)
        return run

    def push(self, ticket: int, gradients, features: Sequence[int] | None = None,
             wait: bool = True, stream=None):
        """Push feature gradients (ordered like the lookup's features, or with
        explicit feature ids).  All-or-nothing; raises EpsError on rejection."""
        n = len(gradients)
        bufs = (Buffer * n)()
        keep = []
        for i, g in enumerate(gradients):
            dev = _is_device(g)
            if not dev:
                g = np.ascontiguousarray(g, dtype=np.float32)
            keep.append(g)
            fid = features[i] if features is not None else i
            bufs[i] = Buffer(fid, 0, int(g.shape[0]), int(g.shape[1]), _ptr(g),
                             self.device if dev else -1, 0)
        st = Status()
        rc = self.lib.eps_b200_push(self._h, ticket, bufs, n, _stream_ptr(stream), int(wait),
                                    C.byref(st))
        _check(rc, st)

    def release(self, ticket: int):
        st = Status()
        _check(self.lib.eps_b200_release(self._h, ticket, C.byref(st)), st)

    def coalesced(self, ticket: int):
        """The ticket's coalesced rows as CompactGradients CSR
        (eps_b200_ticket_coalesced): dict of tables, keys, row_offsets and per
        reference feature, source row and scale."""
        rows, refs = C.c_uint64(0), C.c_uint64(0)
        st = Status()
        _check(self.lib.eps_b200_ticket_coalesced(self._h, ticket, None, None, None, None, None,
                                                  None, 0, 0, C.byref(rows), C.byref(refs),
                                                  C.byref(st)), st)
        U, R = rows.value, refs.value
        out = {"tables": np.zeros(U, np.uint32), "keys": np.zeros(U, np.uint64),
               "row_offsets": np.zeros(U + 1, np.uint64), "features": np.zeros(R, np.uint32),
               "sources": np.zeros(R, np.uint64), "scales": np.zeros(R, np.float32)}
        _check(self.lib.eps_b200_ticket_coalesced(
            self._h, ticket, _ptr(out["tables"]), _ptr(out["keys"]), _ptr(out["row_offsets"]),
            _ptr(out["features"]), _ptr(out["sources"]), _ptr(out["scales"]), U, R,
            C.byref(rows), C.byref(refs), C.byref(st)), st)
        return out

    def synchronize(self):
        st = Status()
        _check(self.lib.eps_b200_synchronize(self._h, C.byref(st)), st)

    def read_state(self, table: int, keys):
        keys = _host_u64(keys)
        if table not in self._tables:
            raise EpsError(INVALID_ARGUMENT, "unknown table")
        d = self._tables[table].dimension
        w = np.empty((len(keys), d), np.float32)
        m = np.empty_like(w)
        v = np.empty_like(w)
        upd = np.empty(len(keys), np.uint64)
        st = Status()
        _check(self.lib.eps_b200_read_state(self._h, table, _ptr(keys), len(keys), _ptr(w),
                                            _ptr(m), _ptr(v), _ptr(upd), C.byref(st)), st)
        return w, m, v, upd

    def load_state(self, table: int, keys, weights, first, second, row_updates=None):
        keys = _host_u64(keys)
        w = np.ascontiguousarray(weights, np.float32)
        m = np.ascontiguousarray(first, np.float32)
        v = np.ascontiguousarray(second, np.float32)
        u = None if row_updates is None else _host_u64(row_updates)
        st = Status()
        _check(self.lib.eps_b200_load_state(self._h, table, _ptr(keys), len(keys), _ptr(w),
                                            _ptr(m), _ptr(v), _ptr(u), C.byref(st)), st)

    def optimizer_state(self, table: int):
        seq = C.c_uint64()
        b1 = C.c_float()
        b2 = C.c_float()
        st = Status()
        _check(self.lib.eps_b200_optimizer_state(self._h, table, C.byref(seq), C.byref(b1),
                                                 C.byref(b2), C.byref(st)), st)
        return seq.value, b1.value, b2.value

    def profile(self, mode: int = -1) -> dict:
        """Per-phase device milliseconds / kernel launches / calls; mode 1 resets
        and starts recording, 0 stops (eps_b200_profile)."""
        n = len(PHASES)
        ms = (C.c_double * n)()
        la = (C.c_uint64 * n)()
        ca = (C.c_uint64 * n)()
        st = Status()
        _check(self.lib.eps_b200_profile(self._h, mode, ms, la, ca, C.byref(st)), st)
        return {p: {"ms": ms[i], "launches": la[i], "calls": ca[i]} for i, p in enumerate(PHASES)}

    # ---- client side of a multi-GPU round (see distributed.ShardedClient)
    def dimension(self, table: int) -> int:
        if table not in self._tables:
            raise EpsError(INVALID_ARGUMENT, "unknown table")
        return self._tables[table].dimension

    def route(self, feats: Sequence[FeatureInput], shard_count: int, counts, stream=None):
        """Partitions device features by key % shard_count (eps_b200_route,
        asynchronous).  `counts` is a device int64 tensor [shard_count,
        5 * len(feats) + 1] that receives the per-shard count rows.  Returns the
        route id."""
        arr, on_device, keep = self._features(feats)
        if not on_device:
            raise EpsError(INVALID_ARGUMENT, "a route needs device inputs")
        rid = C.c_uint64(0)
        st = Status()
        _check(self.lib.eps_b200_route(self._h, arr, len(feats), shard_count, _stream_ptr(stream),
                                       C.byref(rid), _ptr(counts), C.byref(st)), st)
        self._route_keep = getattr(self, "_route_keep", {})
        self._route_keep[rid.value] = keep
        return rid.value

    def route_scatter(self, route: int, payload, stream=None):
        st = Status()
        _check(self.lib.eps_b200_route_scatter(self._h, route, _ptr(payload), _stream_ptr(stream),
                                               C.byref(st)), st)

    def _buffers(self, tensors, rows_cols=None):
        bufs = (Buffer * len(tensors))()
        for i, t in enumerate(tensors):
            bufs[i] = Buffer(i, 0, int(t.shape[0]), int(t.shape[1]), _ptr(t),
                             self.device if _is_device(t) else -1, 0)
        return bufs

    def route_merge(self, route: int, partials, outputs, stream=None):
        st = Status()
        _check(self.lib.eps_b200_route_merge(self._h, route, _ptr(partials), self._buffers(outputs),
                                             _stream_ptr(stream), C.byref(st)), st)

    def route_gather(self, route: int, gradients, send, nonfinite=None, stream=None):
        st = Status()
        _check(self.lib.eps_b200_route_gather(self._h, route, self._buffers(gradients), _ptr(send),
                                              _ptr(nonfinite), _stream_ptr(stream), C.byref(st)), st)

    @staticmethod
    def _schema(peer_counts, tables, poolings):
        pc = np.ascontiguousarray(peer_counts, dtype=np.uint64)
        tb = np.ascontiguousarray(tables, dtype=np.uint32)
        po = np.ascontiguousarray(poolings, dtype=np.uint32)
        return pc, tb, po, int(pc.shape[0]), int(tb.shape[0])

    def serve(self, payload, peer_counts, tables, poolings, partials, read_only=False,
              stream=None):
        """Owner side of a sharded round (eps_b200_serve); returns the ticket."""
        pc, tb, po, n, F = self._schema(peer_counts, tables, poolings)
        ticket = C.c_uint64(0)
        st = Status()
        _check(self.lib.eps_b200_serve(self._h, _ptr(payload), _ptr(pc), _ptr(tb), _ptr(po), n, F,
                                       int(read_only), _ptr(partials), _stream_ptr(stream),
                                       C.byref(ticket), C.byref(st)), st)
        return None if read_only else ticket.value

    def serve_push(self, ticket, gradients, peer_counts, tables, poolings, reject=None,
                   stream=None, wait=False):
        """Owner side of a sharded push (eps_b200_serve_push)."""
        pc, tb, po, n, F = self._schema(peer_counts, tables, poolings)
        st = Status()
        _check(self.lib.eps_b200_serve_push(self._h, ticket, _ptr(gradients), _ptr(pc), _ptr(tb),
                                            _ptr(po), n, F, _ptr(reject), _stream_ptr(stream),
                                            int(wait), C.byref(st)), st)

    def route_release(self, route: int):
        st = Status()
        _check(self.lib.eps_b200_route_release(self._h, route, C.byref(st)), st)
        getattr(self, "_route_keep", {}).pop(route, None)

    # ---- snapshots (DrainAndFlush / Restore, src/store/snapshot.cpp format)
    def snapshot_write(self, path: str, run: str, all_rows: bool = False):
        st = Status()
        _check(self.lib.eps_b200_snapshot_write(self._h, str(path).encode(), run.encode(),
                                                int(all_rows), C.byref(st)), st)

    def snapshot_read(self, path: str, new_run: str):
        st = Status()
        _check(self.lib.eps_b200_snapshot_read(self._h, str(path).encode(), new_run.encode(),
                                               C.byref(st)), st)

    # ---- agent-style updates (CacheBackend::ApplyHost / ApplyCompact)
    def apply_rows(self, table: int, keys, values, learning_rate: float, beta1_power: float,
                   beta2_power: float, optimizer_sequence: int = 0, stream=None):
        """LazyAdam on unique rows with an external optimizer context
        (eps_b200_apply_rows); values: numpy [rows, dim] or a device tensor."""
        keys = _host_u64(keys)
        dev = _is_device(values)
        if not dev:
            values = np.ascontiguousarray(values, dtype=np.float32)
        ctx = UpdateContext(table, learning_rate, beta1_power, beta2_power, optimizer_sequence)
        st = Status()
        _check(self.lib.eps_b200_apply_rows(self._h, C.byref(ctx), _ptr(keys), len(keys),
                                            _ptr(values), int(dev), _stream_ptr(stream),
                                            C.byref(st)), st)

    def apply_compact(self, table: int, keys, source_values, row_offsets, source_rows, scales,
                      learning_rate: float, beta1_power: float, beta2_power: float,
                      optimizer_sequence: int = 0, stream=None):
        """CompactGradients (CSR) expanded on the device and applied with an external
        context (eps_b200_apply_compact); host numpy arrays."""
        keys = _host_u64(keys)
        sv = np.ascontiguousarray(source_values, dtype=np.float32)
        ro, sr = _host_u64(row_offsets), _host_u64(source_rows)
        sc = np.ascontiguousarray(scales, dtype=np.float32)
        dim = self.dimension(table)
        cg = CompactGradients(_ptr(keys), len(keys), dim, _ptr(sv), sv.size // dim, _ptr(ro),
                              _ptr(sr), _ptr(sc), len(sr))
        ctx = UpdateContext(table, learning_rate, beta1_power, beta2_power, optimizer_sequence)
        st = Status()
        _check(self.lib.eps_b200_apply_compact(self._h, C.byref(ctx), C.byref(cg),
                                               _stream_ptr(stream), C.byref(st)), st)

    # ---- synchronous multi-worker round (SynchronousGradientCollector)
    def sync_reduce(self, table: int, workers, reduction: int = REDUCE_SAMPLE_MEAN, stream=None):
        """Reduces one round of worker gradients for `table` on the device
        (eps_b200_sync_reduce).  workers: [(keys, values, sample_count)] with
        device tensors (keys int64 sorted unique, values float32 [rows, dim]).
        Returns (keys, values) device tensors of the ascending key union."""
        import torch
        arr = (WorkerGradients * len(workers))()
        total = 0
        for i, (k, v, c) in enumerate(workers):
            arr[i] = WorkerGradients(_ptr(k) if len(k) else None, _ptr(v) if len(k) else None,
                                     int(k.shape[0]), int(c))
            total += int(k.shape[0])
        dim = self.dimension(table)
        dev = f"cuda:{self.device}"
        keys = torch.empty(max(1, total), dtype=torch.int64, device=dev)
        values = torch.empty((max(1, total), dim), dtype=torch.float32, device=dev)
        rows = C.c_uint64(0)
        st = Status()
        _check(self.lib.eps_b200_sync_reduce(self._h, table, arr, len(workers), reduction,
                                             _ptr(keys), _ptr(values), max(1, total),
                                             C.byref(rows), _stream_ptr(stream), C.byref(st)), st)
        return keys[:rows.value], values[:rows.value]

    def apply_reduced(self, table: int, keys, values, feature: int = 0, stream=None):
        """Applies reduced row gradients as the reference's synchronous applier does
        (src/transport/brpc_synchronous_server.cpp:62-78): one sequence feature of
        the keys, looked up and pushed (one LazyAdam step of the table)."""
        import torch
        n = int(keys.shape[0])
        offs = torch.tensor([0, n], dtype=torch.int64, device=keys.device)
        f = FeatureInput(table, feature, SEQUENCE, keys, offs)
        out = torch.empty((n, self.dimension(table)), dtype=torch.float32, device=keys.device)
        ticket, _ = self.lookup([f], outputs=[out], stream=stream)
        self.push(ticket, [values], features=[feature], wait=True, stream=stream)

    def stats(self) -> dict:
        s = Stats()
        st = Status()
        _check(self.lib.eps_b200_stats(self._h, C.byref(s), C.byref(st)), st)
        return {n: getattr(s, n) for n, _ in Stats._fields_}


def _stream_ptr(stream):
    if stream is None:
        return None
    if hasattr(stream, "cuda_stream"):
        return stream.cuda_stream
    return int(stream)


def snapshot_inspect(path: str):
    """Reads a snapshot file on the host (no GPU): (info dict, [table dicts])."""
    lib = load_library()
    info = SnapshotInfo()
    tabs = (SnapshotTable * 1024)()
    st = Status()
    _check(lib.eps_b200_snapshot_inspect(str(path).encode(), C.byref(info), tabs, 1024,
                                         C.byref(st)), st)
    meta = {"format": info.format, "run": info.run.decode(), "shard": info.shard,
            "shard_count": info.shard_count, "partition_epoch": info.partition_epoch,
            "checksum": info.checksum}
    out = []
    for i in range(info.tables):
        t = tabs[i]
        d = t.definition
        out.append({"id": d.id, "dimension": d.dimension, "learning_rate": d.learning_rate,
                    "has_weight_bounds": d.has_weight_bounds, "initialization_min": d.initialization_min,
                    "initialization_seed": d.initialization_seed,
                    "optimizer_sequence": t.optimizer_sequence, "beta1_power": t.beta1_power,
                    "beta2_power": t.beta2_power, "rows": t.rows})
    return meta, out


def snapshot_rows(path: str, table_index: int, rows: int, dim: int):
    """One table's rows of a snapshot file: (keys, row_updates, w, m, v)."""
    lib = load_library()
    keys = np.zeros(max(1, rows), np.uint64)
    upd = np.zeros(max(1, rows), np.uint64)
    state = np.zeros((max(1, rows), 3, dim), np.float32)
    st = Status()
    _check(lib.eps_b200_snapshot_rows(str(path).encode(), table_index, keys.ctypes.data,
                                      upd.ctypes.data, state.ctypes.data, max(1, rows),
                                      C.byref(st)), st)
    return keys[:rows], upd[:rows], state[:rows, 0], state[:rows, 1], state[:rows, 2]
