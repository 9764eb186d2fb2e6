"""ctypes bindings for the two CPU checkers (test infrastructure only).

* ``Oracle``    -- this repository's C restatement (oracle/eps_oracle.c).
* ``Reference`` -- the unmodified reference CPU parameter server compiled from its
  own sources (oracle/_ref/libeps_ref.so, built by oracle/Makefile), driven
  through ``DistributedClient`` over n in-process ``CpuParameterService`` shards.

Both work on plain numpy arrays.  Neither is part of the product path.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass, field

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_SO = os.path.join(ROOT, "oracle", "_build", "libeps_oracle.so")
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libeps_ref.so")
# the same harness with the reference's CUDA cache backend linked in (make ref-cuda)
REF_CUDA_SO = os.path.join(ROOT, "oracle", "_ref", "libeps_ref_cuda.so")

SUM, MEAN, SEQUENCE = 0, 1, 2

u64p = C.POINTER(C.c_uint64)
f32p = C.POINTER(C.c_float)


def _u64(a):
    return np.ascontiguousarray(a, dtype=np.uint64)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a, t):
    return a.ctypes.data_as(t)


@dataclass
class TableDef:
    """Mirrors TableDefinition + OptimizerConfig (include/eps/types.hpp:76-97)."""
    id: int = 1
    dimension: int = 2
    learning_rate: float = 0.1
    beta1: float = 0.9
    beta2: float = 0.999
    epsilon: float = 1e-8
    initial_beta1_power: float = 0.9
    initial_beta2_power: float = 0.999
    bounds: tuple | None = None
    init_min: float = 0.25
    init_max: float = 0.25
    init_seed: int = 42
    rows: int = 16


@dataclass
class Feature:
    """Mirrors FeatureInput (include/eps/types.hpp:99-107); lengths = offset diffs."""
    table: int
    feature: int
    pooling: int
    keys: np.ndarray
    offsets: np.ndarray
    extra: dict = field(default_factory=dict)

    def __post_init__(self):
        self.keys = _u64(self.keys)
        self.offsets = _u64(self.offsets)

    @property
    def output_rows(self):
        return len(self.keys) if self.pooling == SEQUENCE else len(self.offsets) - 1


# --------------------------------------------------------------------------- oracle
class _EoTable(C.Structure):
    _fields_ = [("id", C.c_uint32), ("dimension", C.c_uint32),
                ("learning_rate", C.c_float), ("beta1", C.c_float), ("beta2", C.c_float),
                ("epsilon", C.c_float), ("beta1_power", C.c_float), ("beta2_power", C.c_float),
                ("optimizer_sequence", C.c_uint64), ("has_bounds", C.c_int32),
                ("bound_min", C.c_float), ("bound_max", C.c_float),
                ("init_min", C.c_float), ("init_max", C.c_float), ("init_seed", C.c_uint64),
                ("rows", C.c_uint64), ("state", f32p), ("updates", u64p)]


class _EoFeature(C.Structure):
    _fields_ = [("table", C.c_uint32), ("feature", C.c_uint32), ("pooling", C.c_uint32),
                ("keys", u64p), ("key_count", C.c_uint64),
                ("offsets", u64p), ("offset_count", C.c_uint64)]


def _load(path):
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is missing: run `make -C oracle oracle ref`")
    return C.CDLL(path)


class Oracle:
    """Dense-table CPU restatement: every table keeps [w|m|v] rows and counters."""

    def __init__(self, tables: list[TableDef]):
        self.lib = _load(ORACLE_SO)
        self.lib.eo_mix.restype = C.c_uint64
        self.lib.eo_mix.argtypes = [C.c_uint64]
        self.lib.eo_initial_weight.restype = C.c_float
        self._defs = {t.id: t for t in tables}
        self._arr = (_EoTable * len(tables))()
        self._state = {}
        for i, t in enumerate(tables):
            st = np.zeros((t.rows, 3, t.dimension), dtype=np.float32)
            upd = np.zeros(t.rows, dtype=np.uint64)
            e = self._arr[i]
            e.id, e.dimension = t.id, t.dimension
            e.learning_rate, e.beta1, e.beta2, e.epsilon = (t.learning_rate, t.beta1,
                                                            t.beta2, t.epsilon)
            e.beta1_power, e.beta2_power = t.initial_beta1_power, t.initial_beta2_power
            e.optimizer_sequence = 0
            e.has_bounds = 1 if t.bounds else 0
            e.bound_min, e.bound_max = (t.bounds if t.bounds else (0.0, 0.0))
            e.init_min, e.init_max, e.init_seed = t.init_min, t.init_max, t.init_seed
            e.rows = t.rows
            e.state = _ptr(st, f32p)
            e.updates = _ptr(upd, u64p)
            self._state[t.id] = (st, upd)
            # initialise the rows with the reference initializer (in C)
            self._init_rows(i, st)

    def _init_rows(self, i, st):
        t = self._arr[i]
        lib = self.lib
        lib.eo_initial_weight.argtypes = [C.POINTER(_EoTable), C.c_uint64, C.c_uint32]
        # vectorised through a C loop: eo_table_init allocates its own memory, so
        # reproduce its loop here through eo_initial_weight for small tables and
        # use the whole-table C routine for large ones.
        if t.rows * t.dimension <= 1 << 16:
            for key in range(t.rows):
                for d in range(t.dimension):
                    st[key, 0, d] = lib.eo_initial_weight(C.byref(t), key, d)
        else:
            tmp = _EoTable.from_buffer_copy(t)
            assert lib.eo_table_init(C.byref(tmp)) == 0
            n = t.rows * 3 * t.dimension
            src = np.ctypeslib.as_array(tmp.state, shape=(n,))
            st.reshape(-1)[:] = src
            lib.eo_table_free(C.byref(tmp))

    def table(self, tid):
        for e in self._arr:
            if e.id == tid:
                return e
        raise KeyError(tid)

    def state(self, tid):
        return self._state[tid]

    def _features(self, feats):
        arr = (_EoFeature * len(feats))()
        for i, f in enumerate(feats):
            a = arr[i]
            a.table, a.feature, a.pooling = f.table, f.feature, f.pooling
            a.keys, a.key_count = _ptr(f.keys, u64p), len(f.keys)
            a.offsets, a.offset_count = _ptr(f.offsets, u64p), len(f.offsets)
        return arr

    def lookup(self, feats, shards=1):
        outs = [np.zeros((f.output_rows, self._defs[f.table].dimension), np.float32)
                for f in feats]
        ptrs = (f32p * len(feats))(*[_ptr(o, f32p) for o in outs])
        rc = self.lib.eo_lookup(self._arr, len(self._arr), self._features(feats),
                                len(feats), shards, ptrs)
        if rc:
            raise ValueError(f"oracle lookup rejected ({rc})")
        return outs

    def push(self, feats, grads):
        grads = [_f32(g) for g in grads]
        ptrs = (f32p * len(feats))(*[_ptr(g, f32p) for g in grads])
        return self.lib.eo_push(self._arr, len(self._arr), self._features(feats),
                                len(feats), ptrs)

    def reduce(self, tid, feats, grads):
        t = self.table(tid)
        total = sum(len(f.keys) for f in feats if f.table == tid)
        rows = np.zeros(max(total, 1), np.uint64)
        vals = np.zeros((max(total, 1), t.dimension), np.float32)
        u = C.c_uint64(0)
        grads = [_f32(g) for g in grads]
        ptrs = (f32p * len(feats))(*[_ptr(g, f32p) for g in grads])
        rc = self.lib.eo_reduce_gradients(C.byref(t), self._features(feats), len(feats),
                                          ptrs, _ptr(rows, u64p), _ptr(vals, f32p),
                                          C.byref(u))
        return rc, rows[:u.value], vals[:u.value]

    def apply_host(self, tid, lr, b1p, b2p, keys, values):
        """eo_apply_host: LazyAdam with an external context; returns 0 or 1 (rejected)."""
        t = self.table(tid)
        keys = _u64(keys)
        values = _f32(values).reshape(-1)
        self.lib.eo_apply_host.argtypes = [C.POINTER(_EoTable), C.c_float, C.c_float, C.c_float,
                                           u64p, f32p, C.c_uint64]
        return self.lib.eo_apply_host(C.byref(t), lr, b1p, b2p, _ptr(keys, u64p), _ptr(values, f32p),
                                      len(keys))

    def expand_compact(self, dim, rows, source_values, row_offsets, source_rows, scales):
        sv = _f32(source_values).reshape(-1)
        ro, sr, sc = _u64(row_offsets), _u64(source_rows), _f32(scales)
        out = np.zeros((rows, dim), np.float32)
        rc = self.lib.eo_expand_compact(C.c_uint32(dim), C.c_uint64(rows), _ptr(sv, f32p),
                                        C.c_uint64(len(sv) // max(1, dim)), _ptr(ro, u64p),
                                        _ptr(sr, u64p), _ptr(sc, f32p), _ptr(out, f32p))
        return rc, out

    def sync_reduce(self, dim, workers, reduction):
        """eo_sync_reduce: workers = [(keys u64[k], values f32[k, dim], sample_count)]."""
        W = len(workers)
        keys = [_u64(k) for k, _, _ in workers]
        vals = [_f32(v).reshape(-1) for _, v, _ in workers]
        kp = (u64p * W)(*[_ptr(k, u64p) for k in keys])
        vp = (f32p * W)(*[_ptr(v, f32p) for v in vals])
        rows = _u64([len(k) for k in keys])
        samples = _u64([c for _, _, c in workers])
        total = max(1, int(rows.sum()))
        ko = np.zeros(total, np.uint64)
        vo = np.zeros((total, dim), np.float32)
        self.lib.eo_sync_reduce.restype = C.c_uint64
        u = self.lib.eo_sync_reduce(C.c_uint32(dim), C.c_uint32(W), kp, vp, _ptr(rows, u64p),
                                    _ptr(samples, u64p), C.c_int(reduction), _ptr(ko, u64p),
                                    _ptr(vo, f32p))
        if u == (1 << 64) - 1:
            raise ValueError("gradient reduction overflow")
        return ko[:u], vo[:u]

    def powers(self, tid):
        t = self.table(tid)
        return t.beta1_power, t.beta2_power, t.optimizer_sequence


# ----------------------------------------------------------------------- reference
class _RhTable(C.Structure):
    _fields_ = [("id", C.c_uint32), ("dimension", C.c_uint32),
                ("learning_rate", C.c_float), ("beta1", C.c_float), ("beta2", C.c_float),
                ("epsilon", C.c_float), ("initial_beta1_power", C.c_float),
                ("initial_beta2_power", C.c_float), ("has_bounds", C.c_int32),
                ("bound_min", C.c_float), ("bound_max", C.c_float),
                ("init_min", C.c_float), ("init_max", C.c_float), ("init_seed", C.c_uint64)]


class _RhFeature(C.Structure):
    _fields_ = [("table", C.c_uint32), ("feature", C.c_uint32), ("pooling", C.c_uint32),
                ("keys", u64p), ("key_count", C.c_uint64),
                ("offsets", u64p), ("offset_count", C.c_uint64)]


def reference_available():
    return os.path.exists(REF_SO)


class Reference:
    """The reference's own CPU path (CpuParameterService x n + DistributedClient)."""

    def __init__(self, tables: list[TableDef], shards: int = 1, state_bytes: int = 8 << 30,
                 run: str | None = None, snapshot_dir: str | None = None, define: bool = True,
                 library: str = REF_SO):
        self.lib = _load(library)
        self.lib.rh_create_run.restype = C.c_void_p
        self.lib.rh_create_run.argtypes = [C.c_uint32, C.c_uint64, C.c_char_p, C.c_char_p,
                                           C.c_char_p]
        for name in ("rh_create_table", "rh_lookup", "rh_push", "rh_release", "rh_read",
                     "rh_stats", "rh_snapshot", "rh_restore"):
            getattr(self.lib, name).restype = C.c_int
        self.lib.rh_destroy.argtypes = [C.c_void_p]
        self.err = C.create_string_buffer(1024)
        self.h = self.lib.rh_create_run(shards, state_bytes,
                                        run.encode() if run else None,
                                        snapshot_dir.encode() if snapshot_dir else None, self.err)
        if not self.h:
            raise RuntimeError(self.err.value.decode())
        self._defs = {t.id: t for t in tables}
        if define:                             # a service to Restore into stays empty
            self.define()

    def define(self):
        """CreateTable through the client (idempotent on shards that already
        hold the table, e.g. after Restore)."""
        for t in self._defs.values():
            rt = _RhTable(t.id, t.dimension, t.learning_rate, t.beta1, t.beta2, t.epsilon,
                          t.initial_beta1_power, t.initial_beta2_power,
                          1 if t.bounds else 0, *(t.bounds if t.bounds else (0.0, 0.0)),
                          t.init_min, t.init_max, t.init_seed)
            self._check(self.lib.rh_create_table(C.c_void_p(self.h), C.byref(rt), self.err))

    def attach_cuda(self, tid, keys, device=0, rows_per_table=1 << 24, state_bytes=64 << 30):
        """The reference's GPU path (library=REF_CUDA_SO, one shard): its
        CudaCacheBackend attached as agent 0 and the rows `keys` of table `tid`
        moved to it; the rows must exist (a lookup has touched them)."""
        fn = self.lib.rh_attach_cuda
        fn.restype = C.c_int
        fn.argtypes = [C.c_void_p, C.c_int32, C.c_uint64, C.c_uint64, C.c_uint32, C.c_uint32,
                       C.c_void_p, C.c_uint64, C.c_char_p]
        k = _u64(keys)
        self._check(fn(C.c_void_p(self.h), device, rows_per_table, state_bytes, tid,
                       self._defs[tid].dimension, k.ctypes.data, len(k), self.err))

    def close(self):
        if self.h:
            self.lib.rh_destroy(C.c_void_p(self.h))
            self.h = None

    __del__ = close

    def _check(self, rc):
        if rc:
            raise ValueError(f"reference rejected ({rc}): {self.err.value.decode()}")

    def lookup(self, feats, read_only=False):
        arr = (_RhFeature * len(feats))()
        for i, f in enumerate(feats):
            arr[i] = _RhFeature(f.table, f.feature, f.pooling, _ptr(f.keys, u64p), len(f.keys),
                                _ptr(f.offsets, u64p), len(f.offsets))
        outs = [np.zeros((f.output_rows, self._defs[f.table].dimension), np.float32)
                for f in feats]
        ptrs = (f32p * len(feats))(*[_ptr(o, f32p) for o in outs])
        batch = C.c_uint64(0)
        self._check(self.lib.rh_lookup(C.c_void_p(self.h), len(feats), arr, int(read_only),
                                       ptrs, C.byref(batch), self.err))
        return batch.value, outs

    def push(self, batch, feats, grads, check=True):
        grads = [_f32(g) for g in grads]
        ids = (C.c_uint32 * len(feats))(*[f.feature for f in feats])
        ptrs = (f32p * len(feats))(*[_ptr(g, f32p) for g in grads])
        rows = (C.c_uint64 * len(feats))(*[g.shape[0] for g in grads])
        dims = (C.c_uint32 * len(feats))(*[self._defs[f.table].dimension for f in feats])
        rc = self.lib.rh_push(C.c_void_p(self.h), batch, len(feats), ids, ptrs, rows, dims,
                              self.err)
        if check:
            self._check(rc)
        return rc

    def release(self, batch):
        self._check(self.lib.rh_release(C.c_void_p(self.h), batch, self.err))

    def read(self, tid, key):
        d = self._defs[tid].dimension
        w, m, v = (np.zeros(d, np.float32) for _ in range(3))
        upd = C.c_uint64(0)
        self._check(self.lib.rh_read(C.c_void_p(self.h), tid, key, _ptr(w, f32p),
                                     _ptr(m, f32p), _ptr(v, f32p), C.byref(upd), self.err))
        return w, m, v, upd.value

    def read_many(self, tid, keys):
        """ReadState of many rows of table `tid` (rh_read_many): (w, m, v, updates)."""
        keys = _u64(keys)
        d = self._defs[tid].dimension
        n = len(keys)
        w, m, v = (np.zeros((n, d), np.float32) for _ in range(3))
        upd = np.zeros(n, np.uint64)
        fn = self.lib.rh_read_many
        fn.restype = C.c_int
        fn.argtypes = [C.c_void_p, C.c_uint32, u64p, C.c_uint64, C.c_uint32, f32p, f32p, f32p,
                       u64p, C.c_char_p]
        self._check(fn(C.c_void_p(self.h), tid, _ptr(keys, u64p), n, d, _ptr(w, f32p),
                       _ptr(m, f32p), _ptr(v, f32p), _ptr(upd, u64p), self.err))
        return w, m, v, upd

    def snapshot(self, snapshot_id: str, shard: int = 0) -> str:
        """DrainAndFlush of one shard; returns the state file path."""
        out = C.create_string_buffer(1024)
        self._check(self.lib.rh_snapshot(C.c_void_p(self.h), shard, snapshot_id.encode(), out,
                                         self.err))
        return out.value.decode()

    def restore(self, path: str, shard: int = 0):
        self._check(self.lib.rh_restore(C.c_void_p(self.h), shard, path.encode(), self.err))

    def stats(self):
        out = (C.c_uint64 * 4)()
        self._check(self.lib.rh_stats(C.c_void_p(self.h), out, self.err))
        return list(out)
