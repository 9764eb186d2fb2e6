"""Consumer-side binding of the framework runtime ABI, eps_runtime_api_v1.

libeps_b200.so exports the reference's runtime function table
(include/eps/runtime_c.h: EpsRuntimeApi with create / destroy / pull / prepare /
pull_prepared / push / command).  A framework op loads it the way the
reference's TensorFlow ops do (adapters/entropy/tensorflow_ops.cc:38-52):
dlopen the library, call ``eps_runtime_api_v1()``, check ``abi_version`` and
``struct_bytes``, then drive the function pointers.  This module is that
consumer in ctypes, so Python callers and the tests use the table exactly as a
framework would; it adds nothing to the runtime's behaviour.

Configuration keys of the B200 runtime (JSON passed to ``create``):
``run``, ``epoch``, ``device``, ``state_bytes``, ``max_live``,
``release_read_only``, ``snapshot_directory``, ``restore`` (a snapshot file
loaded after the tables are created) and ``tables`` -- each table as the
reference's runtime reads it (``id``, ``dimension``, ``dtype``, ``optimizer``,
``initialization``) plus, optionally, ``key_space`` (a dense table of keys
[0, key_space); without it a hashed table of any 64-bit keys, ``capacity`` rows,
default 2^20, created on first touch).
"""
from __future__ import annotations

import ctypes as C
import json
from dataclasses import dataclass
from typing import Any, Sequence

import numpy as np

from . import EpsError, load_library

u64p = C.POINTER(C.c_uint64)

ABI = 1


class EpsStatus(C.Structure):
    _fields_ = [("code", C.c_int32), ("message", C.c_char * 1024)]


class EpsFeature(C.Structure):
    _fields_ = [("table", C.c_uint32), ("feature", C.c_uint32), ("pooling", C.c_uint32),
                ("keys", u64p), ("key_count", C.c_uint64),
                ("offsets", u64p), ("offset_count", C.c_uint64),
                ("has_padding", C.c_int32), ("padding_key", C.c_uint64)]


_Release = C.CFUNCTYPE(None, C.c_void_p)
_Wait = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_void_p, C.POINTER(EpsStatus))


class EpsBuffer(C.Structure):
    _fields_ = [("feature", C.c_uint32), ("rows", C.c_uint64), ("columns", C.c_uint64),
                ("data", C.c_void_p), ("device", C.c_int32), ("owner", C.c_void_p),
                ("release", _Release), ("wait", _Wait)]


class EpsBatch(C.Structure):
    _fields_ = [("handle", C.c_uint64), ("count", C.c_uint64),
                ("buffers", C.POINTER(EpsBuffer)), ("owner", C.c_void_p), ("release", _Release)]


class EpsText(C.Structure):
    _fields_ = [("data", C.c_void_p), ("size", C.c_uint64), ("owner", C.c_void_p),
                ("release", _Release)]


class EpsRuntimeApi(C.Structure):
    _fields_ = [
        ("abi_version", C.c_uint32), ("struct_bytes", C.c_uint32),
        ("create", C.CFUNCTYPE(C.c_int, C.c_char_p, C.POINTER(C.c_void_p), C.POINTER(EpsStatus))),
        ("destroy", C.CFUNCTYPE(None, C.c_void_p)),
        ("pull", C.CFUNCTYPE(C.c_int, C.c_void_p, C.POINTER(EpsFeature), C.c_uint64, C.c_int32,
                             C.c_int32, C.POINTER(EpsBatch), C.POINTER(EpsStatus))),
        ("prepare", C.CFUNCTYPE(C.c_int, C.c_void_p, C.POINTER(EpsFeature), C.c_uint64,
                                u64p, C.POINTER(EpsStatus))),
        ("pull_prepared", C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_uint64, C.c_int32, C.c_int32,
                                      C.POINTER(EpsBatch), C.POINTER(EpsStatus))),
        ("push", C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_uint64, C.POINTER(EpsBuffer), C.c_uint64,
                             C.c_void_p, C.POINTER(EpsStatus))),
        ("command", C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_char_p, C.c_char_p, C.POINTER(EpsText),
                                C.POINTER(EpsStatus))),
    ]


def api() -> EpsRuntimeApi:
    """The function table, checked as a consumer checks it (tensorflow_ops.cc:44-50)."""
    lib = load_library()
    fn = lib.eps_runtime_api_v1
    fn.restype = C.POINTER(EpsRuntimeApi)
    fn.argtypes = []
    table = fn()
    if not table:
        raise EpsError(6, "eps_runtime_api_v1 returned null")
    t = table.contents
    if t.abi_version != ABI or t.struct_bytes < C.sizeof(EpsRuntimeApi):
        raise EpsError(1, f"runtime ABI mismatch ({t.abi_version}, {t.struct_bytes})")
    return t


def _check(rc: int, st: EpsStatus):
    if rc:
        raise EpsError(rc, st.message.decode(errors="replace"))


@dataclass
class DeviceOutput:
    """A pulled feature tensor in GPU memory; exposes __cuda_array_interface__
    (torch.as_tensor(x, device="cuda") views it without a copy while the batch
    is alive)."""
    feature: int
    rows: int
    columns: int
    data: int
    device: int

    @property
    def __cuda_array_interface__(self):
        return {"shape": (self.rows, self.columns), "typestr": "<f4",
                "data": (self.data or 0, False), "version": 3, "strides": None}


class PulledBatch:
    """EpsBatch: ``handle`` (UINT64_MAX for an auto-released read-only pull) and
    one output per feature -- numpy arrays (host pulls, copied out) or
    DeviceOutput views (device pulls, valid until ``release()``)."""

    def __init__(self, batch: EpsBatch, device: bool):
        self._batch = batch
        self.handle = int(batch.handle)
        self.outputs: list[Any] = []
        for i in range(batch.count):
            b = batch.buffers[i]
            if device:
                self.outputs.append(DeviceOutput(b.feature, b.rows, b.columns, b.data or 0, b.device))
            else:
                n = b.rows * b.columns
                arr = np.empty((b.rows, b.columns), np.float32)
                if n:
                    C.memmove(arr.ctypes.data, b.data, n * 4)
                self.outputs.append(arr)
        if not device:
            self.release()

    def wait(self, stream: int = 0):
        """EpsBuffer::wait: makes `stream` wait for the outputs."""
        if not self._batch:
            return
        st = EpsStatus()
        for i in range(self._batch.count):
            b = self._batch.buffers[i]
            _check(b.wait(b.owner, C.c_void_p(stream), C.byref(st)), st)

    def release(self):
        if self._batch is not None and self._batch.owner:
            self._batch.release(self._batch.owner)
        self._batch = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


def _features(feats: Sequence[Any]):
    arr = (EpsFeature * len(feats))()
    keep = []
    for i, f in enumerate(feats):
        keys = np.ascontiguousarray(f.keys, np.uint64)
        offs = np.ascontiguousarray(f.offsets, np.uint64)
        keep += [keys, offs]
        a = arr[i]
        a.table, a.feature, a.pooling = int(f.table), int(f.feature), int(f.pooling)
        a.keys, a.key_count = keys.ctypes.data_as(u64p), len(keys)
        a.offsets, a.offset_count = offs.ctypes.data_as(u64p), len(offs)
        pad = getattr(f, "padding_key", None)
        a.has_padding, a.padding_key = (0, 0) if pad is None else (1, int(pad))
    return arr, keep


class NativeRuntime:
    """One runtime created through the function table (runtime_c.h's create)."""

    def __init__(self, config: dict | str):
        self.api = api()
        text = config if isinstance(config, str) else json.dumps(config)
        h, st = C.c_void_p(), EpsStatus()
        _check(self.api.create(text.encode(), C.byref(h), C.byref(st)), st)
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            self.api.destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def pull(self, feats: Sequence[Any], read_only: bool = False, device: bool = False) -> PulledBatch:
        arr, keep = _features(feats)
        b, st = EpsBatch(), EpsStatus()
        _check(self.api.pull(self._h, arr, len(feats), int(read_only), int(device), C.byref(b),
                             C.byref(st)), st)
        del keep
        return PulledBatch(b, device)

    def prepare(self, feats: Sequence[Any]) -> int:
        arr, keep = _features(feats)
        tok, st = C.c_uint64(), EpsStatus()
        _check(self.api.prepare(self._h, arr, len(feats), C.byref(tok), C.byref(st)), st)
        del keep
        return tok.value

    def pull_prepared(self, token: int, read_only: bool = False, device: bool = False) -> PulledBatch:
        b, st = EpsBatch(), EpsStatus()
        _check(self.api.pull_prepared(self._h, token, int(read_only), int(device), C.byref(b),
                                      C.byref(st)), st)
        return PulledBatch(b, device)

    def push(self, handle: int, grads: Sequence[tuple[int, Any]], stream: int = 0):
        """grads: (feature id, gradient) pairs; a gradient is a float32 numpy
        array [rows, columns] or a CUDA tensor (its device pointer is passed
        with device = its GPU, consumed on `stream`)."""
        bufs = (EpsBuffer * len(grads))()
        keep = []
        for i, (feature, g) in enumerate(grads):
            b = bufs[i]
            b.feature = int(feature)
            if hasattr(g, "is_cuda") and g.is_cuda:
                g = g.contiguous()
                keep.append(g)
                b.rows, b.columns = int(g.shape[0]), int(g.shape[1])
                b.data, b.device = g.data_ptr(), g.device.index or 0
            else:
                a = np.ascontiguousarray(g, np.float32)
                keep.append(a)
                b.rows, b.columns = a.shape
                b.data, b.device = a.ctypes.data, -1
        st = EpsStatus()
        _check(self.api.push(self._h, C.c_uint64(handle), bufs, len(grads), C.c_void_p(stream),
                             C.byref(st)), st)
        del keep

    def command(self, name: str, args: dict | None = None) -> Any:
        out, st = EpsText(), EpsStatus()
        _check(self.api.command(self._h, name.encode(), json.dumps(args or {}).encode(),
                                C.byref(out), C.byref(st)), st)
        try:
            text = C.string_at(out.data, out.size).decode()
        finally:
            if out.owner:
                out.release(out.owner)
        return json.loads(text)
