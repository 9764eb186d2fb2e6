"""The framework runtime ABI (eps_runtime_api_v1, include/eps_b200_runtime_c.h)
as the reference's consumers bind it (include/eps/runtime_c.h,
adapters/entropy/tensorflow_ops.cc:38-52).

CPU: the function table is exported, versioned and layout-identical to the
reference's header (a C consumer compiled against either header reads the same
offsets); configuration errors are reported with the reference's codes before
any GPU work; without a GPU, create fails loudly.
GPU: pull / push through the table bit-exact against the oracle (padding, all
poolings, weight bounds, host and device buffers), a table given as the
reference writes it (no key_space: any 64-bit key, rows created on first touch)
bit-exact against the reference CPU parameter server, the adapter's batch
lifecycle (handles, read-only batches, prepared inputs, live-batch limit,
retired handles), frozen save -> checkpoint export -> resume, restore of the
saved file into a fresh runtime, table modes and control commands.
"""
from __future__ import annotations

import ctypes as C
import json
import os
import re
import subprocess
import tempfile
import types

import numpy as np
import pytest

from conftest import ROOT, gpu_available
from oracle_lib import (MEAN, SEQUENCE, SUM, Feature, Oracle, Reference, TableDef,
                        reference_available)

HEADER = os.path.join(ROOT, "include", "eps_b200_runtime_c.h")
REFERENCE_HEADER_DIR = os.path.join(os.environ.get("EPS_REFERENCE", os.path.join(
    os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))), "reference")),
    "include")
U64_MAX = (1 << 64) - 1

F32 = np.float32


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.fixture(scope="module")
def rt(eps):
    import importlib
    return importlib.import_module("eps_b200.runtime_api")


def table_json(t: TableDef) -> dict:
    o = {"kind": "sparse_lazy_adam", "learning_rate": t.learning_rate, "beta1": t.beta1,
         "beta2": t.beta2, "epsilon": t.epsilon, "initial_beta1_power": t.initial_beta1_power,
         "initial_beta2_power": t.initial_beta2_power}
    if t.bounds:
        o["weight_bounds"] = list(t.bounds)
    return {"id": t.id, "dimension": t.dimension, "dtype": "float32", "key_space": t.rows,
            "optimizer": o, "initialization": {"min": t.init_min, "max": t.init_max,
                                               "seed": t.init_seed}}


def config(tables, **kw) -> dict:
    c = {"run": "runtime-test", "device": 0, "state_bytes": 1 << 30,
         "tables": [table_json(t) for t in tables]}
    c.update(kw)
    return c


# ------------------------------------------------------------------- CPU
LAYOUT_PROGRAM = r'''
#include <stdio.h>
#include <stddef.h>
#include RUNTIME_HEADER
#define F(T, m) printf(#T "." #m " %zu\n", offsetof(T, m))
#define S(T) printf(#T " %zu\n", sizeof(T))
int main(void) {
  S(EpsStatus); F(EpsStatus, code); F(EpsStatus, message);
  S(EpsFeature); F(EpsFeature, table); F(EpsFeature, feature); F(EpsFeature, pooling);
  F(EpsFeature, keys); F(EpsFeature, key_count); F(EpsFeature, offsets);
  F(EpsFeature, offset_count); F(EpsFeature, has_padding); F(EpsFeature, padding_key);
  S(EpsBuffer); F(EpsBuffer, feature); F(EpsBuffer, rows); F(EpsBuffer, columns);
  F(EpsBuffer, data); F(EpsBuffer, device); F(EpsBuffer, owner); F(EpsBuffer, release);
  F(EpsBuffer, wait);
  S(EpsBatch); F(EpsBatch, handle); F(EpsBatch, count); F(EpsBatch, buffers);
  F(EpsBatch, owner); F(EpsBatch, release);
  S(EpsText); F(EpsText, data); F(EpsText, size); F(EpsText, owner); F(EpsText, release);
  S(EpsRuntimeApi); F(EpsRuntimeApi, abi_version); F(EpsRuntimeApi, struct_bytes);
  F(EpsRuntimeApi, create); F(EpsRuntimeApi, destroy); F(EpsRuntimeApi, pull);
  F(EpsRuntimeApi, prepare); F(EpsRuntimeApi, pull_prepared); F(EpsRuntimeApi, push);
  F(EpsRuntimeApi, command);
  printf("ABI %d\n", EPS_RUNTIME_ABI);
  return 0;
}
'''

# A consumer written the way tensorflow_ops.cc loads a runtime: dlopen, dlsym,
# version check, create with a given configuration, report the status.
CONSUMER_PROGRAM = r'''
#include <dlfcn.h>
#include <stdio.h>
#include RUNTIME_HEADER
int main(int argc, char** argv) {
  void* lib = dlopen(argv[1], RTLD_NOW | RTLD_LOCAL);
  if (!lib) { printf("dlopen %s\n", dlerror()); return 2; }
  EpsRuntimeEntry entry = (EpsRuntimeEntry)dlsym(lib, "eps_runtime_api_v1");
  if (!entry) { printf("no entry\n"); return 3; }
  const EpsRuntimeApi* api = entry();
  if (!api || api->abi_version != EPS_RUNTIME_ABI || api->struct_bytes < sizeof(EpsRuntimeApi)) {
    printf("abi mismatch\n"); return 4;
  }
  for (int i = 2; i < argc; ++i) {
    EpsStatus st; void* rt = 0;
    int rc = api->create(argv[i], &rt, &st);
    printf("%d %d %s\n", rc, st.code, st.message);
    if (!rc) api->destroy(rt);
  }
  return 0;
}
'''


def _compile_run(src: str, header: str, incdir: str, args=(), libs=()):
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "p.c")
        open(c, "w").write(src)
        exe = os.path.join(d, "p")
        subprocess.check_call(["gcc", f'-DRUNTIME_HEADER="{header}"', "-I", incdir, c, "-o", exe,
                               *libs])
        return subprocess.run([exe, *args], capture_output=True, text=True, check=True).stdout


def test_header_declares_and_library_exports_the_table(eps):
    text = open(HEADER).read()
    assert re.search(r"EPS_RUNTIME_EXPORT\s+const\s+EpsRuntimeApi\s*\*\s*eps_runtime_api_v1\s*\(", text)
    out = subprocess.run(["nm", "-D", "--defined-only", eps.library_path()], capture_output=True,
                         text=True, check=True).stdout
    assert re.search(r"\bT\s+eps_runtime_api_v1\b", out)


def test_function_table_version_and_size(rt):
    t = rt.api()
    assert t.abi_version == 1
    assert t.struct_bytes == C.sizeof(rt.EpsRuntimeApi)
    for name in ("create", "destroy", "pull", "prepare", "pull_prepared", "push", "command"):
        assert C.cast(getattr(t, name), C.c_void_p).value


def test_layout_matches_ctypes_and_reference_header(rt):
    mine = _compile_run(LAYOUT_PROGRAM, "eps_b200_runtime_c.h", os.path.join(ROOT, "include"))
    got = dict(line.rsplit(" ", 1) for line in mine.strip().splitlines())
    assert got["ABI"] == "1"
    for name, cls in (("EpsStatus", rt.EpsStatus), ("EpsFeature", rt.EpsFeature),
                      ("EpsBuffer", rt.EpsBuffer), ("EpsBatch", rt.EpsBatch),
                      ("EpsText", rt.EpsText), ("EpsRuntimeApi", rt.EpsRuntimeApi)):
        assert int(got[name]) == C.sizeof(cls), name
        for field, _ in cls._fields_:
            assert int(got[f"{name}.{field}"]) == getattr(cls, field).offset, (name, field)
    if not os.path.exists(os.path.join(REFERENCE_HEADER_DIR, "eps", "runtime_c.h")):
        pytest.skip("reference checkout absent: layout pinned against ctypes only")
    ref = _compile_run(LAYOUT_PROGRAM, "eps/runtime_c.h", REFERENCE_HEADER_DIR)
    assert ref == mine


@pytest.mark.parametrize("header,incdir", [("eps_b200_runtime_c.h", os.path.join(ROOT, "include")),
                                           ("eps/runtime_c.h", REFERENCE_HEADER_DIR)])
def test_consumer_compiled_against_either_header_loads_the_library(eps, header, incdir):
    if not os.path.exists(os.path.join(incdir, header)):
        pytest.skip("reference checkout absent")
    t = TableDef(id=1, dimension=4, rows=10)
    configs = ['{"run": ', json.dumps({"run": "x", "tables": [], "cuda": {}}),
               json.dumps({"tables": []}), "[1, 2]",
               json.dumps({"run": "x", "tables": [table_json(t)], "epoch": -1})]
    out = _compile_run(CONSUMER_PROGRAM, header, incdir, args=[eps.library_path(), *configs],
                       libs=["-ldl"]).strip().splitlines()
    codes = [tuple(line.split(" ", 2)) for line in out]
    assert [c[0] for c in codes] == ["1"] * 5, out           # invalid_argument + 1
    assert all(c[0] == c[1] for c in codes)
    assert "truncated JSON" in codes[0][2]
    assert "not supported" in codes[1][2]
    assert "'run'" in codes[2][2]
    assert "unsigned integer" in codes[4][2]


@pytest.mark.skipif(gpu_available(), reason="checks the no-GPU failure path")
def test_create_without_gpu_fails_loudly(rt, eps):
    with pytest.raises(eps.EpsError) as e:
        rt.NativeRuntime(config([TableDef(id=1, dimension=4, rows=10)]))
    assert e.value.code in (eps.UNAVAILABLE, eps.RUN_FAILED)


def test_json_configuration_errors(rt, eps):
    for bad, words in [('{"run": "a", "tables": [], }', "JSON"), ('{"run": "a\\q"}', "escape"),
                       ('{"run": 5, "tables": []}', "string"),
                       ('{"run": "a", "tables": []} x', "trailing"),
                       ('{"run": "a", "tables": [], "training": {}}', "not supported")]:
        with pytest.raises(eps.EpsError) as e:
            rt.NativeRuntime(bad)
        assert e.value.code == eps.INVALID_ARGUMENT and words in str(e.value), (bad, str(e.value))


# ------------------------------------------------------------------- GPU
def _tables():
    return [TableDef(id=1, dimension=32, learning_rate=0.01, init_min=-0.05, init_max=0.05,
                     rows=200, init_seed=7),
            TableDef(id=2, dimension=8, learning_rate=0.05, init_min=-0.1, init_max=0.1, rows=64,
                     bounds=(-0.06, 0.06), init_seed=9)]


def _batch(seed, pad=197):
    rng = np.random.default_rng(seed)
    feats = []
    for fi, (table, rows, pool) in enumerate([(1, 200, SUM), (1, 200, MEAN), (2, 64, SEQUENCE),
                                              (2, 64, MEAN)]):
        lens = rng.integers(0, 6, size=24)
        offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.uint64)
        keys = rng.integers(0, rows, size=int(offs[-1])).astype(np.uint64)
        f = Feature(table, 10 + fi, pool, keys, offs)
        if table == 1:
            keys[rng.random(len(keys)) < 0.25] = pad
            f.padding_key = pad
        feats.append(f)
    return feats


def _drop_padding(f):
    pad = getattr(f, "padding_key", None)
    if pad is None:
        return f, list(range(len(f.keys)))
    keys, offs, pos = [], [0], []
    for b in range(len(f.offsets) - 1):
        for i in range(int(f.offsets[b]), int(f.offsets[b + 1])):
            if int(f.keys[i]) != pad:
                keys.append(int(f.keys[i]))
                pos.append(i)
        offs.append(len(keys))
    return Feature(f.table, f.feature, f.pooling, np.array(keys, np.uint64), offs), pos


def _oracle_round(o, feats, grads):
    compact = [_drop_padding(f) for f in feats]
    ref = o.lookup([c for c, _ in compact])
    want = []
    for f, (c, pos), r in zip(feats, compact, ref):
        if f.pooling == SEQUENCE:
            w = np.zeros((len(f.keys), r.shape[1]), F32)
            w[pos] = r
            want.append(w)
        else:
            want.append(r)
    if grads is not None:
        cg = [g[pos] if f.pooling == SEQUENCE else g for f, (c, pos), g in zip(feats, compact, grads)]
        assert o.push([c for c, _ in compact], cg) == 0
    return want


def _all_rows(t):
    """A sequence feature over every key of table t: reads back the weights."""
    return types.SimpleNamespace(table=t.id, feature=99, pooling=SEQUENCE,
                                 keys=np.arange(t.rows, dtype=np.uint64),
                                 offsets=np.array([0, t.rows], np.uint64))


def _grads(outs, seed):
    rng = np.random.default_rng(seed)
    return [rng.normal(0, 0.02, size=np.asarray(a).shape).astype(F32) for a in outs]


@pytest.mark.gpu
def test_pull_push_bit_exact_vs_oracle(rt):
    ts = _tables()
    r, o = rt.NativeRuntime(config(ts)), Oracle(ts)
    for step in range(3):
        feats = _batch(step)
        b = r.pull(feats)
        assert b.handle == step
        grads = _grads(b.outputs, 100 + step)
        want = _oracle_round(o, feats, grads)
        for f, got, w in zip(feats, b.outputs, want):
            assert np.array_equal(bits(got), bits(w)), (step, f.feature)
        r.push(b.handle, [(f.feature, g) for f, g in zip(feats, grads)])
    for t in ts:
        got = r.pull([_all_rows(t)], read_only=True).outputs[0]
        st, _ = o.state(t.id)
        assert np.array_equal(bits(got), bits(st[:, 0])), t.id
    s = r.command("stats")
    assert s[0]["updates"] > 0 and s[0]["live_tickets"] == 0
    r.close()


@pytest.mark.gpu
def test_device_buffers_match_host_path(rt):
    import torch
    ts = _tables()
    host, dev = rt.NativeRuntime(config(ts)), rt.NativeRuntime(config(ts))
    stream = torch.cuda.current_stream().cuda_stream
    for step in range(3):
        feats = _batch(10 + step)
        hb = host.pull(feats)
        db = dev.pull(feats, device=True)
        assert db.handle == hb.handle
        db.wait(stream)
        outs = [torch.as_tensor(x, device="cuda") for x in db.outputs]
        for f, a, d in zip(feats, hb.outputs, outs):
            assert d.shape == a.shape and np.array_equal(bits(d.cpu().numpy()), bits(a)), f.feature
        grads = _grads(hb.outputs, 200 + step)
        host.push(hb.handle, [(f.feature, g) for f, g in zip(feats, grads)])
        dgrads = [torch.from_numpy(g).cuda() for g in grads]
        dev.push(db.handle, [(f.feature, g) for f, g in zip(feats, dgrads)], stream=stream)
        del outs
        db.release()
    for t in ts:
        a = host.pull([_all_rows(t)], read_only=True).outputs[0]
        b = dev.pull([_all_rows(t)], read_only=True).outputs[0]
        assert np.array_equal(bits(a), bits(b))


@pytest.mark.gpu
def test_batch_lifecycle(rt, eps):
    ts = _tables()
    r = rt.NativeRuntime(config(ts, max_live=3))
    feats = _batch(1)
    ro = r.pull(feats, read_only=True)            # read-only batches stay live until released
    assert ro.handle == 0
    with pytest.raises(eps.EpsError) as e:
        r.push(0, [(f.feature, np.zeros_like(a)) for f, a in zip(feats, ro.outputs)])
    assert e.value.code == eps.INVALID_ARGUMENT and "invalid adapter Push" in str(e.value)
    with pytest.raises(eps.EpsError) as e:
        r.command("join")
    assert e.value.code == eps.UNAVAILABLE
    r.command("release", {"handle": 0})
    r.command("release", {"handle": 0})           # completed: acknowledged again
    with pytest.raises(eps.EpsError) as e:
        r.command("release", {"handle": 77})
    assert e.value.code == eps.RETIRED_REQUEST
    b1, b2 = r.pull(feats), r.pull(feats)
    assert (b1.handle, b2.handle) == (1, 2)
    grads = _grads(b1.outputs, 5)
    bad = [(f.feature, g) for f, g in zip(feats, grads)]
    with pytest.raises(eps.EpsError) as e:        # a feature missing
        r.push(1, bad[:-1])
    assert "invalid adapter Push" in str(e.value)
    with pytest.raises(eps.EpsError) as e:        # shape mismatch
        r.push(1, bad[:-1] + [(bad[-1][0], bad[-1][1][:-1] if len(bad[-1][1]) > 1 else
                                np.zeros((5, 8), F32))])
    assert "shape mismatch" in str(e.value)
    with pytest.raises(eps.EpsError) as e:        # duplicate feature
        r.push(1, bad[:-1] + [bad[0]])
    assert "duplicate gradient feature" in str(e.value)
    r.push(1, list(reversed(bad)))                # matched by feature id, any order
    r.push(1, bad)                                # pushed: acknowledged without effect
    r.command("release", {"handle": 2})
    with pytest.raises(eps.EpsError) as e:
        r.push(2, bad)
    assert e.value.code == eps.RETIRED_REQUEST
    live = [r.pull(feats) for _ in range(3)]      # the live-batch limit
    with pytest.raises(eps.EpsError) as e:
        r.pull(feats)
    assert e.value.code == eps.CAPACITY_EXCEEDED
    for b in live:
        r.command("release", {"handle": b.handle})
    # prepared inputs
    tok0, tok1 = r.prepare(feats), r.prepare(_batch(2))
    assert (tok0, tok1) == (0, 1)
    with pytest.raises(eps.EpsError) as e:
        r.pull(feats)
    assert e.value.code == eps.UNAVAILABLE and "prepared" in str(e.value)
    p = r.pull_prepared(tok0)
    r.command("cancel_prepared", {"token": tok1})
    with pytest.raises(eps.EpsError) as e:
        r.command("cancel_prepared", {"token": tok1})
    assert e.value.code == eps.RETIRED_REQUEST
    with pytest.raises(eps.EpsError):
        r.pull_prepared(tok1)
    r.command("release", {"handle": p.handle})
    direct = r.pull(feats, read_only=True)       # same state: same outputs
    for a, b in zip(p.outputs, direct.outputs):
        assert np.array_equal(bits(a), bits(b))
    r.command("release", {"handle": direct.handle})
    r.command("join")
    for name in ("training_arm", "training_status"):
        with pytest.raises(eps.EpsError) as e:
            r.command(name)
        assert "not configured" in str(e.value)
    with pytest.raises(eps.EpsError):
        r.command("no_such_command")
    assert r.command("endpoint") == ""
    r.command("close")
    with pytest.raises(eps.EpsError) as e:
        r.command("stats")
    assert e.value.code == eps.UNAVAILABLE and "closed" in str(e.value)


@pytest.mark.gpu
def test_save_export_resume_and_restore(rt, eps):
    ts = _tables()
    with tempfile.TemporaryDirectory() as d:
        r, o = rt.NativeRuntime(config(ts, snapshot_directory=d)), Oracle(ts)
        for step in range(2):
            feats = _batch(30 + step)
            b = r.pull(feats)
            grads = _grads(b.outputs, 300 + step)
            _oracle_round(o, feats, grads)
            if step == 0:
                with pytest.raises(eps.EpsError) as e:     # a live batch blocks the save
                    r.command("save", {"id": "ckpt"})
                assert e.value.code == eps.UNAVAILABLE
            r.push(b.handle, [(f.feature, g) for f, g in zip(feats, grads)])
        paths = r.command("save", {"id": "ckpt-1"})
        assert paths == [os.path.join(d, "ckpt-1", "shard-0.bin")]
        with pytest.raises(eps.EpsError) as e:             # frozen
            r.pull(_batch(5))
        assert e.value.code == eps.UNAVAILABLE and "closed" in str(e.value)
        # export in chunks with the checksum continuation
        data, off, checksum, tail = b"", 0, 14695981039346656037, ""
        while True:
            c = r.command("read_checkpoint", {"id": "ckpt-1", "shard": 0, "offset": off,
                                              "max_bytes": 333, "checksum": checksum, "tail": tail})
            data += bytes.fromhex(c["data"])
            off, checksum, tail = c["offset"] + len(bytes.fromhex(c["data"])), c["checksum"], c["tail"]
            if c["eof"]:
                break
        assert data == open(paths[0], "rb").read()
        assert checksum == int.from_bytes(data[-8:], "little")
        with pytest.raises(eps.EpsError) as e:
            r.command("read_checkpoint", {"id": "other", "shard": 0, "offset": 0, "max_bytes": 8,
                                          "checksum": 14695981039346656037, "tail": ""})
        assert e.value.code == eps.UNAVAILABLE
        meta, tabs = eps.snapshot_inspect(paths[0])
        assert meta["run"] == "runtime-test" and meta["checksum"] == checksum
        assert sorted(t["id"] for t in tabs) == [1, 2]
        r.command("resume", {"id": "ckpt-1"})
        r.command("resume", {"id": "ckpt-1"})              # idempotent once resumed
        saved = [r.pull([_all_rows(t)], read_only=True).outputs[0] for t in ts]
        for t, w in zip(ts, saved):
            st, _ = o.state(t.id)
            assert np.array_equal(bits(w), bits(st[:, 0]))
        # a fresh runtime restored from the file continues identically
        r2 = rt.NativeRuntime(config(ts, run="runtime-test-2", restore=paths[0]))
        prov = r2.command("restored_from")[0]
        assert prov["loaded"] and prov["pristine"] and prov["source_run"] == "runtime-test"
        assert prov["bytes"] == len(data) and prov["checksum"] == checksum
        feats = _batch(40)
        b1, b2 = r.pull(feats), r2.pull(feats)
        for a, b in zip(b1.outputs, b2.outputs):
            assert np.array_equal(bits(a), bits(b))
        grads = _grads(b1.outputs, 400)
        r.push(b1.handle, [(f.feature, g) for f, g in zip(feats, grads)])
        r2.push(b2.handle, [(f.feature, g) for f, g in zip(feats, grads)])
        assert not r2.command("restored_from")[0]["pristine"]
        for t in ts:
            a = r.pull([_all_rows(t)], read_only=True).outputs[0]
            b = r2.pull([_all_rows(t)], read_only=True).outputs[0]
            assert np.array_equal(bits(a), bits(b))


@pytest.mark.gpu
def test_read_only_release_and_table_modes(rt, eps):
    ts = _tables()
    r = rt.NativeRuntime(config(ts))
    with pytest.raises(eps.EpsError):
        r.command("table_mode", {"table": 1, "prediction": True})   # needs release_read_only
    r = rt.NativeRuntime(config(ts, release_read_only=True))
    feats = _batch(3)
    assert r.pull(feats, read_only=True).handle == U64_MAX
    r.command("table_mode", {"table": 1, "prediction": True})
    t1 = [f for f in feats if f.table == 1]
    assert r.pull(t1).handle == U64_MAX                          # prediction table: read-only
    with pytest.raises(eps.EpsError) as e:
        r.pull(feats)                                           # mixes training and prediction
    assert "mixes" in str(e.value)
    r.command("table_mode", {"table": 1, "prediction": False})
    b = r.pull(feats)
    assert b.handle != U64_MAX
    r.command("release", {"handle": b.handle})
    r.command("abort")
    with pytest.raises(eps.EpsError):
        r.pull(feats)


@pytest.mark.gpu
@pytest.mark.skipif(not reference_available(), reason="oracle/_ref not built")
def test_reference_table_json_takes_any_64bit_key(rt):
    """A table in the reference's own JSON (no key_space) is a hashed table:
    random 64-bit keys, the all-ones key among them, rows created on first
    touch; three pull / push rounds and the final weights equal the reference's
    CPU parameter server (oracle/_ref) bit for bit."""
    rng = np.random.default_rng(21)
    t = TableDef(id=1, dimension=32, learning_rate=0.01, init_min=-0.05, init_max=0.05,
                 init_seed=42)
    j = table_json(t)
    del j["key_space"]
    j["capacity"] = 4096
    r = rt.NativeRuntime({"run": "hashed", "device": 0, "state_bytes": 1 << 28, "tables": [j]})
    ref = Reference([t], shards=1)
    pool = np.unique(np.concatenate([rng.integers(0, 2**63, size=600, dtype=np.int64)
                                     .astype(np.uint64) * np.uint64(2),
                                     np.array([U64_MAX], np.uint64)]))
    touched = set()
    for step in range(3):
        feats = []
        for fi, pooling in enumerate((SUM, MEAN, SEQUENCE)):
            lens = rng.integers(0, 7, size=32)
            offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.uint64)
            keys = pool[rng.integers(0, len(pool), size=int(offs[-1]))]
            touched.update(int(k) for k in keys)
            feats.append(Feature(1, 20 + fi, pooling, keys, offs))
        b = r.pull(feats)
        batch, want = ref.lookup(feats)
        for f, got, w in zip(feats, b.outputs, want):
            assert np.array_equal(bits(got), bits(w)), (step, f.feature)
        grads = _grads(b.outputs, 300 + step)
        r.push(b.handle, [(f.feature, g) for f, g in zip(feats, grads)])
        ref.push(batch, feats, grads)
    keys = np.array(sorted(touched), np.uint64)
    got = r.pull([types.SimpleNamespace(table=1, feature=99, pooling=SEQUENCE, keys=keys,
                                        offsets=np.array([0, len(keys)], np.uint64))],
                 read_only=True).outputs[0]
    rw, _, _, _ = ref.read_many(1, keys)
    assert np.array_equal(bits(got), bits(rw))
    ref.close()
    r.close()
