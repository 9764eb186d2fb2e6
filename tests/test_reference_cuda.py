"""The reference's own GPU path: its CUDA cache backend (src/cuda/cache_backend.cu,
the reference's eps_cuda target) compiled from the reference sources for sm_100a
by `make -C oracle ref-cuda`, attached to a CpuParameterService shard as its
agent, with the batch's rows migrated to it and the client's gathers resolved
through the reference's MakeCacheResolver (the wiring of the reference's
tests/cache_tests.cpp:45-49 with the CUDA backend).  It is the GPU baseline that
the B200 path is compared with.

* CPU: the library builds, and without a GPU attaching the backend fails with
  the reference's own CUDA error.
* ``refgpu`` marker (run explicitly, ``-m refgpu``, on a B200; not part of
  ``-m gpu``): pull + push rounds of cfg1, of cfg2 sub-batches (batch 1024: the backend
  stages at most 64 MiB and 16 MiB compact packets per call,
  src/cuda/cache_backend.cu:212-214, src/access/compact_gradients.cpp:15) and of
  cfg4 sub-batches (32,768 gradient rows; the push is also timed alone) through
  that path, timed on the host clock as the API is synchronous; the pulls must
  match the reference's CPU path within the reference CUDA test's tolerance
  (1e-5, tests/cuda_tests.cpp:14).  Prints one JSON line per config, also written
  to $EPS_REF_CUDA_OUT/ref_cuda_<config>.json when that variable names a folder."""
import ctypes
import json
import os
import subprocess
import time

import numpy as np
import pytest

from oracle_lib import REF_CUDA_SO, Feature, Reference, TableDef

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.environ.get("EPS_REFERENCE", os.path.join(
    os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))), "reference"))


def gpu_present():
    """A CUDA device answers (asked of the driver directly: no framework start-up)."""
    try:
        cuda = ctypes.CDLL("libcuda.so.1")
        count = ctypes.c_int(0)
        return cuda.cuInit(0) == 0 and cuda.cuDeviceGetCount(ctypes.byref(count)) == 0 \
            and count.value > 0
    except OSError:
        return False


def library():
    if os.path.isdir(os.path.join(REF, "src", "cuda")):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), f"REF={REF}", "ref-cuda"],
                       check=True, capture_output=True, timeout=900)
    if not os.path.exists(REF_CUDA_SO):
        pytest.skip("the reference's CUDA backend is not built (its sources are not present)")
    return REF_CUDA_SO


def as_reference(w):
    tables = [TableDef(id=t.id, dimension=t.dimension, learning_rate=1e-3, init_min=-0.05,
                       init_max=0.05, init_seed=7, rows=t.rows) for t in w.tables]
    feats = [Feature(f.table, f.feature, f.pooling, f.keys, f.offsets) for f in w.features]
    return w, tables, feats


def cfg2_subbatch(workloads, batch, seed=2):
    return as_reference(workloads.config2(seed=seed, batch=batch))


def test_reference_cuda_backend_fails_loudly_without_a_gpu(workloads):
    if gpu_present():
        pytest.skip("a GPU is present: the measurement runs under -m refgpu")
    lib = library()
    w, tables, feats = cfg2_subbatch(workloads, 16)
    ref = Reference(tables, shards=1, library=lib)
    batch, _ = ref.lookup(feats, read_only=True)
    ref.release(batch)
    with pytest.raises(ValueError, match="reference rejected"):
        ref.attach_cuda(tables[0].id, np.unique(np.concatenate([f.keys for f in feats]))[:8])
    ref.close()


@pytest.mark.refgpu
@pytest.mark.parametrize("config", ["cfg1", "cfg2-1024", "cfg4-32768"])
def test_reference_cuda_backend_rounds(workloads, config):
    if not gpu_present():
        pytest.skip("needs a GPU")
    lib = library()
    warmup, steps = 3, (100 if config == "cfg1" else 10)
    if config == "cfg1":
        w, tables, feats = as_reference(workloads.config1())
    elif config == "cfg4-32768":
        w, tables, feats = as_reference(workloads.config4(n=32768))
    else:
        w, tables, feats = cfg2_subbatch(workloads, 1024)
    ref = Reference(tables, shards=1, library=lib)
    cpu = Reference(tables, shards=1)
    b0, _ = ref.lookup(feats, read_only=True)     # creates the rows on the shard
    ref.release(b0)
    unique = 0
    for t in tables:
        keys = np.unique(np.concatenate([f.keys for f in feats if f.table == t.id]))
        ref.attach_cuda(t.id, keys)
        unique += len(keys)
    # first round against the CPU path
    b1, outs_gpu = ref.lookup(feats)
    c1, outs_cpu = cpu.lookup(feats)
    for g, c in zip(outs_gpu, outs_cpu):
        np.testing.assert_allclose(g, c, rtol=1e-5, atol=1e-5)
    ref.push(b1, feats, w.gradients)
    cpu.push(c1, feats, w.gradients)
    for _ in range(warmup):
        b, _ = ref.lookup(feats)
        ref.push(b, feats, w.gradients)
    t0 = time.perf_counter()
    push_s = 0.0
    for _ in range(steps):
        b, _ = ref.lookup(feats)
        p0 = time.perf_counter()
        ref.push(b, feats, w.gradients)
        push_s += time.perf_counter() - p0
    dt = (time.perf_counter() - t0) / steps
    b2, outs_gpu = ref.lookup(feats, read_only=True)
    ref.release(b2)
    # the CPU path after the same number of pushes
    for _ in range(warmup + steps):
        c, _ = cpu.lookup(feats)
        cpu.push(c, feats, w.gradients)
    c2, outs_cpu = cpu.lookup(feats, read_only=True)
    cpu.release(c2)
    for g, c in zip(outs_gpu, outs_cpu):
        np.testing.assert_allclose(g, c, rtol=1e-5, atol=1e-5)
    line = {"impl": "reference-cuda-backend", "metric": "embedding rows/s per round (pull+push+Adam)",
            "value": w.occurrences / dt, "unit": "rows/s", "ms_per_round": dt * 1e3,
            "push_ms_per_round": push_s / steps * 1e3,
            "workload": f"{config}: {w.occurrences} occurrences, {unique} unique rows, "
                        f"all resident on the GPU ({w.name})",
            "steps": steps, "warmup": warmup, "timing": "host clock around synchronous API calls"}
    print(json.dumps(line))
    out = os.environ.get("EPS_REF_CUDA_OUT")
    if out and os.path.isdir(out):
        with open(os.path.join(out, f"ref_cuda_{config}.json"), "w") as f:
            f.write(json.dumps(line) + "\n")
    ref.close()
    cpu.close()
