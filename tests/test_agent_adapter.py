"""The GpuCacheAgent adapter (package agent/b200_cache_agent.cpp) on CPU.

tests/agent_check.cpp drives the adapter and the reference's own
HostCacheBackend (src/cache/host_backend.cpp) through the same seeded calls --
the backend contract directly, then behind a CpuParameterService with the agent
attached (the flow of the reference's tests/cache_tests.cpp) -- and requires
bit-identical results and equal error codes.  Here it is linked against
oracle/fake_b200_abi.cpp, a CPU stand-in of the C ABI built on the oracle, so
the adapter's host logic (residency map, slots, generations, budgets, skipped
occurrences as padding keys, error mapping) is checked without a GPU.  Linked
against the real libeps_b200.so it is the GPU test of the adapter (``-m gpu``:
the same calls plus GatherDevice on a B200); on a machine without a GPU that
build must fail loudly at construction (no CPU fallback).

The programs link the reference compiled from its sources (oracle/_ref), so
they are built only where the reference's headers are present."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.environ.get("EPS_REFERENCE", os.path.join(
    os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))), "reference"))
OUT = os.path.join(ROOT, "oracle", "_ref")


def build(target, binary):
    path = os.path.join(OUT, binary)
    if os.path.isdir(os.path.join(REF, "include", "eps")):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), f"REF={REF}", "ref", target],
                       check=True, capture_output=True, timeout=900)
    if not os.path.exists(path):
        pytest.skip("the reference's headers are not present to build " + binary)
    return path


def test_adapter_matches_host_cache_backend_bit_exact():
    exe = build("agent-fake", "agent_check_fake")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "agent_check: PASS" in r.stdout


@pytest.mark.skipif(not os.path.exists(os.path.join(
    ROOT, "distributed-recommendation-model-training-system_b200", "libeps_b200.so")),
    reason="libeps_b200.so is not built")
def test_adapter_on_the_real_library_fails_loudly_without_a_gpu():
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present: the real-library check is a GPU test")
    except ImportError:
        pass
    exe = build("agent", "agent_check")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 1
    assert "agent_check: FAIL B200 cache agent:" in r.stderr, r.stdout + r.stderr


@pytest.mark.gpu
def test_adapter_on_the_real_library_matches_host_cache_backend():
    exe = os.path.join(OUT, "agent_check")
    if os.path.isdir(os.path.join(REF, "include", "eps")):
        exe = build("agent", "agent_check")
    if not os.path.exists(exe):
        pytest.skip("agent_check is built where the reference's headers are present")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "agent_check: PASS" in r.stdout
    assert "device results not checked" not in r.stdout      # GatherDevice ran
