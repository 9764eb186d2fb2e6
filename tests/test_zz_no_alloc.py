"""The allocation-free lookup (eps_b200_lookup_noalloc) against the regular lookup.

Some callers cannot allocate GPU memory while serving a request (an inference
engine or framework that owns all device memory through its own pool, or a
latency-critical serving loop that must never wait on an allocator).  For them the
library offers a read-only pooled lookup whose per-call feature descriptors live
in a fixed per-GPU array instead of a freshly allocated block.  This test calls it
through the C ABI twice in a row, with different feature sets, and checks each
result bit for bit (the tolerance of every lookup parity test here) against
eps_b200_lookup on the same inputs.  It also checks the property the entry point
exists for: a call changes neither the device's free memory nor the
stream-ordered memory pool's usage.  The file is named to be collected last.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

_POOL_RESERVED_CURRENT, _POOL_USED_CURRENT = 5, 7     # cudaMemPoolAttr values


def _pool_usage(device):
    """(reserved, used) bytes of the device's default stream-ordered memory pool,
    read through the CUDA runtime the process has loaded; None if unavailable."""
    try:
        rt = ctypes.CDLL("libcudart.so.12")
    except OSError:
        return None
    pool = ctypes.c_void_p()
    if rt.cudaDeviceGetDefaultMemPool(ctypes.byref(pool), device):
        return None
    out = []
    for attr in (_POOL_RESERVED_CURRENT, _POOL_USED_CURRENT):
        v = ctypes.c_uint64(0)
        if rt.cudaMemPoolGetAttribute(pool, attr, ctypes.byref(v)):
            return None
        out.append(v.value)
    return tuple(out)


def _features(eps, torch, rng, specs):
    feats = []
    for fid, (table, pooling, rows, bags, max_bag) in enumerate(specs):
        lengths = rng.integers(0, max_bag + 1, size=bags)
        offsets = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
        keys = rng.integers(0, rows, size=int(offsets[-1])).astype(np.int64)
        feats.append(eps.FeatureInput(table, 10 + fid, pooling, torch.from_numpy(keys).cuda(),
                                      torch.from_numpy(offsets).cuda()))
    return feats


def test_noalloc_lookup_matches_regular_lookup_twice(eps):
    torch = pytest.importorskip("torch")
    store = eps.ParameterStore(device=0, state_bytes=1 << 30)
    store.create_table(eps.TableDefinition(id=1, dimension=64, key_space=5000))
    store.create_table(eps.TableDefinition(id=2, dimension=32, key_space=3000,
                                           initialization_seed=7))
    rng = np.random.default_rng(123)
    calls = [
        [(1, eps.SUM, 5000, 300, 20), (1, eps.MEAN, 5000, 200, 40), (2, eps.SEQUENCE, 3000, 50, 9),
         (2, eps.MEAN, 3000, 100, 3)],
        [(2, eps.SUM, 3000, 77, 64), (1, eps.SEQUENCE, 5000, 20, 5)],
    ]
    for specs in calls:
        feats = _features(eps, torch, rng, specs)
        _, expected = store.lookup(feats, read_only=True)
        outputs = [torch.full_like(e, float("nan")) for e in expected]
        store.lookup_noalloc(feats, outputs)
        store.synchronize()
        for got, want in zip(outputs, expected):
            assert got.shape == want.shape
            assert torch.equal(got.view(torch.int32), want.view(torch.int32))
        # the property itself: once the library's code is loaded (first call),
        # a call allocates nothing -- the device's free memory and the pool's
        # reserved / used bytes are the same before and after it
        torch.cuda.synchronize()
        free0, pool0 = torch.cuda.mem_get_info(0)[0], _pool_usage(0)
        store.lookup_noalloc(feats, outputs)
        store.synchronize()
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info(0)[0] == free0
        assert _pool_usage(0) == pool0
        for got, want in zip(outputs, expected):
            assert torch.equal(got.view(torch.int32), want.view(torch.int32))
    with pytest.raises(eps.EpsError) as e:
        too_many = _features(eps, torch, rng, [(1, eps.SUM, 5000, 2, 2)] * 257)
        store.lookup_noalloc(too_many, [torch.empty((2, 64), device="cuda")] * 257)
    assert e.value.code == eps.CAPACITY_EXCEEDED
    # the same per-feature checks as the regular lookup: a padding key together
    # with explicit valid lengths is refused by both
    keys = torch.tensor([1, 2, 3], dtype=torch.int64, device="cuda")
    offs = torch.tensor([0, 3], dtype=torch.int64, device="cuda")
    lens = torch.tensor([3], dtype=torch.int64, device="cuda")
    bad = [eps.FeatureInput(1, 99, eps.SUM, keys, offs, valid_lengths=lens, padding_key=0)]
    for call in (lambda: store.lookup(bad, read_only=True),
                 lambda: store.lookup_noalloc(bad, [torch.empty((1, 64), device="cuda")])):
        with pytest.raises(eps.EpsError) as e:
            call()
        assert e.value.code == eps.INVALID_ARGUMENT
    store.close()
