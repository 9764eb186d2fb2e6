"""The allocation-free lookup (eps_b200_lookup_noalloc) against the regular lookup.

Some callers cannot allocate GPU memory while serving a request (an inference
engine or framework that owns all device memory through its own pool, or a
latency-critical serving loop that must never wait on an allocator).  For them the
library offers a read-only pooled lookup whose per-call feature descriptors live
in a fixed per-GPU array instead of a freshly allocated block.  This test calls it
through the C ABI twice in a row, with different feature sets, and checks each
result bit for bit (the tolerance of every lookup parity test here) against
eps_b200_lookup on the same inputs.  The file is named to be collected last.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


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
    with pytest.raises(eps.EpsError) as e:
        too_many = _features(eps, torch, rng, [(1, eps.SUM, 5000, 2, 2)] * 257)
        store.lookup_noalloc(too_many, [torch.empty((2, 64), device="cuda")] * 257)
    assert e.value.code == eps.CAPACITY_EXCEEDED
    store.close()
