"""Multi-GPU round (distributed.ShardedClient): n ranks, rows sharded by key % n.

One round of n ranks must equal, bit for bit, the reference's DistributedClient
over n shards serving ONE combined request: the features of every rank in rank
order (ids r * F + f), then one push of all their gradients.

* gloo, world size 2, CPU: the exchange logic of ShardedClient (counts, payload,
  partial and gradient all-to-alls, agreed errors) over a numpy stand-in store;
  outputs against the oracle's n-shard lookup, pushed rows against a numpy
  ReduceGradients of the combined request;
* GPU, one device: n = 3 ranks emulated as threads (one ParameterStore per rank
  on the same GPU, in-process exchange), the real kernels end to end, outputs
  and the updated [w|m|v] + counters against the oracle;
* GPU, >= 2 devices: the same over NCCL, one process per GPU.
"""
from __future__ import annotations

import importlib
import os
import socket
import threading

import numpy as np
import pytest

import sharded_harness as H
from conftest import gpu_available, import_package
from oracle_lib import Feature, Oracle

F32 = np.float32


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _client_module():
    import_package()
    return importlib.import_module("eps_b200.distributed")


def _inputs(eps, feats, device):
    import torch
    return [eps.FeatureInput(f.table, f.feature, f.pooling,
                             torch.from_numpy(f.keys.astype(np.int64)).to(device),
                             torch.from_numpy(f.offsets.astype(np.int64)).to(device))
            for f in feats]


def test_payload_layout():
    D = _client_module()
    counts = np.array([[3, 2, 0], [0, 0, 0], [4, 1, 0]], np.uint64)
    keys_at, off_at, len_at, uniq_at, total = D.payload_layout(counts)
    assert list(keys_at) == [0, 3, 3] and list(off_at) == [7, 10, 11]
    assert list(len_at) == [7 + 3 + 3, 7 + 3 + 3 + 2, 7 + 3 + 3 + 2] and total == 7 + 2 * 3 + 3
    # a deduplicated group (4 keys in 4 one-key bags, 2 distinct): [0, 2, k, k]
    # after the lengths region
    counts = np.array([[3, 2, 0], [4, 4, 2]], np.uint64)
    keys_at, off_at, len_at, uniq_at, total = D.payload_layout(counts)
    assert list(keys_at) == [0, 3] and list(off_at) == [7, 10]
    assert list(len_at) == [7 + 6 + 2, 7 + 6 + 2 + 2] and list(uniq_at) == [21, 21]
    assert total == 7 + 2 * 6 + 2 + (2 + 2)


# ------------------------------------------------------------------ gloo, CPU
def _gloo_worker(rank, n, port, steps):
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=n,
                            init_method=f"tcp://127.0.0.1:{port}")
    try:
        eps = import_package()
        D = _client_module()
        oracle = Oracle(H.TABLES)
        weights = {t.id: oracle.state(t.id)[0][:, 0, :].copy() for t in H.TABLES}
        dims = {t.id: t.dimension for t in H.TABLES}
        store = H.FakeShardStore(rank, n, weights)
        client = D.ShardedClient(store, device="cpu")
        for step in range(steps):
            batches = [H.make_batch(r, step) for r in range(n)]
            feats, grads = batches[rank]
            handle, outs = client.lookup(_inputs(eps, feats, "cpu"))
            cf, cg = H.concat(batches)
            ref = oracle.lookup(cf, shards=n)
            F = len(feats)
            for f in range(F):
                assert np.array_equal(bits(outs[f].numpy()), bits(ref[rank * F + f])), (step, f)
            client.push(handle, [torch.from_numpy(g) for g in grads])
            want = H.reduce_gradients([(f.table, f.pooling, f.keys, f.offsets,
                                        np.diff(f.offsets.astype(np.int64))) for f in cf], cg, dims)
            got = H.reduce_gradients(*store.pushed[-1], dims)
            owned = {k: v for k, v in want.items() if k[1] % n == rank}
            assert set(got) == set(owned)
            for k, v in owned.items():
                assert np.array_equal(bits(got[k]), bits(v)), k
        # an invalid key on one rank is rejected on every rank, before any exchange
        feats, grads = H.make_batch(rank, 99)
        if rank == 1:
            feats[0].keys[0] = 10 ** 6
        with pytest.raises(eps.EpsError):
            client.lookup(_inputs(eps, feats, "cpu"))
        # a non-finite gradient on one rank rejects the push on every rank; the
        # round stays releasable
        feats, grads = H.make_batch(rank, 100)
        handle, outs = client.lookup(_inputs(eps, feats, "cpu"))
        if rank == 0:
            grads[1][0, 0] = np.inf
        with pytest.raises(eps.EpsError):
            client.push(handle, [torch.from_numpy(g) for g in grads], wait=True)
        client.release(handle)
        assert not store.routes and not store.tickets
    finally:
        dist.destroy_process_group()


def test_sharded_round_gloo_two_ranks():
    import torch.multiprocessing as mp
    mp.spawn(_gloo_worker, args=(2, _port(), 3), nprocs=2, join=True)


# ------------------------------------------------------- GPU, ranks as threads
def _make_store(eps, rank, n, device=0):
    s = eps.ParameterStore(device=device, shard_id=rank, shard_count=n, state_bytes=1 << 30)
    for t in H.TABLES:
        s.create_table(eps.TableDefinition(
            id=t.id, dimension=t.dimension, key_space=t.rows, learning_rate=t.learning_rate,
            beta1=t.beta1, beta2=t.beta2, epsilon=t.epsilon,
            initial_beta1_power=t.initial_beta1_power, initial_beta2_power=t.initial_beta2_power,
            weight_bounds=t.bounds, initialization_min=t.init_min, initialization_max=t.init_max,
            initialization_seed=t.init_seed, shard_count=n))
    return s


def _check_state(store, oracle, rank, n):
    for t in H.TABLES:
        keys = np.array([k for k in range(t.rows) if k % n == rank], np.uint64)
        w, m, v, u = store.read_state(t.id, keys)
        st, upd = oracle.state(t.id)
        assert np.array_equal(bits(w), bits(st[keys.astype(np.int64), 0]))
        assert np.array_equal(bits(m), bits(st[keys.astype(np.int64), 1]))
        assert np.array_equal(bits(v), bits(st[keys.astype(np.int64), 2]))
        assert np.array_equal(u, upd[keys.astype(np.int64)])
        assert store.optimizer_state(t.id)[0] == oracle.powers(t.id)[2]


def _rank_body(eps, D, store, client, rank, n, steps, device, oracle_outputs, oracle_lock,
               onehot=False):
    import torch
    for step in range(steps):
        batches = [H.make_batch(r, step, onehot=onehot) for r in range(n)]
        feats, grads = batches[rank]
        handle, outs = client.lookup(_inputs(eps, feats, device))
        with oracle_lock:
            ref = oracle_outputs[step]
        F = len(feats)
        for f in range(F):
            assert np.array_equal(bits(outs[f].cpu().numpy()), bits(ref[rank * F + f])), (step, f)
        client.push(handle, [torch.from_numpy(g).to(device) for g in grads], wait=True)


@pytest.mark.gpu
@pytest.mark.skipif(not gpu_available(), reason="needs a GPU")
@pytest.mark.parametrize("onehot", [False, True])
def test_sharded_round_three_ranks_one_gpu(onehot):
    """Three ranks as threads on one GPU against the oracle serving the combined
    request.  The sequence feature's groups (and, with `onehot`, the one-key sum
    and mean features') hold duplicate keys, so their owners return distinct
    rows only; outputs and state must still be bit-exact."""
    import torch
    eps = import_package()
    D = _client_module()
    n, steps = 3, 3
    oracle = Oracle(H.TABLES)
    outputs = {}
    for step in range(steps):                     # the combined requests, in order
        cf, cg = H.concat([H.make_batch(r, step, onehot=onehot) for r in range(n)])
        outputs[step] = oracle.lookup(cf, shards=n)
        assert oracle.push(cf, cg) == 0
    comm = H.ThreadComm(n)
    stores = [_make_store(eps, r, n) for r in range(n)]
    errors = []

    def run(rank):
        try:
            comm.bind(rank)
            torch.cuda.set_device(0)
            client = D.ShardedClient(stores[rank], device="cuda:0", comm=comm)
            _rank_body(eps, D, stores[rank], client, rank, n, steps, "cuda:0", outputs,
                       threading.Lock(), onehot=onehot)
        except BaseException as e:          # noqa: BLE001 -- reported below
            errors.append((rank, e))
            comm.barrier.abort()

    threads = [threading.Thread(target=run, args=(r,)) for r in range(n)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=300)
    assert not errors, errors
    for r, s in enumerate(stores):
        s.synchronize()
        _check_state(s, oracle, r, n)
        assert s.stats()["live_tickets"] == 0
        s.close()


def _drop_padding(f, pad):
    """PrepareAdapterInput (src/access/prepare_queue.cpp:58-85) on the host: the
    feature without its padding keys, and the kept positions."""
    keep = f.keys != np.uint64(pad)
    lens = np.diff(f.offsets.astype(np.int64))
    bag = np.repeat(np.arange(len(lens)), lens)
    kept = np.bincount(bag[keep], minlength=len(lens))
    offs = np.concatenate([[0], np.cumsum(kept)]).astype(np.uint64)
    return Feature(f.table, f.feature, f.pooling, f.keys[keep], offs), np.nonzero(keep)[0]


@pytest.mark.gpu
@pytest.mark.skipif(not gpu_available(), reason="needs a GPU")
def test_sharded_round_with_padding_three_ranks_one_gpu():
    """Adapter padding in the multi-GPU round: padding keys go to no shard, every
    shard gets the kept counts as valid lengths (mean divides by them), sequence
    positions holding padding read zeros -- bit for bit the reference's adapter
    (PrepareAdapterInput) followed by its n-shard lookup and push of the
    combined request."""
    import torch
    eps = import_package()
    D = _client_module()
    n, steps, pad = 3, 2, 7
    rng = np.random.default_rng(5)
    batches = {}
    for step in range(steps):
        for r in range(n):
            feats, grads = H.make_batch(r, step)
            for f in feats:
                f.keys[rng.random(len(f.keys)) < 0.3] = pad
            if len(feats[1].offsets) > 3 and feats[1].offsets[3] > feats[1].offsets[2]:
                feats[1].keys[int(feats[1].offsets[2]):int(feats[1].offsets[3])] = pad  # all padding
            batches[(r, step)] = (feats, grads)
    oracle = Oracle(H.TABLES)
    expect = {}
    for step in range(steps):
        cf, cg = H.concat([batches[(r, step)] for r in range(n)])
        compact = [_drop_padding(f, pad) for f in cf]
        outs = oracle.lookup([c for c, _ in compact], shards=n)
        full = []
        for f, (c, pos), o in zip(cf, compact, outs):
            if f.pooling == H.SEQUENCE:
                z = np.zeros((len(f.keys), o.shape[1]), np.float32)
                z[pos] = o
                full.append(z)
            else:
                full.append(o)
        expect[step] = full
        cgrads = [g[pos] if f.pooling == H.SEQUENCE else g
                  for f, (c, pos), g in zip(cf, compact, cg)]
        assert oracle.push([c for c, _ in compact], cgrads) == 0
    comm = H.ThreadComm(n)
    stores = [_make_store(eps, r, n) for r in range(n)]
    errors = []

    def run(rank):
        try:
            comm.bind(rank)
            torch.cuda.set_device(0)
            client = D.ShardedClient(stores[rank], device="cuda:0", comm=comm)
            for step in range(steps):
                feats, grads = batches[(rank, step)]
                ins = [eps.FeatureInput(f.table, f.feature, f.pooling,
                                        torch.from_numpy(f.keys.astype(np.int64)).cuda(),
                                        torch.from_numpy(f.offsets.astype(np.int64)).cuda(),
                                        padding_key=pad) for f in feats]
                handle, outs = client.lookup(ins)
                F = len(feats)
                for f in range(F):
                    assert np.array_equal(bits(outs[f].cpu().numpy()),
                                          bits(expect[step][rank * F + f])), (step, f)
                client.push(handle, [torch.from_numpy(g).cuda() for g in grads], wait=True)
        except BaseException as e:          # noqa: BLE001 -- reported below
            errors.append((rank, e))
            comm.barrier.abort()

    threads = [threading.Thread(target=run, args=(r,)) for r in range(n)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=300)
    assert not errors, errors
    for r, s in enumerate(stores):
        s.synchronize()
        _check_state(s, oracle, r, n)
        assert s.stats()["live_tickets"] == 0
        s.close()


# ------------------------------------------------------------ GPU, NCCL ranks
def _nccl_worker(rank, n, port, steps, kind):
    import datetime
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=n,
                            init_method=f"tcp://127.0.0.1:{port}",
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device(f"cuda:{rank}"))
    try:
        eps = import_package()
        D = _client_module()
        oracle = Oracle(H.TABLES)
        outputs = {}
        for step in range(steps):
            cf, cg = H.concat([H.make_batch(r, step) for r in range(n)])
            outputs[step] = oracle.lookup(cf, shards=n)
            assert oracle.push(cf, cg) == 0
        store = _make_store(eps, rank, n, device=rank)
        comm = D.NcclComm.from_process_group(rank)
        comm_in = D.NcclComm.from_process_group(rank)
        if kind == "native":
            client = D.NativeClient(store, comm, comm_in)
        else:
            client = D.ShardedClient(store, comm=comm, input_comm=comm_in)
        _rank_body(eps, D, store, client, rank, n, steps, f"cuda:{rank}", outputs,
                   threading.Lock())
        store.synchronize()
        _check_state(store, oracle, rank, n)
        # an invalid key on one rank is rejected on every rank before any exchange
        feats, grads = H.make_batch(rank, 99)
        if rank == 1:
            feats[0].keys[0] = 10 ** 6
        with pytest.raises(eps.EpsError):
            client.lookup(_inputs(eps, feats, f"cuda:{rank}"))
        # a non-finite gradient on one rank rejects the push on every shard
        feats, grads = H.make_batch(rank, 100)
        handle, outs = client.lookup(_inputs(eps, feats, f"cuda:{rank}"))
        if rank == 0:
            grads[1][0, 0] = np.nan
        with pytest.raises(eps.EpsError):
            client.push(handle, [torch.from_numpy(g).cuda(rank) for g in grads], wait=True)
        client.release(handle)
        store.synchronize()
        _check_state(store, oracle, rank, n)            # nothing was applied
        assert store.stats()["live_tickets"] == 0
        if kind == "native":
            client.close()
        comm.close()
        comm_in.close()
        store.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(not gpu_available(), reason="needs a GPU")
@pytest.mark.parametrize("kind", ["native", "python"])
def test_sharded_round_nccl_all_gpus(kind):
    """One process per GPU over NCCL: the C++ client (NativeClient, the measured
    path) and the Python ShardedClient over the library's NCCL communicator."""
    import torch
    import torch.multiprocessing as mp
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs at least two GPUs")
    n = min(n, 8)
    mp.spawn(_nccl_worker, args=(n, _port(), 3, kind), nprocs=n, join=True)
