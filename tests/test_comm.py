"""Host collectives across real processes (2, 3 and 4 ranks) over TCP loopback.

Mirrors the reference's collective tests and adds bit-equality with the
reference's own algorithms (run from baseline/_ref on the same inputs).
"""
import multiprocessing as mp
import os
import sys

import numpy as np
import pytest

from dtrain_b200.parallel.comm import CommError, ProcessGroup, StoreServer, partition

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")


def _entry(rank, world, addr, fn, args, q, use_ref):
    try:
        if use_ref:
            sys.path.insert(0, REF)
            from dtrain.comm import ProcessGroup as RefPG
            pg = RefPG(rank, world, addr, timeout=30)
        else:
            pg = ProcessGroup(rank, world, addr, timeout=30)
        res = fn(pg, *args)
        pg.close()
        q.put((rank, res))
    except BaseException as e:  # noqa: BLE001
        q.put((rank, e))


def _run(world, fn, *args, timeout=90, use_ref=False):
    srv = StoreServer()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_entry, args=(r, world, srv.address, fn, args, q, use_ref)) for r in range(world)]
    for p in ps:
        p.start()
    out = {}
    for _ in range(world):
        r, res = q.get(timeout=timeout)
        out[r] = res
    for p in ps:
        p.join(timeout)
    srv.close()
    errs = [v for v in out.values() if isinstance(v, BaseException)]
    if errs:
        raise errs[0]
    return [out[r] for r in range(world)]


def _allreduce(pg, sizes, algo, dtype):
    out = []
    for i, n in enumerate(sizes):
        x = np.random.default_rng(1000 * i + pg.rank).standard_normal(n).astype(dtype)
        pg.allreduce(x, algo)
        out.append(x)
    return out


SIZES = [0, 1, 2, 3, 5, 7, 64, 1000, 12345]


@pytest.mark.parametrize("world", [2, 3, 4])
@pytest.mark.parametrize("algo", ["ring", "direct"])
def test_allreduce_matches_numpy_sum(world, algo):
    res = _run(world, _allreduce, SIZES, algo, np.float64)
    for i, n in enumerate(SIZES):
        expect = sum(np.random.default_rng(1000 * i + r).standard_normal(n) for r in range(world))
        for r in range(world):
            np.testing.assert_allclose(res[r][i], expect, rtol=1e-12, atol=1e-12)
            assert np.array_equal(res[r][i], res[0][i])


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "dtrain")), reason="reference not installed in baseline/_ref")
@pytest.mark.parametrize("algo", ["ring", "direct"])
def test_allreduce_bit_equal_to_reference_algorithms(algo):
    sizes = [1, 7, 1000, 12345]
    ours = _run(3, _allreduce, sizes, algo, np.float32)
    ref = _run(3, _allreduce, sizes, algo, np.float32, use_ref=True)
    for a, b in zip(ours, ref):
        for x, y in zip(a, b):
            assert np.array_equal(x, y)


def _rs_ag(pg, n):
    flat = np.arange(n, dtype=np.float64) * (pg.rank + 1)
    mine = np.array(pg.reduce_scatter(flat), copy=True)
    b = partition(n, pg.world)
    full = np.zeros(n)
    full[b[pg.rank]:b[pg.rank + 1]] = mine
    pg.all_gather(full)
    return mine, full


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("n", [1, 3, 10, 1001])
def test_reduce_scatter_and_all_gather(world, n):
    res = _run(world, _rs_ag, n)
    total = np.arange(n, dtype=np.float64) * sum(range(1, world + 1))
    b = partition(n, world)
    for r, (mine, full) in enumerate(res):
        np.testing.assert_array_equal(mine, total[b[r]:b[r + 1]])
        np.testing.assert_array_equal(full, total)


def _bcast_async(pg):
    x = np.full(100, float(pg.rank))
    pg.broadcast(x, root=1)
    works = [pg.allreduce_async(np.full(10, float(i + pg.rank))) for i in range(5)]
    for w in works:
        w.wait()
    return x


def test_broadcast_and_async_order():
    for x in _run(3, _bcast_async):
        np.testing.assert_array_equal(x, np.ones(100))


def _torch_fn(pg):
    import torch
    t = torch.full((17,), float(pg.rank + 1), dtype=torch.float64)
    pg.allreduce(t, "ring")
    return t.numpy().copy()


def test_torch_tensors_are_accepted():
    for x in _run(2, _torch_fn):
        np.testing.assert_array_equal(x, np.full(17, 3.0))


def test_partition_matches_reference_rule():
    assert partition(10, 4) == [0, 3, 6, 8, 10]
    assert partition(3, 4) == [0, 1, 2, 3, 3]
    assert partition(0, 2) == [0, 0, 0]


def _dies(pg):
    if pg.rank == 1:
        os._exit(3)  # crash without closing cleanly
    x = np.ones(1000)
    try:
        pg.allreduce(x)
    except CommError as e:
        return e
    return None


def test_peer_failure_raises_commerror_not_hang():
    srv = StoreServer()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_entry, args=(r, 2, srv.address, _dies, (), q, False)) for r in range(2)]
    for p in ps:
        p.start()
    r, res = q.get(timeout=60)
    assert r == 0 and isinstance(res, CommError)
    for p in ps:
        p.join(10)
    srv.close()


def test_store_wire_compatible_with_reference():
    if not os.path.isdir(os.path.join(REF, "dtrain")):
        pytest.skip("reference not installed")
    sys.path.insert(0, REF)
    try:
        from dtrain.comm import Store as RefStore
        from dtrain.comm import StoreServer as RefServer
    finally:
        sys.path.remove(REF)
    from dtrain_b200.utils.store import Store
    ours_srv, ref_srv = StoreServer(), RefServer()
    try:
        for srv_addr in (ours_srv.address, ref_srv.address):
            a, b = Store(srv_addr), RefStore(srv_addr)
            a.set("k", b"v1")
            assert b.get("k") == b"v1"
            assert a.add("n", 5) == 5 and b.add("n", 2) == 7
            a.close()
            b.close()
    finally:
        ours_srv.close()
        ref_srv.close()
