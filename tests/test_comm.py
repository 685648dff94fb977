"""Host (TCP) collectives across real processes on loopback, 2 to 4 ranks.

Pinned behaviours (the reference's collective tests, tests/test_comm.py there):
all-reduce equals the fp64 sum and is bit-identical on every rank, for ring and
direct orders and awkward sizes (empty, single element, not divisible by the
world); reduce-scatter leaves each rank its partition of the total and all-gather
restores the whole buffer; broadcast copies the root's buffer; asynchronous
all-reduces complete in issue order; a peer that dies mid-collective makes the
survivor raise CommError instead of hanging.  Added here: bit-equality with the
reference's own algorithms on the same inputs, torch tensors as buffers, the
partition rule, and the store's wire compatibility with the reference's.
"""
import os
import sys
import time

import numpy as np
import pytest
from harness import HAVE_REF, REF, run_ranks

from dtrain_b200.parallel.comm import CommError, StoreServer, partition

SIZES = [0, 1, 4, 9, 31, 257, 4099, 20000]


def _rank_data(rank: int, n: int, tag: int, dtype=np.float64) -> np.ndarray:
    return np.random.default_rng([tag, rank]).standard_normal(n).astype(dtype)


def _allreduce_sizes(pg, algo, dtype):
    out = []
    for tag, n in enumerate(SIZES):
        x = _rank_data(pg.rank, n, tag, dtype)
        pg.allreduce(x, algo)
        out.append(x)
    return out


@pytest.mark.parametrize("algo", ["ring", "direct"])
@pytest.mark.parametrize("world", [2, 3, 4])
def test_allreduce_is_the_sum_and_identical_on_every_rank(world, algo):
    res = run_ranks(world, _allreduce_sizes, algo, np.float64)
    for tag, n in enumerate(SIZES):
        total = np.sum([_rank_data(r, n, tag) for r in range(world)], axis=0) if n else np.zeros(0)
        for r in range(world):
            assert res[r][tag].shape == (n,)
            np.testing.assert_allclose(res[r][tag], total, rtol=1e-12, atol=1e-12)
            assert res[r][tag].tobytes() == res[0][tag].tobytes(), (world, algo, n, r)


@pytest.mark.skipif(not HAVE_REF, reason="reference not installed in baseline/_ref")
@pytest.mark.parametrize("algo", ["ring", "direct"])
def test_allreduce_bits_equal_the_reference_algorithms(algo):
    ours = run_ranks(3, _allreduce_sizes, algo, np.float32)
    ref = run_ranks(3, _allreduce_sizes, algo, np.float32, group="reference")
    for a, b in zip(ours, ref):
        for x, y in zip(a, b):
            assert x.tobytes() == y.tobytes()


def _scatter_then_gather(pg, n):
    data = (np.arange(n, dtype=np.float64) % 97) * (pg.rank + 2)  # small integers: exact sums
    mine = np.array(pg.reduce_scatter(data), copy=True)
    b = partition(n, pg.world)
    rebuilt = np.full(n, np.nan)
    rebuilt[b[pg.rank]:b[pg.rank + 1]] = mine
    pg.all_gather(rebuilt)
    return mine, rebuilt


@pytest.mark.parametrize("world", [2, 3, 4])
@pytest.mark.parametrize("n", [1, 5, 17, 2049])
def test_reduce_scatter_then_all_gather_rebuilds_the_total(world, n):
    total = (np.arange(n, dtype=np.float64) % 97) * sum(r + 2 for r in range(world))
    b = partition(n, world)
    for r, (mine, rebuilt) in enumerate(run_ranks(world, _scatter_then_gather, n)):
        np.testing.assert_array_equal(mine, total[b[r]:b[r + 1]])
        np.testing.assert_array_equal(rebuilt, total)


def _broadcast_and_fifo(pg, k):
    x = np.arange(64, dtype=np.float64) + 100 * pg.rank
    pg.broadcast(x, root=pg.world - 1)
    bufs = [np.full(8, float(i * 10 + pg.rank)) for i in range(k)]
    works = [pg.allreduce_async(b) for b in bufs]
    for w in reversed(works):  # waiting out of order must not reorder the collectives
        w.wait()
    return x, [b[0] for b in bufs]


def test_broadcast_and_async_allreduces_complete_in_issue_order():
    world, k = 3, 6
    for x, firsts in run_ranks(world, _broadcast_and_fifo, k):
        np.testing.assert_array_equal(x, np.arange(64, dtype=np.float64) + 100 * (world - 1))
        assert firsts == [float(world * i * 10 + sum(range(world))) for i in range(k)]


def _sum_torch(pg):
    import torch
    t = torch.arange(11, dtype=torch.float64) * (pg.rank + 1)
    pg.allreduce(t, "direct")
    return t.numpy().copy()


def test_torch_tensors_are_reduced_in_place():
    for x in run_ranks(2, _sum_torch):
        np.testing.assert_array_equal(x, np.arange(11, dtype=np.float64) * 3)


def test_partition_gives_the_remainder_to_the_lowest_ranks():
    assert partition(10, 4) == [0, 3, 6, 8, 10]
    assert partition(3, 4) == [0, 1, 2, 3, 3]
    assert partition(0, 2) == [0, 0, 0]
    assert partition(7, 1) == [0, 7]


def _die_or_wait(pg):
    if pg.rank == 1:
        os._exit(3)  # gone without closing its sockets cleanly
    t0 = time.monotonic()
    try:
        pg.allreduce(np.ones(4096))
    except CommError as e:
        return ("commerror", time.monotonic() - t0, str(e)[:60])
    return ("no error", time.monotonic() - t0, "")


def test_dead_peer_raises_commerror_instead_of_hanging():
    (kind, waited, _), = run_ranks(2, _die_or_wait, expect=[0], timeout=20.0)
    assert kind == "commerror"
    assert waited < 20.0


@pytest.mark.skipif(not HAVE_REF, reason="reference not installed in baseline/_ref")
def test_store_wire_format_interoperates_with_the_reference():
    sys.path.insert(0, REF)
    try:
        from dtrain.comm import Store as RefStore
        from dtrain.comm import StoreServer as RefServer
    finally:
        sys.path.remove(REF)
    from dtrain_b200.utils.store import Store
    servers = [StoreServer(), RefServer()]
    try:
        for srv in servers:
            ours, theirs = Store(srv.address), RefStore(srv.address)
            ours.set("key", b"value")
            assert theirs.get("key") == b"value"
            theirs.set("back", b"\x00\x01")
            assert ours.get("back") == b"\x00\x01"
            assert ours.add("ctr", 5) == 5 and theirs.add("ctr", 2) == 7
            ours.close()
            theirs.close()
    finally:
        for srv in servers:
            srv.close()
