"""File-descriptor all-gather between processes (the hand-off of CUDA VMM peer memory),
exercised with ordinary files on CPU ranks: every rank must receive a working
descriptor of every peer's file, in rank order, over several numbered calls."""
import multiprocessing as mp
import os
import tempfile

from dtrain_b200.parallel.nvlink import FdExchange, store_exchange
from dtrain_b200.utils.store import Store, StoreServer


def _rank(rank, world, addr, tmp, q):
    try:
        ex = store_exchange(Store(addr), rank, world, prefix="fdx-test/")
        fdx = FdExchange(rank, world, ex, timeout=30)
        seen, kept = [], []
        for call in range(3):
            path = os.path.join(tmp, f"r{rank}c{call}")
            with open(path, "wb") as f:
                f.write(f"rank {rank} call {call}".encode())
            fd = os.open(path, os.O_RDONLY)
            got = fdx.all_gather(fd, 100 + call)
            os.close(fd)
            row = []
            for r, g in enumerate(got):
                if r == rank:
                    assert g is None
                    row.append(None)
                    continue
                pfd, size = g
                row.append((os.pread(pfd, 64, 0).decode(), size))
                os.close(pfd)
            seen.append(row)
            kept.append(len(fdx.pending))
        fdx.close()
        q.put((rank, (seen, kept)))
    except BaseException as e:  # noqa: BLE001
        q.put((rank, e))


def test_descriptors_reach_every_peer_in_order():
    world = 3
    srv = StoreServer()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with tempfile.TemporaryDirectory() as tmp:
        ps = [ctx.Process(target=_rank, args=(r, world, srv.address, tmp, q)) for r in range(world)]
        for p in ps:
            p.start()
        out = dict(q.get(timeout=60) for _ in range(world))
        for p in ps:
            p.join(30)
    srv.close()
    for r in range(world):
        assert not isinstance(out[r], BaseException), out[r]
        for call, row in enumerate(out[r][0]):
            for p in range(world):
                if p == r:
                    assert row[p] is None
                else:
                    assert row[p] == (f"rank {p} call {call}", 100 + call)


def _rank_slow_sender(rank, world, addr, tmp, q):
    """Rank 2 pauses after its first send, so rank 0 finishes call 0 and sends its call-1
    descriptor to rank 1 while rank 1 still waits for rank 2's call-0 message: rank 1 must
    keep the early message for call 1."""
    import socket
    import time
    if rank == 2:
        orig = socket.send_fds
        state = {"n": 0}

        def slow(sock, buffers, fds, *args, **kw):
            out = orig(sock, buffers, fds, *args, **kw)
            state["n"] += 1
            if state["n"] == 1:
                time.sleep(1.0)
            return out
        socket.send_fds = slow
    _rank(rank, world, addr, tmp, q)


def test_a_message_for_the_next_call_is_kept_until_then():
    world = 3
    srv = StoreServer()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with tempfile.TemporaryDirectory() as tmp:
        ps = [ctx.Process(target=_rank_slow_sender, args=(r, world, srv.address, tmp, q)) for r in range(world)]
        for p in ps:
            p.start()
        out = dict(q.get(timeout=60) for _ in range(world))
        for p in ps:
            p.join(30)
    srv.close()
    for r in range(world):
        assert not isinstance(out[r], BaseException), out[r]
        for call, row in enumerate(out[r][0]):
            for p in range(world):
                assert row[p] is None if p == r else row[p] == (f"rank {p} call {call}", 100 + call)
    assert out[1][1][0] >= 1, "rank 1 should have held rank 0's call-1 message while finishing call 0"


def _rank_bcast(rank, world, addr, tmp, q):
    """Broadcasts from alternating roots interleaved with an all-gather: the numbered
    calls keep each descriptor with its own call."""
    try:
        ex = store_exchange(Store(addr), rank, world, prefix="fdx-bcast/")
        fdx = FdExchange(rank, world, ex, timeout=30)
        seen = []
        for call, root in enumerate([0, 2, 1]):
            fd = None
            if rank == root:
                path = os.path.join(tmp, f"root{root}c{call}")
                with open(path, "wb") as f:
                    f.write(f"from {root} call {call}".encode())
                fd = os.open(path, os.O_RDONLY)
            got = fdx.broadcast(fd, 7 + call if rank == root else 0, root=root)
            if rank == root:
                os.close(fd)
                assert got is None
                seen.append(None)
            else:
                pfd, size = got
                seen.append((os.pread(pfd, 64, 0).decode(), size))
                os.close(pfd)
            mine = os.open(os.devnull, os.O_RDONLY)
            assert sum(g is not None for g in fdx.all_gather(mine, 1)) == world - 1
            os.close(mine)
        fdx.close()
        q.put((rank, seen))
    except BaseException as e:  # noqa: BLE001
        q.put((rank, e))


def test_broadcast_reaches_every_other_rank():
    world = 3
    srv = StoreServer()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with tempfile.TemporaryDirectory() as tmp:
        ps = [ctx.Process(target=_rank_bcast, args=(r, world, srv.address, tmp, q)) for r in range(world)]
        for p in ps:
            p.start()
        out = dict(q.get(timeout=60) for _ in range(world))
        for p in ps:
            p.join(30)
    srv.close()
    for r in range(world):
        assert not isinstance(out[r], BaseException), out[r]
        for call, root in enumerate([0, 2, 1]):
            assert out[r][call] == (None if r == root else (f"from {root} call {call}", 7 + call))
