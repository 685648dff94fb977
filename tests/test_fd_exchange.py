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
        seen = []
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
        fdx.close()
        q.put((rank, seen))
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
        for call, row in enumerate(out[r]):
            for p in range(world):
                if p == r:
                    assert row[p] is None
                else:
                    assert row[p] == (f"rank {p} call {call}", 100 + call)
