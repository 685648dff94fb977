"""CUDA VMM peer memory shared by file descriptor (NVLinkGroup(memory="vmm")).

Two processes on one GPU: each allocates with ``vmm_alloc``, fills its buffer,
passes the descriptor to the other over ``FdExchange`` and maps the other's buffer
with ``vmm_import``.  Every step is synchronised on the host (the store); no kernel
waits on the other process.  Then rank 1 unmaps its memory and exits, and rank 0
still reads rank 1's values through its own mapping: the importer's reference keeps
the physical memory alive after the exporter is gone.
"""
import multiprocessing as mp
import os
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

N = 1 << 20


def _rank(rank, addr, q):
    try:
        from dtrain_b200.ops._ext import lib
        from dtrain_b200.parallel.nvlink import FdExchange, store_exchange
        from dtrain_b200.utils.store import Store
        torch.cuda.set_device(0)
        C = lib()
        store = Store(addr)
        fdx = FdExchange(rank, 2, store_exchange(store, rank, 2, prefix="vmm-test/"), timeout=60)
        ptr, fd, size = C.vmm_alloc(N * 4)
        assert size >= N * 4
        mine = C.tensor_from_ptr(ptr, [N], torch.float32, 0)
        assert float(mine.abs().sum()) == 0.0, "vmm_alloc must zero the memory"
        mine.fill_(float(rank + 1))
        torch.cuda.synchronize()
        got = fdx.all_gather(fd, size)
        os.close(fd)
        pfd, psize = got[1 - rank]
        peer_ptr = C.vmm_import(pfd, psize)
        os.close(pfd)
        peer = C.tensor_from_ptr(peer_ptr, [N], torch.float32, 0)
        first = float(peer.sum())
        store.add("vmm-test/read", 1)
        while int(store.add("vmm-test/read", 0)) < 2:
            time.sleep(0.01)
        if rank == 1:
            # the exporter lets go of everything and leaves
            C.vmm_free(peer_ptr)
            C.vmm_free(ptr)
            store.set("vmm-test/gone", b"1")
            fdx.close()
            q.put((rank, (first, None)))
            return
        store.get("vmm-test/gone")  # blocks until rank 1 has unmapped and is exiting
        after = float(peer.sum())
        C.vmm_free(peer_ptr)
        C.vmm_free(ptr)
        fdx.close()
        q.put((rank, (first, after)))
    except BaseException as e:  # noqa: BLE001
        q.put((rank, e))


def test_vmm_peer_memory_maps_across_processes_and_outlives_the_exporter():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from dtrain_b200.utils.store import StoreServer
    srv = StoreServer()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_rank, args=(r, srv.address, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = dict(q.get(timeout=120) for _ in range(2))
    for p in ps:
        p.join(60)
    srv.close()
    for r in range(2):
        assert not isinstance(out[r], BaseException), out[r]
    assert out[0][0] == 2.0 * N and out[1][0] == 1.0 * N
    assert out[0][1] == 2.0 * N, "rank 1's memory must stay readable through rank 0's mapping"
