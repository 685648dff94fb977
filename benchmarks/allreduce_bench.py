"""Host (TCP) all-reduce latency and bus bandwidth of ``parallel.comm.ProcessGroup``.

Counterpart of the reference's benchmarks/allreduce_bench.py for the host
collectives:

    python benchmarks/allreduce_bench.py --world 4 --out results.json

``--impl reference`` (or ``both``) times the reference's own host ProcessGroup
from its installed copy in baseline/_ref on the same machine.

Starts ``--world`` processes on this machine (rendezvous store + TCP mesh over
loopback), then times the ``ring`` and ``direct`` all-reduce of float32 zeros
from 1 KiB to 64 MiB: the median of the timed calls after three warm-ups,
measured on rank 0 between barriers.  Bus bandwidth follows the NCCL convention,
2 (W-1)/W * bytes / time.  (The reference also compares OpenMPI; mpi4py is not
part of this image, so that column is not produced.)  The device collectives
over NVLink are measured by benchmarks/collectives_bench.py.
"""
from __future__ import annotations

import argparse
import json
import multiprocessing as mp
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

SIZES = [1 << k for k in range(10, 27, 2)]  # 1 KiB .. 64 MiB


def _reps(nbytes: int) -> int:
    return max(5, min(200, (64 << 20) // max(nbytes, 1) // 4))


def _rank_main(rank: int, world: int, addr: str, algos, q, impl: str = "ours"):
    if impl == "reference":
        # the reference's own host ProcessGroup, from its installed copy
        sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
        from dtrain.comm import ProcessGroup
    else:
        from dtrain_b200.parallel.comm import ProcessGroup
    pg = ProcessGroup(rank, world, addr, timeout=120)
    tag = "reference" if impl == "reference" else "dtrain_b200"
    rows = []
    for algo in algos:
        for nbytes in SIZES:
            x = np.zeros(nbytes // 4, np.float32)  # zeros: repeated sums stay finite
            for _ in range(3):
                pg.allreduce(x, algo)
            ts = []
            for _ in range(_reps(nbytes)):
                pg.barrier()
                t0 = time.perf_counter()
                pg.allreduce(x, algo)
                ts.append(time.perf_counter() - t0)
            sec = float(np.median(ts))
            rows.append({"impl": f"{tag}-{algo}", "world": world, "bytes": nbytes, "seconds": sec,
                         "latency_us": sec * 1e6, "bus_GBps": 2 * (world - 1) / world * nbytes / sec / 1e9})
    pg.close()
    if rank == 0:
        q.put(rows)


def run(world: int, algos=("ring", "direct"), impl: str = "ours") -> list:
    from dtrain_b200.utils.store import StoreServer
    srv = StoreServer()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, srv.address, algos, q, impl)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        rows = q.get(timeout=3600)
    finally:
        for p in procs:
            p.join(60)
            if p.is_alive():
                p.kill()
        srv.close()
    return rows


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--world", type=int, default=4)
    ap.add_argument("--algos", default="ring,direct")
    ap.add_argument("--out", default=None)
    ap.add_argument("--impl", choices=["ours", "reference", "both"], default="ours",
                    help="this stack's host ProcessGroup, the reference's (baseline/_ref), or both in turn")
    a = ap.parse_args(argv)
    os.environ.setdefault("OMP_NUM_THREADS", "1")
    impls = ["ours", "reference"] if a.impl == "both" else [a.impl]
    rows = [r for impl in impls for r in run(a.world, tuple(a.algos.split(",")), impl)]
    for r in rows:
        print(json.dumps(r))
    if a.out:
        with open(a.out, "w") as f:
            json.dump(rows, f, indent=1)
    return 0


if __name__ == "__main__":
    sys.exit(main())
