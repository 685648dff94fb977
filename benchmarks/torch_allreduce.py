"""This package's all-reduce against torch.distributed.all_reduce: exactness and speed.

Counterpart of the reference's benchmarks/torch_allreduce.py (same flags, same
JSON layout).  Host ranks over TCP compare the ``ring`` all-reduce of
``parallel.comm.ProcessGroup`` with gloo:

    python -m dtrain_b200.launch --nproc 4 -- python benchmarks/torch_allreduce.py \
        --torch-init /tmp/gloo_ar --out ar.json

1. Exactness: every rank draws float32 and float64 arrays (rank-dependent seed);
   both libraries reduce the same inputs.  Rank 0 records, per dtype, the largest
   difference between the two results, the fraction of bit-identical elements and
   each library's error against the exactly rounded sum (math.fsum).
2. Speed (unless --no-speed): median host latency of float32 all-reduces from
   1 KiB to 64 MiB between barriers, with bus bandwidth 2 (W-1)/W * bytes / time.

The GPU comparison (NVLink kernels vs NCCL, device-timed) is
benchmarks/collectives_bench.py.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from dtrain_b200.parallel.comm import init_from_env  # noqa: E402

SIZES = [1 << k for k in range(10, 27, 2)]


def _reps(nbytes: int) -> int:
    return max(5, min(200, (64 << 20) // max(nbytes, 1) // 4))


def _exactness(pg, n: int, dtype) -> dict:
    world, rank = pg.world, pg.rank
    xs = [np.random.default_rng([7, r]).standard_normal(n).astype(dtype) for r in range(world)]
    ours = xs[rank].copy()
    pg.allreduce(ours, "ring")
    t = torch.from_numpy(xs[rank].copy())
    dist.all_reduce(t)
    gloo = t.numpy()
    if rank != 0:
        return {}
    stacked = np.stack([x.astype(np.float64) for x in xs], axis=1)
    exact = np.array([math.fsum(row) for row in stacked])
    return {
        "max_abs_diff_dtrain_vs_gloo": float(np.max(np.abs(ours.astype(np.float64) - gloo))),
        "bit_identical_frac": float(np.mean(ours == gloo)),
        "max_abs_err_dtrain": float(np.max(np.abs(ours.astype(np.float64) - exact))),
        "max_abs_err_gloo": float(np.max(np.abs(gloo.astype(np.float64) - exact))),
        "max_abs_value": float(np.max(np.abs(exact))),
    }


def _speed(pg, world: int) -> list:
    rows = []
    for impl in ("dtrain-ring", "gloo"):
        for nbytes in SIZES:
            x = np.zeros(nbytes // 4, np.float32)
            tx = torch.from_numpy(x)
            op = (lambda: pg.allreduce(x, "ring")) if impl == "dtrain-ring" else (lambda: dist.all_reduce(tx))
            for _ in range(3):
                op()
            ts = []
            for _ in range(_reps(nbytes)):
                pg.barrier()
                dist.barrier()
                t0 = time.perf_counter()
                op()
                ts.append(time.perf_counter() - t0)
            sec = float(np.median(ts))
            rows.append({"impl": impl, "bytes": nbytes, "seconds": sec, "latency_us": sec * 1e6,
                         "bus_GBps": 2 * (world - 1) / world * nbytes / sec / 1e9})
    return rows


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--torch-init", required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--n-check", type=int, default=200_000)
    ap.add_argument("--no-speed", action="store_true")
    a = ap.parse_args(argv)
    torch.set_num_threads(1)
    pg = init_from_env()
    dist.init_process_group("gloo", init_method=f"file://{a.torch_init}", rank=pg.rank, world_size=pg.world)
    result = {"world": pg.world, "torch": torch.__version__, "check": {}, "speed": []}
    for dtype in (np.float32, np.float64):
        rec = _exactness(pg, a.n_check, dtype)
        if rec:
            result["check"][np.dtype(dtype).name] = rec
    if not a.no_speed:
        result["speed"] = _speed(pg, pg.world)
    if pg.rank == 0:
        with open(a.out, "w") as f:
            json.dump(result, f, indent=1)
    dist.barrier()
    dist.destroy_process_group()
    pg.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
