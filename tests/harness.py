"""Shared machinery for the multi-process tests.

``run_ranks(world, body, *args, group=...)`` starts a rendezvous store and one
spawned process per rank; each builds a process group of the requested kind
(this stack's TCP group, the reference's TCP group from ``baseline/_ref``, or
this stack's NVLink group on GPU ``rank``, optionally with NVSwitch multicast), calls ``body(pg, *args)`` and sends
the result back.  Results come back in rank order; the first rank that raised
makes the call raise (with that rank's traceback).  A body may also end its
process on purpose (a crash test); ``expect`` then names the ranks whose
results the caller waits for.

``run_job(workdir, mode, world, flags)`` runs the training CLI - directly for
``--mode single``, through the restart-all launcher otherwise - and returns the
exit code, the saved parameters, the JSON log lines and stderr.
"""
from __future__ import annotations

import dataclasses
import json
import multiprocessing as mp
import os
import subprocess
import sys
import traceback

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")
HAVE_REF = os.path.isdir(os.path.join(REF, "dtrain"))
PY = sys.executable


class RankError(RuntimeError):
    pass


def _make_group(kind: str, rank: int, world: int, addr: str, timeout: float):
    if kind == "tcp":
        from dtrain_b200.parallel.comm import ProcessGroup
        return ProcessGroup(rank, world, addr, timeout=timeout)
    if kind == "reference":
        sys.path.insert(0, REF)
        from dtrain.comm import ProcessGroup as RefGroup
        return RefGroup(rank, world, addr, timeout=timeout)
    if kind in ("nvlink", "nvls"):
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        import torch
        from dtrain_b200.parallel.nvlink import NVLinkGroup, store_exchange
        from dtrain_b200.utils.store import Store
        torch.cuda.set_device(rank)
        store = Store(addr, 60)
        return NVLinkGroup(rank, world, torch.device("cuda", rank), store_exchange(store, rank, world),
                           timeout=timeout, nvls=(kind == "nvls"))
    raise ValueError(kind)


def _rank_main(rank, world, addr, kind, timeout, body, args, q):
    pg = None
    try:
        pg = _make_group(kind, rank, world, addr, timeout)
        res = body(pg, *args)
        pg.close()
        pg = None
        q.put((rank, "ok", res))
    except BaseException as e:  # noqa: BLE001 - everything goes back to the test
        q.put((rank, "error", f"{e!r}\n{traceback.format_exc()}"))
    finally:
        # a multicast-mapped group is always closed (all ranks barrier, then unbind):
        # a process must not exit with its memory still bound to the switch
        if pg is not None and kind == "nvls":
            try:
                pg.close()
            except BaseException:  # noqa: BLE001
                pass


def run_ranks(world: int, body, *args, group: str = "tcp", timeout: float = 30.0, wait_s: float = 240.0,
              expect=None):
    from dtrain_b200.utils.store import StoreServer
    srv = StoreServer()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, srv.address, group, timeout, body, args, q))
             for r in range(world)]
    for p in procs:
        p.start()
    want = list(range(world)) if expect is None else list(expect)
    got = {}
    try:
        while len(got) < len(want):
            r, status, res = q.get(timeout=wait_s)
            got[r] = (status, res)
    finally:
        for p in procs:
            p.join(30)
            if p.is_alive():
                p.kill()
        srv.close()
    for r in sorted(got):
        if got[r][0] == "error":
            raise RankError(f"rank {r} failed:\n{got[r][1]}")
    return [got[r][1] for r in want]


@dataclasses.dataclass
class Job:
    code: int
    params: dict | None
    log: list
    stderr: str


def run_job(workdir, mode: str, world: int = 1, flags=(), *, name: str, restarts: int = 0,
            package: str = "dtrain_b200", launcher_flags=(), timeout: float = 600.0) -> Job:
    """One training run; ``name`` keys its output files inside ``workdir``."""
    params_path = os.path.join(str(workdir), f"{name}.npz")
    log_path = os.path.join(str(workdir), f"{name}.jsonl")
    worker = [PY, "-m", f"{package}.train", "--mode", mode, "--save-params", params_path, "--log", log_path,
              *flags]
    if mode == "single":
        cmd = worker
    else:
        cmd = [PY, "-m", f"{package}.launch", "--nproc", str(world), "--max-restarts", str(restarts),
               "--timeout", "30", *launcher_flags, "--", *worker]
    path = REF if package == "dtrain" else ROOT
    env = dict(os.environ, OMP_NUM_THREADS="1", OPENBLAS_NUM_THREADS="1",
               PYTHONPATH=path + os.pathsep + os.environ.get("PYTHONPATH", ""))
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=timeout, cwd=ROOT)
    params = dict(np.load(params_path)) if os.path.exists(params_path) else None
    log = [json.loads(line) for line in open(log_path)] if os.path.exists(log_path) else []
    return Job(r.returncode, params, log, r.stderr)


def max_param_diff(a: dict, b: dict) -> float:
    assert a is not None and b is not None, "a run saved no parameters"
    assert a.keys() == b.keys()
    return max(float(np.max(np.abs(a[k] - b[k]))) for k in a)


def launch_script(workdir, world: int, script: str, args, tag: str, timeout: float = 600.0):
    """Runs ``benchmarks/<script>`` on ``world`` CPU ranks through the launcher, with a
    fresh gloo rendezvous file; raises with the tail of the output on failure."""
    init = os.path.join(str(workdir), f"rdv-{tag}")
    cmd = [PY, "-m", "dtrain_b200.launch", "--nproc", str(world), "--timeout", "60", "--",
           PY, os.path.join(ROOT, "benchmarks", script), "--torch-init", init, *args]
    env = dict(os.environ, OMP_NUM_THREADS="1", OPENBLAS_NUM_THREADS="1", MKL_NUM_THREADS="1",
               PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=timeout, cwd=ROOT)
    if r.returncode != 0:
        raise RankError(f"{script} on {world} ranks failed:\n{r.stdout[-2000:]}\n{r.stderr[-3000:]}")
    return r
