"""Elastic restart-all launcher (semantics of dtrain/launch.py:24-77).

    python -m dtrain_b200.launch --nproc N [--max-restarts K] [--timeout S] -- CMD ARGS...

Starts a rendezvous store and N workers with RANK, LOCAL_RANK, WORLD_SIZE,
STORE_ADDR, DTRAIN_PREFIX=a{attempt}/, DTRAIN_RESTART_COUNT, DTRAIN_TIMEOUT and
one BLAS thread each.  When a worker exits non-zero the launcher prints
"rank r exited with c", sends SIGTERM to the others (SIGKILL after 10 s) and,
while restarts remain, prints "restarting" and starts the whole group again in a
fresh rendezvous namespace; the training script resumes from its latest
checkpoint.  Exit code 0 when every worker of an attempt exits 0, otherwise the
failing worker's code.

On a GPU node each worker drives the GPU ``LOCAL_RANK``; a worker only leaves
between steps, so no kernel or collective of its own is in flight, and the
survivors' device-side waits time out into a host ``CommError`` (``DTRAIN_TIMEOUT``).
"""
from __future__ import annotations

import argparse
import os
import signal
import subprocess
import sys
import time

from .utils.store import StoreServer


def _stop_all(procs, grace: float = 10.0):
    for p in procs:
        if p.poll() is None:
            p.send_signal(signal.SIGTERM)
    deadline = time.monotonic() + grace
    for p in procs:
        try:
            p.wait(max(0.0, deadline - time.monotonic()))
        except subprocess.TimeoutExpired:
            p.kill()
            p.wait()


def run(nproc: int, cmd: list[str], max_restarts: int = 0, timeout: float = 60.0, poll: float = 0.05) -> int:
    store = StoreServer()
    try:
        code = 1
        for attempt in range(max_restarts + 1):
            procs = []
            for r in range(nproc):
                env = dict(os.environ)
                env.update(RANK=str(r), LOCAL_RANK=str(r), WORLD_SIZE=str(nproc), STORE_ADDR=store.address,
                           DTRAIN_PREFIX=f"a{attempt}/", DTRAIN_RESTART_COUNT=str(attempt),
                           DTRAIN_TIMEOUT=str(timeout),
                           OMP_NUM_THREADS=os.environ.get("OMP_NUM_THREADS", "1"),
                           OPENBLAS_NUM_THREADS=os.environ.get("OPENBLAS_NUM_THREADS", "1"))
                procs.append(subprocess.Popen(cmd, env=env))
            failed = None
            while failed is None:
                codes = [p.poll() for p in procs]
                for r, c in enumerate(codes):
                    if c not in (None, 0):
                        failed = (r, c)
                        break
                if failed is None:
                    if all(c == 0 for c in codes):
                        return 0
                    time.sleep(poll)
            r, code = failed
            print(f"[launch] attempt {attempt}: rank {r} exited with {code}; stopping the group",
                  file=sys.stderr, flush=True)
            _stop_all(procs)
            if attempt == max_restarts:
                return code
            print(f"[launch] restarting (restart {attempt + 1}/{max_restarts})", file=sys.stderr, flush=True)
        return code
    finally:
        store.close()


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--nproc", type=int, required=True)
    ap.add_argument("--max-restarts", type=int, default=0)
    ap.add_argument("--timeout", type=float, default=60.0)
    ap.add_argument("cmd", nargs=argparse.REMAINDER)
    a = ap.parse_args(argv)
    cmd = a.cmd[1:] if a.cmd and a.cmd[0] == "--" else a.cmd
    sys.exit(run(a.nproc, cmd, a.max_restarts, a.timeout))


if __name__ == "__main__":
    main()
