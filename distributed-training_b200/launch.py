"""Elastic restart-all launcher (behaviour of dtrain/launch.py:24-77).

    python -m dtrain_b200.launch --nproc N [--max-restarts K] [--timeout S] [--exit-log F] -- CMD ARGS...

One attempt = one rendezvous store namespace and N worker processes.  Each worker
gets RANK, LOCAL_RANK (its GPU on this node), WORLD_SIZE, STORE_ADDR,
DTRAIN_PREFIX=a{attempt}/, DTRAIN_RESTART_COUNT, DTRAIN_TIMEOUT and one BLAS/OpenMP
thread unless the caller set more.  The attempt succeeds when every worker exits 0.
The first worker to exit non-zero ends it: the launcher reports "rank r exited
with c", stops the rest of the group (SIGTERM to each worker's process group, then
SIGKILL after a grace period) and, while restarts remain, reports "restarting" and
starts a new attempt whose workers resume from the latest checkpoint.  The exit
code is 0, or the first failing worker's code when no restart is left.

How it differs from a polling loop: every worker runs in its own session (so a
signal reaches the processes it started too), and the launcher sleeps in
``poll(2)`` on the workers' pidfds, waking exactly when one of them exits.  Each
attempt's exits are kept as ``ExitRecord``s (``Launcher.history``) and, with
``--exit-log``, appended to a JSON-lines file.

On a GPU node a worker only leaves between steps (``--fail-at-step``
synchronises first), so none of its kernels or collectives is in flight; the
survivors' device-side waits time out into a host ``CommError`` (DTRAIN_TIMEOUT)
and they exit non-zero in turn.
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import os
import select
import signal
import subprocess
import sys
import time

from .utils.store import StoreServer

STOP_GRACE_S = 10.0


@dataclasses.dataclass
class ExitRecord:
    attempt: int
    rank: int
    pid: int
    code: int            # exit status, or -signal for a worker killed by a signal
    after_s: float       # seconds since the attempt started
    cause: str           # "ok", "failed" (first non-zero exit), "stopped" (ended by the launcher)


class _Attempt:
    """The N worker processes of one attempt and a blocking wait for their exits."""

    def __init__(self, index: int, cmd: list[str], envs: list[dict]):
        self.index = index
        self.t0 = time.monotonic()
        self.procs = [subprocess.Popen(cmd, env=env, start_new_session=True) for env in envs]
        self.rank_of = {p.pid: r for r, p in enumerate(self.procs)}
        self.fds: dict[int, int] = {}
        if hasattr(os, "pidfd_open"):
            for p in self.procs:
                try:
                    self.fds[os.pidfd_open(p.pid)] = p.pid
                except OSError:  # kernel without pidfds: fall back to short waits
                    self.fds.clear()
                    break
        self.live = set(self.rank_of)

    def next_exits(self, timeout: float | None, poll: float) -> list[tuple[int, int]]:
        """Block until at least one live worker exits (or ``timeout`` passes); returns
        [(rank, code)] for every worker found exited, reaped."""
        deadline = None if timeout is None else time.monotonic() + timeout
        while self.live:
            done = []
            if self.fds:
                pl = select.poll()
                for fd, pid in self.fds.items():
                    if pid in self.live:
                        pl.register(fd, select.POLLIN)
                wait_ms = None if deadline is None else max(0, int((deadline - time.monotonic()) * 1000))
                for fd, _ in pl.poll(wait_ms):
                    done.append(self.fds[fd])
            else:
                for p in self.procs:
                    if p.pid in self.live and p.poll() is not None:
                        done.append(p.pid)
                if not done:
                    time.sleep(poll)
            out = []
            for pid in done:
                p = self.procs[self.rank_of[pid]]
                out.append((self.rank_of[pid], p.wait()))
                self.live.discard(pid)
            if out:
                return sorted(out)
            if deadline is not None and time.monotonic() >= deadline:
                return []
        return []

    def signal_all(self, sig: int):
        for p in self.procs:
            if p.pid in self.live:
                try:
                    os.killpg(p.pid, sig)
                except ProcessLookupError:
                    pass

    def close(self):
        for fd in self.fds:
            os.close(fd)
        self.fds.clear()


class Launcher:
    """Restart-all supervisor; ``run()`` returns the job's exit code."""

    def __init__(self, nproc: int, cmd: list[str], max_restarts: int = 0, timeout: float = 60.0,
                 poll: float = 0.05, exit_log: str | None = None):
        if nproc < 1 or not cmd:
            raise ValueError("need --nproc >= 1 and a command")
        self.nproc, self.cmd, self.max_restarts = nproc, list(cmd), max_restarts
        self.timeout, self.poll, self.exit_log = timeout, poll, exit_log
        self.history: list[ExitRecord] = []

    def worker_env(self, store_addr: str, attempt: int, rank: int) -> dict:
        env = dict(os.environ)
        env.setdefault("OMP_NUM_THREADS", "1")
        env.setdefault("OPENBLAS_NUM_THREADS", "1")
        env.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(self.nproc), STORE_ADDR=store_addr,
                   DTRAIN_PREFIX=f"a{attempt}/", DTRAIN_RESTART_COUNT=str(attempt), DTRAIN_TIMEOUT=str(self.timeout))
        return env

    def _note(self, att: _Attempt, rank: int, code: int, cause: str):
        rec = ExitRecord(att.index, rank, att.procs[rank].pid, code, round(time.monotonic() - att.t0, 3), cause)
        self.history.append(rec)
        if self.exit_log:
            with open(self.exit_log, "a") as f:
                f.write(json.dumps(dataclasses.asdict(rec)) + "\n")

    def _stop(self, att: _Attempt):
        att.signal_all(signal.SIGTERM)
        end = time.monotonic() + STOP_GRACE_S
        while att.live:
            left = end - time.monotonic()
            if left <= 0:
                att.signal_all(signal.SIGKILL)
                left = None  # SIGKILL always ends them
            for rank, code in att.next_exits(left, self.poll):
                self._note(att, rank, code, "stopped")

    def _attempt(self, store_addr: str, index: int) -> int:
        """Runs one attempt; 0 when every worker exits 0, else the first failure's code."""
        att = _Attempt(index, self.cmd, [self.worker_env(store_addr, index, r) for r in range(self.nproc)])
        try:
            while att.live:
                exits = att.next_exits(None, self.poll)
                bad = [(r, c) for r, c in exits if c != 0]
                for r, c in exits:
                    self._note(att, r, c, "ok" if c == 0 else "failed")
                if bad:
                    r, c = bad[0]
                    print(f"[launch] attempt {index}: rank {r} exited with {c}; stopping the group",
                          file=sys.stderr, flush=True)
                    self._stop(att)
                    return c
            return 0
        finally:
            att.close()

    def run(self) -> int:
        store = StoreServer()
        try:
            code = 1
            for index in range(self.max_restarts + 1):
                code = self._attempt(store.address, index)
                if code == 0 or index == self.max_restarts:
                    return code
                print(f"[launch] restarting (restart {index + 1}/{self.max_restarts})", file=sys.stderr, flush=True)
            return code
        finally:
            store.close()


def run(nproc: int, cmd: list[str], max_restarts: int = 0, timeout: float = 60.0, poll: float = 0.05,
        exit_log: str | None = None) -> int:
    """Function form of ``Launcher(...).run()`` (the reference's ``launch.run`` signature,
    plus ``exit_log``; ``poll`` only matters on kernels without pidfds)."""
    return Launcher(nproc, cmd, max_restarts, timeout, poll, exit_log).run()


def main(argv=None):
    ap = argparse.ArgumentParser(description="restart-all launcher for dtrain_b200 workers")
    ap.add_argument("--nproc", type=int, required=True, help="workers (one per GPU on a GPU node)")
    ap.add_argument("--max-restarts", type=int, default=0)
    ap.add_argument("--timeout", type=float, default=60.0, help="DTRAIN_TIMEOUT for the workers' waits (s)")
    ap.add_argument("--exit-log", default=None, help="append one JSON line per worker exit to this file")
    ap.add_argument("cmd", nargs=argparse.REMAINDER)
    a = ap.parse_args(argv)
    cmd = list(a.cmd)
    if cmd[:1] == ["--"]:
        cmd = cmd[1:]
    sys.exit(Launcher(a.nproc, cmd, a.max_restarts, a.timeout, exit_log=a.exit_log).run())


if __name__ == "__main__":
    main()
