"""SIGTERM handling of a GPU worker (train._StopRequest), on the host with a fake group.

A stopping worker may be blocked in a call that does not return to Python (on a GPU:
a synchronisation waiting on a collective whose peer is gone).  The signal must still
reach the group: a watcher thread, woken through ``signal.set_wakeup_fd``, calls the
group's ``abort()``.  Here the blocked call is a read from a pipe that only the fake
``abort()`` writes to, so the worker can only get out through the watcher."""
import os
import signal
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

WORKER = r"""
import os, sys
sys.path.insert(0, sys.argv[1])
from dtrain_b200.train import _StopRequest
r, w = os.pipe()

class FakeGroup:
    backend = "nvlink"
    def abort(self):
        os.write(w, b"A")

stop = _StopRequest().install()
stop.abort_on_signal(FakeGroup())
print("ready", flush=True)
got = os.read(r, 1)  # blocked: the SIGTERM handler alone would not end this read
print("unblocked", got.decode(), stop.requested, flush=True)
"""


def test_sigterm_aborts_the_group_while_the_main_thread_is_blocked():
    p = subprocess.Popen([sys.executable, "-c", WORKER, ROOT], stdout=subprocess.PIPE, text=True)
    try:
        assert p.stdout.readline().strip() == "ready"
        time.sleep(0.2)
        p.send_signal(signal.SIGTERM)
        out, _ = p.communicate(timeout=20)
    finally:
        if p.poll() is None:
            p.kill()
    assert p.returncode == 0
    assert out.strip() == "unblocked A True"


def test_cpu_groups_get_no_watcher():
    from dtrain_b200.train import _StopRequest

    class TcpGroup:
        backend = "tcp"

        def abort(self):
            raise AssertionError("a host group is never aborted by the watcher")

    stop = _StopRequest()
    stop.abort_on_signal(TcpGroup())
    assert stop._pipe is None
