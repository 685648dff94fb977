"""Process groups and collectives.

Two backends share one API (the reference's, dtrain/comm.py:241-432):

* ``ProcessGroup`` (this module) - host memory over a TCP full mesh.  It serves
  the CPU ranks used by host-side fault tests and by the float64 oracle mode, and
  it is the bootstrap channel of the GPU backend.
* ``NVLinkGroup`` (``parallel/nvlink.py``) - CUDA tensors, collectives run as
  sm_100a kernels that read and write peer GPU memory over NVLink / NVSwitch.

Both use fixed summation orders, so every rank ends with bit-identical results:

* ``algo="ring"``:   chunk c of ``partition(n, W)`` is summed x_c + x_{c+1} + ... + x_{c-1}
  (the order a ring reduce-scatter produces, dtrain/comm.py:342-355);
* ``algo="direct"``: every element is summed x_0 + x_1 + ... + x_{W-1} (dtrain/comm.py:374-391).

Every message on the TCP backend carries (sequence number, byte count); a
mismatch raises ``CommError("protocol desync ...")`` instead of corrupting data,
and every blocking receive has a timeout (``DTRAIN_TIMEOUT``), so a crashed peer
surfaces as ``CommError`` rather than a hang.
"""
from __future__ import annotations

import os
import queue
import socket
import struct
import threading

import numpy as np

from ..utils.store import CommError, Store, StoreServer  # noqa: F401  (re-exported API)

_HDR = struct.Struct("<QQ")       # sequence number, payload bytes
_INLINE_MIN = 64 << 10            # sends up to this size always go out on the caller's thread
_INLINE_CAP = 1 << 20             # ... and up to this size when the socket buffers are large


def partition(n: int, world: int) -> list[int]:
    """Chunk boundaries shared by the ring collectives and ZeRO: rank r owns [b[r], b[r+1]).

    The first ``n % world`` ranks get one extra element (dtrain/comm.py:220-226);
    this fixes ZeRO shard sizes and therefore the checkpoint layout.
    """
    q, rem = divmod(int(n), int(world))
    bounds = [0]
    for r in range(world):
        bounds.append(bounds[-1] + q + (r < rem))
    return bounds


def _as_array(x) -> np.ndarray:
    """A NumPy view of a contiguous host array or CPU tensor (shares memory)."""
    if isinstance(x, np.ndarray):
        return x
    try:
        import torch
    except ImportError:  # pragma: no cover
        torch = None
    if torch is not None and isinstance(x, torch.Tensor):
        if x.device.type != "cpu":
            raise TypeError("the TCP process group works on host memory; use NVLinkGroup for CUDA tensors")
        return x.detach().numpy()
    raise TypeError(f"unsupported buffer type {type(x).__name__}")


class Work:
    """Handle of an asynchronous collective; ``wait()`` re-raises its error."""

    def __init__(self):
        self._done = threading.Event()
        self._error: BaseException | None = None

    def _finish(self, err: BaseException | None = None):
        self._error = err
        self._done.set()

    def is_completed(self) -> bool:
        return self._done.is_set()

    def wait(self):
        self._done.wait()
        if self._error is not None:
            raise self._error


class _Link:
    """One TCP connection to a peer, with a dedicated sender thread (full duplex)."""

    def __init__(self, sock: socket.socket, timeout: float):
        self.sock = sock
        sock.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
        for opt in (socket.SO_SNDBUF, socket.SO_RCVBUF):
            try:
                sock.setsockopt(socket.SOL_SOCKET, opt, 4 << 20)
            except OSError:
                pass
        sock.settimeout(timeout)
        # A send that fits in the kernel's socket buffers returns without waiting for the
        # reader, so it can go out on the caller's thread (no hand-off to the sender
        # thread).  Up to W-1 such messages of a ring may sit unread on one connection,
        # and Linux reports twice the usable buffer size, so the inline limit stays at a
        # sixteenth of the smaller reported buffer (8 unread messages still fit).
        try:
            room = min(sock.getsockopt(socket.SOL_SOCKET, socket.SO_SNDBUF),
                       sock.getsockopt(socket.SOL_SOCKET, socket.SO_RCVBUF))
        except OSError:
            room = 0
        self.inline_max = max(_INLINE_MIN, min(_INLINE_CAP, room // 16))
        self.error: BaseException | None = None
        self._jobs: queue.SimpleQueue = queue.SimpleQueue()
        self._pending = 0
        self._lock = threading.Lock()
        self._thread = threading.Thread(target=self._send_loop, name="dtb-link-send", daemon=True)
        self._thread.start()

    def _send_loop(self):
        while True:
            job = self._jobs.get()
            if job is None:
                return
            payload, done = job
            try:
                _sendall_chain(self.sock, payload)
            except BaseException as e:  # noqa: BLE001 - reported to the waiter
                self.error = e
            with self._lock:
                self._pending -= 1
            done.set()

    def post(self, seq: int, data: np.ndarray) -> threading.Event:
        view = memoryview(np.ascontiguousarray(data)).cast("B")
        done = threading.Event()
        hdr = _HDR.pack(seq, view.nbytes)
        with self._lock:
            idle = self._pending == 0
            if not (idle and view.nbytes <= self.inline_max):
                self._pending += 1
        if idle and view.nbytes <= self.inline_max:
            # fits in the socket buffer: sendall returns without waiting for the reader
            try:
                if view.nbytes <= _INLINE_MIN:
                    self.sock.sendall(hdr + view.tobytes())
                else:  # no copy of a large payload just to prepend the header
                    self.sock.sendall(hdr)
                    self.sock.sendall(view)
            except BaseException as e:  # noqa: BLE001
                self.error = e
            done.set()
            return done
        self._jobs.put((hdr + view.tobytes() if view.nbytes <= _INLINE_MIN else _Chain(hdr, view), done))
        return done

    def _recv_into(self, view: memoryview):
        got, n = 0, view.nbytes
        while got < n:
            try:
                k = self.sock.recv_into(view[got:], n - got)
            except socket.timeout as e:
                raise CommError("timed out waiting for a peer") from e
            except OSError as e:
                raise CommError(f"peer connection failed: {e}") from e
            if k == 0:
                raise CommError("peer closed the connection")
            got += k

    def fetch(self, seq: int, out: np.ndarray):
        hdr = bytearray(_HDR.size)
        self._recv_into(memoryview(hdr))
        rseq, nbytes = _HDR.unpack(hdr)
        if rseq != seq or nbytes != out.nbytes:
            raise CommError(f"protocol desync: expected seq {seq} / {out.nbytes} bytes, "
                            f"got seq {rseq} / {nbytes} bytes")
        if nbytes:
            self._recv_into(memoryview(out).cast("B"))

    def close(self, wait: float = 5.0):
        # the sender finishes what it holds, then exits; it is joined so no thread of
        # this link is still running when the interpreter shuts down
        self._jobs.put(None)
        self._thread.join(wait)
        try:
            self.sock.close()
        except OSError:
            pass


class _Chain:
    """Header + large payload sent without concatenating them."""

    def __init__(self, hdr: bytes, view: memoryview):
        self.hdr, self.view = hdr, view


def _sendall_chain(sock, payload):
    if isinstance(payload, _Chain):
        sock.sendall(payload.hdr)
        if payload.view.nbytes:
            sock.sendall(payload.view)
    else:
        sock.sendall(payload)


class ProcessGroup:
    """Host-memory collectives over a TCP full mesh (one connection per rank pair)."""

    backend = "tcp"

    def __init__(self, rank: int, world: int, store_addr: str, timeout: float = 60.0, prefix: str = ""):
        self.rank, self.world, self.timeout, self.prefix = int(rank), int(world), float(timeout), prefix
        self.seq = 0
        self.bytes_sent = 0
        self.store = Store(store_addr, timeout)
        self.links: dict[int, _Link] = {}
        srv = socket.create_server(("127.0.0.1", 0))
        srv.settimeout(timeout)
        self.store.set(f"{prefix}addr/{self.rank}", f"127.0.0.1:{srv.getsockname()[1]}".encode())
        # lower ranks accept, higher ranks dial: every pair gets exactly one connection
        for peer in range(self.rank):
            host, port = self.store.get(f"{prefix}addr/{peer}").decode().rsplit(":", 1)
            s = socket.create_connection((host, int(port)), timeout=timeout)
            s.sendall(struct.pack("<I", self.rank))
            self.links[peer] = _Link(s, timeout)
        for _ in range(self.world - self.rank - 1):
            try:
                s, _ = srv.accept()
            except socket.timeout as e:
                raise CommError("timed out waiting for peers to connect") from e
            s.settimeout(timeout)
            ident = b""
            while len(ident) < 4:
                more = s.recv(4 - len(ident))
                if not more:
                    raise CommError("peer closed during handshake")
                ident += more
            (peer,) = struct.unpack("<I", ident)
            self.links[peer] = _Link(s, timeout)
        srv.close()
        self._fifo: queue.SimpleQueue = queue.SimpleQueue()
        self._worker = threading.Thread(target=self._drain, name="dtb-comm-fifo", daemon=True)
        self._worker.start()
        self.barrier()

    # ------------------------------------------------------------ transport
    def _next(self) -> int:
        self.seq += 1
        return self.seq

    def _settle(self, link: _Link, ev: threading.Event):
        if not ev.wait(self.timeout):
            raise CommError("timed out sending to a peer")
        if link.error is not None:
            raise CommError(f"send failed: {link.error}")

    def _exchange(self, to: int, data: np.ndarray, frm: int, out: np.ndarray, seq: int):
        link = self.links[to]
        ev = link.post(seq, data)
        self.bytes_sent += data.nbytes
        self.links[frm].fetch(seq, out)
        self._settle(link, ev)

    # ---------------------------------------------------------- ring passes
    def _ring_reduce(self, flat: np.ndarray, bounds: list[int]):
        """W-1 ring steps; afterwards rank r holds the total of chunk (r+1) % W."""
        W, r = self.world, self.rank
        nxt, prv = (r + 1) % W, (r - 1) % W
        scratch = np.empty(max(bounds[i + 1] - bounds[i] for i in range(W)), flat.dtype)
        for step in range(W - 1):
            out_c, in_c = (r - step) % W, (r - step - 1) % W
            lo, hi = bounds[in_c], bounds[in_c + 1]
            recv = scratch[: hi - lo]
            self._exchange(nxt, flat[bounds[out_c]:bounds[out_c + 1]], prv, recv, self._next())
            flat[lo:hi] += recv

    def _ring_gather(self, flat: np.ndarray, bounds: list[int], first: int):
        """W-1 ring steps starting with rank r holding chunk (r + first) % W."""
        W, r = self.world, self.rank
        nxt, prv = (r + 1) % W, (r - 1) % W
        for step in range(W - 1):
            out_c, in_c = (r + first - step) % W, (r + first - step - 1) % W
            self._exchange(nxt, flat[bounds[out_c]:bounds[out_c + 1]], prv,
                           flat[bounds[in_c]:bounds[in_c + 1]], self._next())

    # ---------------------------------------------------------- collectives
    def allreduce(self, arr, algo: str = "ring"):
        """In-place sum over all ranks; returns ``arr``."""
        a = _as_array(arr)
        if self.world == 1:
            return arr
        if not a.flags.c_contiguous:
            raise ValueError("allreduce needs a contiguous array")
        flat = a.reshape(-1)
        if algo == "ring":
            bounds = partition(flat.size, self.world)
            self._ring_reduce(flat, bounds)
            self._ring_gather(flat, bounds, first=1)
        elif algo in ("direct", "oneshot"):
            self._direct(flat)
        else:
            raise ValueError(f"unknown all-reduce algorithm {algo!r}")
        return arr

    def _direct(self, flat: np.ndarray):
        seq = self._next()
        snapshot = flat.copy()
        posted = [(self.links[p], self.links[p].post(seq, snapshot)) for p in range(self.world) if p != self.rank]
        self.bytes_sent += flat.nbytes * (self.world - 1)
        parts = {self.rank: snapshot}
        for p in range(self.world):
            if p != self.rank:
                buf = np.empty_like(flat)
                self.links[p].fetch(seq, buf)
                parts[p] = buf
        for link, ev in posted:
            self._settle(link, ev)
        total = parts[0].copy()
        for p in range(1, self.world):
            total += parts[p]
        flat[...] = total

    def reduce_scatter(self, flat):
        """Sum over ranks; this rank's partition of ``flat`` then holds the total
        (other partitions hold partial sums).  Returns a view of that partition."""
        a = _as_array(flat)
        bounds = partition(a.size, self.world)
        if self.world > 1:
            self._ring_reduce(a, bounds)
            # one more hop so that rank r owns chunk r
            W, r = self.world, self.rank
            have = (r + 1) % W
            mine = np.empty(bounds[r + 1] - bounds[r], a.dtype)
            self._exchange((r + 1) % W, a[bounds[have]:bounds[have + 1]], (r - 1) % W, mine, self._next())
            a[bounds[r]:bounds[r + 1]] = mine
        lo, hi = bounds[self.rank], bounds[self.rank + 1]
        return flat[lo:hi]

    def all_gather(self, flat):
        """Copy each rank's partition of ``flat`` to every rank (in place)."""
        a = _as_array(flat)
        if self.world > 1:
            self._ring_gather(a, partition(a.size, self.world), first=0)
        return flat

    def broadcast(self, arr, root: int = 0):
        a = _as_array(arr)
        if self.world == 1:
            return arr
        flat = a.reshape(-1)
        seq = self._next()
        if self.rank == root:
            posted = [(self.links[p], self.links[p].post(seq, flat)) for p in range(self.world) if p != root]
            for link, ev in posted:
                self._settle(link, ev)
            self.bytes_sent += flat.nbytes * (self.world - 1)
        else:
            self.links[root].fetch(seq, flat)
        return arr

    def barrier(self):
        self.allreduce(np.zeros(1, np.float64))

    # --------------------------------------------------------------- async
    def allreduce_async(self, arr, algo: str = "ring") -> Work:
        """Queue an all-reduce on the comm thread (FIFO: all ranks issue in the same order)."""
        w = Work()
        self._fifo.put((arr, algo, w))
        return w

    def _drain(self):
        while True:
            job = self._fifo.get()
            if job is None:
                return
            arr, algo, w = job
            try:
                self.allreduce(arr, algo)
                w._finish()
            except BaseException as e:  # noqa: BLE001 - surfaced by Work.wait
                w._finish(e)

    def close(self):
        self._fifo.put(None)
        if self._worker is not threading.current_thread():
            self._worker.join(self.timeout)
        for link in self.links.values():
            link.close()
        self.store.close()


def init_from_env(timeout: float | None = None) -> ProcessGroup:
    """The default group from RANK / WORLD_SIZE / STORE_ADDR (set by the launcher)."""
    t = timeout if timeout is not None else float(os.environ.get("DTRAIN_TIMEOUT", "60"))
    return ProcessGroup(int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), os.environ["STORE_ADDR"], t,
                        prefix=os.environ.get("DTRAIN_PREFIX", ""))

