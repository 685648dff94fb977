"""Rendezvous key/value store over TCP (host side).

Behaviour and wire format follow the reference store (dtrain/comm.py:40-124) so a
client of either can talk to a server of the other:

* request  = ``<BII>`` (op, key length, value length) + key bytes + value bytes
* response = ``<I>`` (value length) + value bytes
* op 1 ``set``  stores the value and wakes waiters
* op 2 ``get``  blocks until the key exists, then returns its value
* op 3 ``add``  adds an integer (decimal text) to the key (missing = 0), returns the new value

Additional ops used only by this package: 4 ``check`` (non-blocking: returns
b"1" if the key exists, else b"0") and 5 ``delete``.

The server runs one accept thread and one thread per client connection; all
state sits behind a single condition variable.  The client retries the initial
connection until a deadline, like the reference, and raises ``CommError`` when
the server goes away.
"""
from __future__ import annotations

import socket
import struct
import threading
import time

_REQ = struct.Struct("<BII")
_LEN = struct.Struct("<I")

OP_SET, OP_GET, OP_ADD, OP_CHECK, OP_DELETE = 1, 2, 3, 4, 5


class CommError(RuntimeError):
    """A peer, the store, or a device-side wait failed (crash, timeout, desync)."""


def _read_exact(sock: socket.socket, n: int) -> bytes | None:
    chunks, got = [], 0
    while got < n:
        try:
            b = sock.recv(n - got)
        except OSError:
            return None
        if not b:
            return None
        chunks.append(b)
        got += len(b)
    return b"".join(chunks)


class StoreServer:
    """Threaded TCP key/value server.  ``address`` is ``"host:port"``."""

    def __init__(self, host: str = "127.0.0.1", port: int = 0):
        self._listener = socket.create_server((host, port), reuse_port=False)
        self._listener.settimeout(0.2)
        self._kv: dict[str, bytes] = {}
        self._cv = threading.Condition()
        self._closing = False
        self._clients: list[socket.socket] = []
        self._acceptor = threading.Thread(target=self._accept_loop, name="dtb-store-accept", daemon=True)
        self._acceptor.start()

    @property
    def address(self) -> str:
        h, p = self._listener.getsockname()[:2]
        return f"{h}:{p}"

    def _accept_loop(self):
        while not self._closing:
            try:
                conn, _ = self._listener.accept()
            except socket.timeout:
                continue
            except OSError:
                return
            conn.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
            self._clients.append(conn)
            threading.Thread(target=self._serve, args=(conn,), name="dtb-store-conn", daemon=True).start()

    def _apply(self, op: int, key: str, val: bytes) -> bytes | None:
        with self._cv:
            if op == OP_SET:
                self._kv[key] = val
                self._cv.notify_all()
                return b""
            if op == OP_GET:
                while key not in self._kv:
                    if self._closing:
                        return None
                    self._cv.wait(0.5)
                return self._kv[key]
            if op == OP_ADD:
                cur = int(self._kv.get(key, b"0")) + int(val)
                self._kv[key] = str(cur).encode()
                self._cv.notify_all()
                return self._kv[key]
            if op == OP_CHECK:
                return b"1" if key in self._kv else b"0"
            if op == OP_DELETE:
                self._kv.pop(key, None)
                return b""
        return None

    def _serve(self, conn: socket.socket):
        try:
            while not self._closing:
                hdr = _read_exact(conn, _REQ.size)
                if hdr is None:
                    return
                op, klen, vlen = _REQ.unpack(hdr)
                body = _read_exact(conn, klen + vlen) if klen + vlen else b""
                if body is None:
                    return
                out = self._apply(op, body[:klen].decode(), body[klen:])
                if out is None:
                    return
                conn.sendall(_LEN.pack(len(out)) + out)
        except OSError:
            return
        finally:
            try:
                conn.close()
            except OSError:
                pass

    def close(self):
        self._closing = True
        with self._cv:
            self._cv.notify_all()
        try:
            self._listener.close()
        except OSError:
            pass
        for c in self._clients:
            try:
                c.close()
            except OSError:
                pass


class Store:
    """Client of a ``StoreServer`` (or of the reference's store server)."""

    def __init__(self, address: str, timeout: float = 60.0):
        host, port = address.rsplit(":", 1)
        self.address = address
        self.timeout = timeout
        end = time.monotonic() + timeout
        while True:
            try:
                self._sock = socket.create_connection((host, int(port)), timeout=timeout)
                break
            except OSError:
                if time.monotonic() > end:
                    raise CommError(f"cannot reach store at {address}")
                time.sleep(0.05)
        self._sock.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
        self._lock = threading.Lock()

    def _call(self, op: int, key: str, val: bytes = b"") -> bytes:
        k = key.encode()
        with self._lock:
            try:
                self._sock.sendall(_REQ.pack(op, len(k), len(val)) + k + val)
            except OSError as e:
                raise CommError(f"store connection failed: {e}") from e
            hdr = _read_exact(self._sock, _LEN.size)
            if hdr is None:
                raise CommError("store connection closed")
            (n,) = _LEN.unpack(hdr)
            out = _read_exact(self._sock, n) if n else b""
            if out is None:
                raise CommError("store connection closed")
            return out

    def set(self, key: str, val: bytes) -> None:
        self._call(OP_SET, key, val)

    def get(self, key: str) -> bytes:
        return self._call(OP_GET, key)

    def add(self, key: str, n: int) -> int:
        return int(self._call(OP_ADD, key, str(int(n)).encode()))

    def check(self, key: str) -> bool:
        return self._call(OP_CHECK, key) == b"1"

    def delete(self, key: str) -> None:
        self._call(OP_DELETE, key)

    def close(self) -> None:
        try:
            self._sock.close()
        except OSError:
            pass
