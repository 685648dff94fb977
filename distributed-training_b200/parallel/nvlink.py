"""GPU process group: collectives as sm_100a kernels over NVLink / NVSwitch peer memory.

Same API as the host ``ProcessGroup`` (dtrain/comm.py:241-432): ``allreduce``,
``reduce_scatter``, ``all_gather``, ``broadcast``, ``barrier``,
``allreduce_async`` -> work handle, ``close``, ``rank``, ``world``, ``seq``.

Memory model.  ``alloc(numel, dtype)`` is a collective: every rank allocates a
buffer of the same size (cudaMalloc), exports an IPC handle, publishes it through
the bootstrap ``exchange`` function and opens its peers' handles.  With
``memory="vmm"`` (or ``DTB_PEER_MEMORY=vmm``) the buffer is a CUDA VMM allocation
instead, exported as a file descriptor and passed to the peers over Unix sockets
(``FdExchange``); each peer's import holds its own reference to the physical
memory, so a rank that dies does not unmap memory that the others still read.  Collectives on
tensors that live inside such a buffer run in place, reading and writing peer
memory directly from the kernel (``csrc/comm.cu``); other CUDA tensors are staged
through a symmetric scratch buffer.  DDP and ZeRO allocate their flat gradient,
master and working-copy buffers here, so their collectives never copy.

Ordering and failure.  Collectives are stream-ordered on the caller's current
stream (``allreduce_async`` uses a dedicated comm stream and returns a handle
whose ``wait()`` makes the current stream wait on it, like NCCL).  Every rank
must issue the same collectives in the same order, and one group's collectives
never run concurrently with each other; each kernel synchronises with its peers
through per-CTA epoch flags, and every wait gives up after ``timeout`` seconds,
writing an error code to a host-mapped status word.  ``check()`` turns a non-zero
status into ``CommError``.

Graph capture.  The flag epochs come from a counter on the device that each
collective advances itself, so a collective's launch is the same every time:
collectives can be captured in a CUDA graph (DDP captures its per-bucket
all-reduces inside the backward it replays) and mixed freely with eager calls.
"""
from __future__ import annotations

import os
import socket
import struct
import uuid

import torch

from ..ops._ext import lib
from ..utils.store import CommError
from .comm import partition

DT = {torch.float32: 0, torch.bfloat16: 1}
ORDER_RANK, ORDER_CYCLIC = 0, 1
ALGO_ONESHOT, ALGO_TWOSHOT = 0, 1
# [max CTAs][max ranks] uint32 flags, then a ring of 16 uint64 collective descriptors
_SIG_BYTES = 8192
# One-shot moves (W-1) x the data into every rank but needs one cross-rank barrier
# fewer than two-shot; its result is written out of place and copied back.
# DTB_ONESHOT_MAX_BYTES overrides the size up to which "auto" picks it.
_ONESHOT_ENV = os.environ.get("DTB_ONESHOT_MAX_BYTES")


def auto_allreduce_plan(world: int, nbytes: int) -> tuple[str, int]:
    """(method, CTA count; 0 = sized by the message) that ``method="auto"`` uses for an
    all-reduce of ``nbytes`` over ``world`` ranks, from the CUDA-graph sweeps on B200
    (benchmarks/collectives_bench.py at W = 2 and 4, fp32 and bf16):

    * W = 2: one-shot moves the same bytes as two-shot and skips a barrier, so it wins
      up to 16 MiB; above that two-shot with 128 CTAs (585 vs 510 GB/s for NCCL at 256 MiB).
    * W = 3..4: one-shot up to 512 KiB, one-shot with 128 CTAs up to 4 MiB, two-shot
      at 8 MiB, two-shot with 128 CTAs from 16 MiB.
    * W > 4 (not measured): one-shot up to 256 KiB - its traffic grows with W - and
      two-shot above, with 128 CTAs from 16 MiB.
    Only the fixed-order methods are chosen (NVLS is opt-in).
    """
    mib = 1 << 20
    if _ONESHOT_ENV is not None:
        return ("oneshot", 0) if nbytes <= int(_ONESHOT_ENV) else ("twoshot", 128 if nbytes >= 16 * mib else 0)
    if world <= 2:
        return ("oneshot", 0) if nbytes <= 16 * mib else ("twoshot", 128)
    if world <= 4:
        if nbytes <= 512 * 1024:
            return "oneshot", 0
        if nbytes <= 4 * mib:
            return "oneshot", 128
        return ("twoshot", 0) if nbytes < 16 * mib else ("twoshot", 128)
    if nbytes <= 256 * 1024:
        return "oneshot", 0
    return ("twoshot", 0) if nbytes < 16 * mib else ("twoshot", 128)


class FdExchange:
    """All-gather of file descriptors between the ranks of one node (no counterpart in
    the reference, whose peers share nothing but TCP connections, dtrain/comm.py:132-217).

    Each rank listens on an abstract Unix socket whose name goes through the bootstrap
    ``exchange`` once.  ``all_gather(fd, size)`` connects to every peer and sends
    ``(rank, tag, size)`` with the descriptor attached (SCM_RIGHTS), then accepts one
    connection per peer.  Calls are collective and numbered; a message that belongs to
    a later call (a fast peer already on the next allocation) is kept until then.
    """

    def __init__(self, rank: int, world: int, exchange, timeout: float = 60.0):
        self.rank, self.world, self.timeout = int(rank), int(world), float(timeout)
        self.name = f"\0dtb-fd-{uuid.uuid4().hex}-{self.rank}"
        self.sock = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
        self.sock.bind(self.name)
        self.sock.listen(max(16, 2 * self.world))
        self.sock.settimeout(self.timeout)
        self.names = [n.decode() for n in exchange("fdx/sock", self.name.encode())]
        self.calls = 0
        self.pending: dict[tuple[int, int], tuple[int, int]] = {}

    def _send(self, p: int, tag: int, fd: int, size: int):
        hdr = struct.pack("<iiq", self.rank, tag, int(size))
        with socket.socket(socket.AF_UNIX, socket.SOCK_STREAM) as c:
            c.settimeout(self.timeout)
            c.connect(self.names[p])
            socket.send_fds(c, [hdr], [int(fd)])

    def _collect(self, tag: int, need: set[int]) -> dict[int, tuple[int, int]]:
        got: dict[int, tuple[int, int]] = {}
        for p in list(need):
            if (tag, p) in self.pending:
                got[p] = self.pending.pop((tag, p))
                need.discard(p)
        while need:
            try:
                conn, _ = self.sock.accept()
            except socket.timeout as e:
                raise CommError(f"descriptor exchange: no message from ranks {sorted(need)}") from e
            with conn:
                conn.settimeout(self.timeout)
                msg, fds, _, _ = socket.recv_fds(conn, struct.calcsize("<iiq"), 1)
            if len(msg) != struct.calcsize("<iiq") or len(fds) != 1:
                raise CommError("descriptor exchange: malformed message")
            r, t, sz = struct.unpack("<iiq", msg)
            if t == tag and r in need:
                got[r] = (fds[0], sz)
                need.discard(r)
            elif t > tag:
                self.pending[(t, r)] = (fds[0], sz)
            else:
                os.close(fds[0])
                raise CommError(f"descriptor exchange: rank {r} sent call {t} during call {tag}")
        return got

    def all_gather(self, fd: int, size: int) -> list[tuple[int, int] | None]:
        """Returns, per rank, (received descriptor, size) - None at this rank's index.
        The caller owns the received descriptors."""
        tag = self.calls
        self.calls += 1
        for p in range(self.world):
            if p != self.rank:
                self._send(p, tag, fd, size)
        got = self._collect(tag, {p for p in range(self.world) if p != self.rank})
        return [got.get(p) for p in range(self.world)]

    def broadcast(self, fd: int | None, size: int, root: int = 0) -> tuple[int, int] | None:
        """``root`` sends its descriptor to every other rank; the others return
        (received descriptor, size), which they own; the root returns None."""
        tag = self.calls
        self.calls += 1
        if self.rank == root:
            for p in range(self.world):
                if p != root:
                    self._send(p, tag, fd, size)
            return None
        return self._collect(tag, {root})[root]

    def close(self):
        self.sock.close()
        for fd, _ in self.pending.values():
            os.close(fd)
        self.pending.clear()


class SymmetricBuffer:
    """One peer-mapped allocation: a local tensor view plus every rank's base pointer."""

    def __init__(self, group: "NVLinkGroup", nbytes: int, multicast: bool = False):
        C = lib()
        self.nbytes = int(nbytes)
        self.vmm = group.memory == "vmm"
        self.ptrs = []
        self._opened = []
        self.mc_ptr = 0  # NVSwitch multicast address of this buffer (0: none)
        if multicast and not self.vmm:
            raise ValueError("a multicast-mapped buffer needs memory='vmm'")
        if self.vmm:
            want = max(self.nbytes, 256)
            if multicast:  # the whole allocation is bound to the multicast object
                g = group._mc_gran
                want = (want + g - 1) // g * g
            ptr, fd, size = C.vmm_alloc(want)
            self.ptr = int(ptr)
            try:
                got = group._fdx.all_gather(fd, size)
            finally:
                os.close(fd)
            group._nalloc += 1
            for r, g in enumerate(got):
                if r == group.rank:
                    self.ptrs.append(self.ptr)
                    continue
                pfd, psize = g
                try:
                    if psize != size:
                        raise CommError(f"vmm: rank {r} mapped {psize} bytes, this rank {size}")
                    p = int(C.vmm_import(pfd, psize))
                finally:
                    os.close(pfd)
                self.ptrs.append(p)
                self._opened.append(p)
            if multicast:
                self.mc_ptr = self._map_multicast(group, int(size))
        else:
            ptr, handle = C.symm_alloc(max(self.nbytes, 256))
            self.ptr = int(ptr)
            handles = group._exchange(f"symm/{group._nalloc}", bytes(handle.numpy().tobytes()))
            group._nalloc += 1
            for r, h in enumerate(handles):
                if r == group.rank:
                    self.ptrs.append(self.ptr)
                else:
                    p = int(C.symm_open(torch.frombuffer(bytearray(h), dtype=torch.uint8)))
                    self.ptrs.append(p)
                    self._opened.append(p)
        self.device = group.device

    def _map_multicast(self, group: "NVLinkGroup", size: int) -> int:
        """Rank 0 creates an NVSwitch multicast object of ``size`` bytes and passes it
        to the others by file descriptor; every rank joins it, the ranks confirm over
        the host that all of them joined (the driver would block a bind forever on a
        rank that could not), then each binds this buffer's allocation and maps the
        object.  Returns the multicast address."""
        C = lib()
        if group.rank == 0:
            mc, fd = C.mc_create(size, group.world)
            try:
                group._fdx.broadcast(fd, size, root=0)
            finally:
                os.close(fd)
        else:
            fd, psize = group._fdx.broadcast(None, 0, root=0)
            try:
                if psize != size:
                    raise CommError(f"multicast: rank 0 made {psize} bytes, this rank needs {size}")
                mc = C.mc_import(fd)
            finally:
                os.close(fd)
        err = ""
        try:
            C.mc_add_device(mc)
        except RuntimeError as e:
            err = str(e).splitlines()[0]
        group._mc_joins += 1
        votes = group._exchange(f"mc-join/{group._mc_joins}", err.encode())
        if any(votes):
            C.mc_release(mc)
            bad = {r: v.decode() for r, v in enumerate(votes) if v}
            raise CommError(f"multicast: ranks could not join the NVSwitch multicast object: {bad}")
        return int(C.mc_bind_map(mc, self.ptr, size, group.world))

    def tensor(self, numel: int, dtype: torch.dtype, byte_offset: int = 0) -> torch.Tensor:
        assert byte_offset + numel * torch.tensor([], dtype=dtype).element_size() <= self.nbytes
        return lib().tensor_from_ptr(self.ptr + byte_offset, [int(numel)], dtype, self.device.index)

    def contains(self, t: torch.Tensor) -> int | None:
        """Byte offset of ``t`` inside this buffer, or None."""
        p = t.data_ptr()
        end = p + t.numel() * t.element_size()
        if self.ptr <= p and end <= self.ptr + self.nbytes:
            return p - self.ptr
        return None

    def free(self):
        C = lib()
        if self.mc_ptr:
            C.mc_free(self.mc_ptr)
            self.mc_ptr = 0
        for p in self._opened:
            if self.vmm:
                C.vmm_free(p)
            else:
                C.symm_close(p)
        self._opened = []
        if self.ptr:
            if self.vmm:
                C.vmm_free(self.ptr)
            else:
                C.symm_free(self.ptr)
            self.ptr = 0


class GPUWork:
    """Handle of an asynchronous GPU collective (event on the comm stream)."""

    def __init__(self, event: torch.cuda.Event, group: "NVLinkGroup"):
        self.event, self.group = event, group

    def wait(self):
        """Make the current stream wait for the collective (no host synchronisation)."""
        torch.cuda.current_stream().wait_event(self.event)

    def synchronize(self):
        self.event.synchronize()
        self.group.check()

    def is_completed(self) -> bool:
        return self.event.query()


class NVLinkGroup:
    backend = "nvlink"

    def __init__(self, rank: int, world: int, device, exchange, timeout: float = 60.0, blocks: int = 0,
                 comm_priority: int = 0, memory: str | None = None, nvls: bool | None = None):
        """``exchange(key, payload: bytes) -> list[bytes]`` is the bootstrap all-gather
        (over the rendezvous store or torch.distributed); it is used only at set-up.
        ``blocks`` caps the CTAs of one collective kernel (0: sized by the message);
        ``comm_priority`` is the CUDA priority of the stream that runs the asynchronous
        collectives (lower is more urgent: -1 lets their CTAs take SMs ahead of queued
        compute work); ``memory`` is "ipc" (cudaMalloc + IPC handles, the default) or
        "vmm" (CUDA VMM allocations shared by file descriptor); the environment
        variable DTB_PEER_MEMORY sets the default.  ``nvls`` (default: the
        environment variable DTB_NVLS=1) also maps every buffer from ``alloc`` through
        an NVSwitch multicast object, which enables ``method="nvls"`` (switch-side
        reduction with multimem instructions); it implies ``memory="vmm"``."""
        if world > int(lib().comm_max_ranks()):
            raise ValueError(f"NVLinkGroup supports up to {lib().comm_max_ranks()} ranks per node")
        self.rank, self.world = int(rank), int(world)
        self.device = torch.device(device)
        self.blocks = int(blocks)
        self._exchange_fn = exchange
        self._nalloc = 0
        self.nvls = bool(int(os.environ.get("DTB_NVLS", "0"))) if nvls is None else bool(nvls)
        self.nvls = self.nvls and self.world > 1
        self.memory = (memory or os.environ.get("DTB_PEER_MEMORY", "vmm" if self.nvls else "ipc")).lower()
        if self.memory not in ("ipc", "vmm"):
            raise ValueError(f"unknown peer memory kind {self.memory!r} (ipc or vmm)")
        if self.nvls and self.memory != "vmm":
            raise ValueError("NVLS collectives need memory='vmm' (multicast objects bind VMM allocations)")
        self._mc_gran = 0
        self._mc_joins = 0
        if self.nvls:
            with torch.cuda.device(self.device):
                if not lib().mc_supported():
                    raise CommError("NVLS requested but this GPU does not support NVSwitch multicast")
                self._mc_gran = int(lib().mc_granularity(self.world))
        self._closes = 0
        self._fdx = FdExchange(self.rank, self.world, exchange, timeout) if self.memory == "vmm" else None
        self.seq = 0            # collectives issued
        self.buffers: list[SymmetricBuffer] = []
        self._eng = None
        with torch.cuda.device(self.device):
            lib().comm_status_clear()
            lib().comm_abort_prepare()
            self._sig = self._new_buffer(_SIG_BYTES)
            # native state: signal pads, registered buffers, flag epoch, timeout
            self._eng = lib().CommEngine(self.rank, self.world, self._sig.ptrs, float(timeout), self.blocks)
            self.comm_stream = torch.cuda.Stream(device=self.device, priority=int(comm_priority))
        self._staging: SymmetricBuffer | None = None
        self._sq_parts = None
        self.barrier()
        self.synchronize()

    # ------------------------------------------------------------ plumbing
    @property
    def epoch(self) -> int:
        """Last flag epoch this rank's collectives used (read from the device counter,
        synchronously; it advances identically on every rank)."""
        return int(self._eng.device_epoch())

    @property
    def timeout(self) -> float:
        return float(self._eng.timeout)

    @timeout.setter
    def timeout(self, t: float):
        self._eng.timeout = float(t)

    def _exchange(self, key: str, payload: bytes) -> list[bytes]:
        return self._exchange_fn(key, payload)

    def _new_buffer(self, nbytes: int, multicast: bool = False) -> SymmetricBuffer:
        b = SymmetricBuffer(self, nbytes, multicast=multicast)
        self.buffers.append(b)
        if self._eng is not None:
            self._eng.register_buffer(b.ptrs, b.nbytes, b.mc_ptr)
        return b

    def alloc(self, numel: int, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """Collective: a zero-filled peer-mapped tensor (same size on every rank);
        multicast-mapped too when the group was made with ``nvls``."""
        esz = torch.tensor([], dtype=dtype).element_size()
        with torch.cuda.device(self.device):
            buf = self._new_buffer(int(numel) * esz, multicast=self.nvls)
        return buf.tensor(numel, dtype)

    def _locate(self, t: torch.Tensor):
        for b in self.buffers:
            off = b.contains(t)
            if off is not None:
                return b, off
        return None, None

    @property
    def _sigs(self):
        return self._sig.ptrs

    def _issued(self):
        self._eng.note_issued()
        self.seq += 1

    def _stage(self, nbytes: int) -> SymmetricBuffer:
        if self._staging is None or self._staging.nbytes < nbytes:
            # growth is collective: every rank stages the same sizes in the same order
            self.synchronize()
            self._staging = self._new_buffer(max(nbytes, 1 << 20), multicast=self.nvls)
        return self._staging

    def check(self):
        """Raise CommError if a collective kernel timed out waiting for a peer, or found
        that the ranks had issued different collectives (desynchronised ranks)."""
        code = int(lib().comm_status())
        if code == 5:
            raise CommError(f"NVLink process group aborted on rank {self.rank} (abort() was called)")
        if code == 3:
            raise CommError(f"NVLink collective failed on rank {self.rank} (device status 3): collective desync - "
                            "the ranks issued different collectives (kind, size or dtype) at the same point")
        if code:
            raise CommError(f"NVLink collective failed on rank {self.rank} (device status {code}): "
                            "a peer did not arrive within the timeout")

    def synchronize(self):
        torch.cuda.synchronize(self.device)
        self.check()

    def abort(self):
        """Make every collective of this rank that is waiting, or that is still to run,
        give up at once (its "failed" word is set through the copy engine); ``check()``
        then raises CommError.  Safe to call from another thread while this process is
        blocked on the GPU - the way a stopping worker ends a wait for a peer that is
        gone without waiting out the timeout.  The group is unusable afterwards."""
        with torch.cuda.device(self.device):
            lib().comm_abort(self._sig.ptr)

    # ---------------------------------------------------------- collectives
    def _order(self, algo: str) -> int:
        return ORDER_CYCLIC if algo == "ring" else ORDER_RANK

    def allreduce(self, t: torch.Tensor, algo: str = "ring", scale: float = 1.0, method: str = "auto",
                  blocks: int = 0, lean: bool = False, sq=None):
        """In-place sum (times ``scale``) over ranks.

        ``algo`` selects the summation order: "ring" (dtrain ring order) or
        "direct" (rank order).  ``method`` selects the data movement: "oneshot"
        (every rank reduces everything: latency-optimal), "twoshot" (reduce-scatter
        + all-gather: bandwidth-optimal), "nvls" (sums formed in the NVSwitch by
        multimem.ld_reduce and written to every rank by multimem.st: the least
        NVLink traffic from 4 ranks up; needs a group made with ``nvls``; every rank
        gets the same bits, but the order of the additions is the switch's, so
        ``algo`` does not apply) or "auto" (method and CTA count by size and world,
        ``auto_allreduce_plan``).  Two-shot on a peer-mapped tensor
        also takes ``blocks`` (CTA count, 0: by size), ``lean`` (128-thread CTAs
        that share SMs with running GEMMs) and ``sq = (pad, base, stride)``: CTA b
        writes the sum of squares of the scaled values it reduced into slot
        ``rank * stride + base + b`` of every rank's fp64 ``pad`` (peer-mapped).
        """
        if self.world == 1:
            if scale != 1.0:
                t.mul_(scale)
            return t
        if not t.is_contiguous():
            raise ValueError("allreduce needs a contiguous tensor")
        if t.dtype not in DT:
            raise TypeError("NVLink allreduce supports float32 and bfloat16")
        n = t.numel()
        nbytes = n * t.element_size()
        if method == "auto":
            if lean or sq is not None:
                method = "twoshot"
            else:
                method, plan_blocks = auto_allreduce_plan(self.world, nbytes)
                if not blocks and not self.blocks:
                    blocks = plan_blocks
        if method == "nvls":
            return self._allreduce_nvls(t, scale, blocks, sq, lean)
        if method == "twoshot" and self._eng.contains(t):
            # fast path: one native call, in place on the peer-mapped tensor
            pad, base, stride = sq if sq is not None else (None, 0, 0)
            self._eng.allreduce_inplace(t, self._order(algo), scale, int(blocks or self.blocks), bool(lean), pad,
                                        int(base), int(stride))
            self.seq += 1
            return t
        if lean or sq is not None:
            raise ValueError("lean / sum-of-squares all-reduce needs a peer-mapped tensor and method='twoshot'")
        buf, off = self._locate(t)
        staged = buf is None
        # one-shot writes out of place: it needs scratch for the result (and for the
        # input too when t is not peer-mapped); size the staging buffer once, up front
        need = nbytes * ((2 if staged else 1) if method == "oneshot" else (1 if staged else 0))
        stage = self._stage(need) if need else None
        if staged:
            buf, off = stage, 0
            buf.tensor(n, t.dtype).copy_(t.reshape(-1))
        C = lib()
        if method == "oneshot":
            if stage is buf and not staged:
                raise RuntimeError("one-shot scratch aliases the input")
            out = stage.tensor(n, t.dtype, nbytes if staged else 0)
            C.allreduce(self._sigs, self.rank, buf.ptrs, off, n, DT[t.dtype], out.data_ptr(), DT[t.dtype],
                        ALGO_ONESHOT, self._order(algo), scale, self.timeout, int(blocks or self.blocks), False, [], 0,
                        0)
            t.reshape(-1).copy_(out)
        else:
            C.allreduce(self._sigs, self.rank, buf.ptrs, off, n, DT[t.dtype], 0, DT[t.dtype], ALGO_TWOSHOT,
                        self._order(algo), scale, self.timeout, int(blocks or self.blocks), False, [], 0, 0)
            if staged:
                t.reshape(-1).copy_(buf.tensor(n, t.dtype))
        self._issued()
        return t

    def _allreduce_nvls(self, t: torch.Tensor, scale: float, blocks: int, sq, lean: bool = False):
        if not self.nvls:
            raise ValueError("method='nvls' needs a group made with nvls=True (DTB_NVLS=1)")
        n, esz = t.numel(), t.element_size()
        # fp32: any 4-byte aligned start; bf16: whole 16-byte vectors only
        ok = t.dtype == torch.float32 or (t.data_ptr() % 16 == 0 and n % 8 == 0)
        if self._eng.has_multicast(t) and ok:
            pad, base, stride = sq if sq is not None else (None, 0, 0)
            self._eng.allreduce_nvls(t, scale, int(blocks or self.blocks), bool(lean), pad, int(base), int(stride))
            self.seq += 1
            return t
        if sq is not None or lean:
            raise ValueError("a lean or sum-of-squares NVLS all-reduce needs a tensor from alloc()")
        if not ok:  # bf16 that does not form whole 16-byte vectors
            return self.allreduce(t, scale=scale, method="twoshot", blocks=blocks)
        stage = self._stage(n * esz)
        buf = stage.tensor(n, t.dtype)
        buf.copy_(t.reshape(-1))
        self._eng.allreduce_nvls(buf, scale, int(blocks or self.blocks), False, None, 0, 0)
        self.seq += 1
        t.reshape(-1).copy_(buf)
        return t

    def collective_blocks(self, nbytes: int, lean: bool = False) -> int:
        """CTAs an all-reduce of ``nbytes`` launches (``blocks=0``, this group's cap applied)."""
        return int(lib().collective_blocks(int(nbytes), int(self.blocks), bool(lean)))

    def sq_total(self, pad: torch.Tensor, out: torch.Tensor, stride: int, lo: int, hi: int) -> torch.Tensor:
        """``out[0]`` = sum of ``pad[r * stride + s]`` over ranks r and slots lo <= s < hi,
        in a fixed order (the same bits on every rank)."""
        lib().sq_total(pad, out, self.world, int(stride), int(lo), int(hi))
        return out

    def reduce_scatter(self, flat: torch.Tensor, scale: float = 1.0, sq_parts: torch.Tensor | None = None,
                       method: str = "ring"):
        """Sum over ranks; this rank's partition then holds the total.  Returns a view
        of it.  ``method``: "ring" (dtrain's ring order, bit-equal to it) or "nvls"
        (fp32 sums formed in the NVSwitch; a group made with ``nvls``).  With
        ``sq_parts`` (fp64, symmetric) the kernel also writes per-CTA sums of squares
        of the reduced partition."""
        n = flat.numel()
        b = partition(n, self.world)
        if self.world > 1:
            if not self._eng.contains(flat):
                raise ValueError("reduce_scatter needs a tensor allocated with NVLinkGroup.alloc")
            sqp = sq_parts.data_ptr() if sq_parts is not None else 0
            self.seq += 1
            if method == "nvls":
                if not (self.nvls and self._eng.has_multicast(flat)):
                    raise ValueError("method='nvls' needs a tensor from alloc() of a group made with nvls=True")
                return self._eng.reduce_scatter_nvls(flat, scale, sqp, self._rs_blocks())
            if method != "ring":
                raise ValueError(f"unknown reduce-scatter method {method!r} (ring or nvls)")
            return self._eng.reduce_scatter(flat, ORDER_CYCLIC, scale, sqp, self._rs_blocks())
        elif scale != 1.0:
            flat.mul_(scale)
        return flat[b[self.rank]:b[self.rank + 1]]

    def _rs_blocks(self) -> int:
        # a fixed CTA count (the ZeRO update reads exactly this many squared-norm
        # partials per rank); 64 CTAs keep enough peer loads in flight for NVLink
        return self.blocks or 64

    def all_gather(self, flat: torch.Tensor):
        if self.world > 1:
            if not self._eng.contains(flat):
                raise ValueError("all_gather needs a tensor allocated with NVLinkGroup.alloc")
            self._eng.all_gather(flat)
            self.seq += 1
        return flat

    def broadcast(self, t: torch.Tensor, root: int = 0, cast_to: torch.Tensor | None = None):
        """Copy root's ``t`` to every rank (optionally also casting fp32 -> bf16 into ``cast_to``)."""
        if self.world == 1:
            if cast_to is not None:
                cast_to.copy_(t)
            return t
        buf, off = self._locate(t)
        staged = buf is None
        nbytes = t.numel() * t.element_size()
        if staged:
            buf, off = self._stage(nbytes), 0
            if self.rank == root:
                buf.tensor(nbytes, torch.uint8).copy_(t.reshape(-1).view(torch.uint8))
        if cast_to is not None and t.dtype != torch.float32:
            raise TypeError("broadcast cast_to needs a float32 source")
        c16 = cast_to.data_ptr() if cast_to is not None else 0
        src = buf.ptr + off  # every rank's copy of the payload after the first phase
        lib().broadcast(self._sigs, self.rank, buf.ptrs, off, nbytes, root, src if cast_to is not None else 0, c16,
                        t.numel() if cast_to is not None else 0, self.timeout, self.blocks)
        self._issued()
        if staged and self.rank != root:
            t.reshape(-1).view(torch.uint8).copy_(buf.tensor(nbytes, torch.uint8))
        return t

    def barrier(self):
        self._eng.barrier()
        self.seq += 1

    def allreduce_async(self, t: torch.Tensor, algo: str = "ring", scale: float = 1.0,
                        method: str = "auto", **kw) -> GPUWork:
        """Launch on the comm stream after the work already queued on the current stream
        (also inside a CUDA-graph capture: the comm stream forks from the capturing
        stream and ``wait()`` joins it back).  ``kw``: ``blocks``, ``lean``, ``sq`` as
        for ``allreduce``; ``stamps = (buf, before, after)`` writes device timestamps
        into the int64 ``buf`` around the kernel, on the comm stream."""
        stamps = kw.pop("stamps", None)
        cur = torch.cuda.current_stream(self.device)
        self.comm_stream.wait_stream(cur)
        with torch.cuda.stream(self.comm_stream):
            if stamps is not None:
                lib().stamp(stamps[0], stamps[1])
            self.allreduce(t, algo, scale, method, **kw)
            if stamps is not None:
                lib().stamp(stamps[0], stamps[2])
            ev = torch.cuda.Event()
            ev.record(self.comm_stream)
        if not self._eng.contains(t):
            # allocator-owned memory: keep it alive until the comm stream is done
            t.record_stream(self.comm_stream)
        return GPUWork(ev, self)

    def close(self):
        try:
            torch.cuda.synchronize(self.device)
        except Exception:  # noqa: BLE001 - closing after a failure must not raise
            pass
        if any(b.mc_ptr for b in self.buffers):
            # no rank unbinds its memory from a multicast object while another rank's
            # multimem instructions may still reach it
            self._closes += 1
            self._exchange(f"nvls-close/{self._closes}", b"")
        for b in self.buffers:
            b.free()
        self.buffers = []
        if self._eng is not None:
            self._eng.forget_buffers()
        if self._fdx is not None:
            self._fdx.close()
            self._fdx = None


def store_exchange(store, rank: int, world: int, prefix: str = ""):
    """Bootstrap all-gather over the rendezvous store."""

    def ex(key: str, payload: bytes) -> list[bytes]:
        store.set(f"{prefix}nvl/{key}/{rank}", payload)
        return [store.get(f"{prefix}nvl/{key}/{r}") for r in range(world)]

    return ex


def torch_exchange():
    """Bootstrap all-gather over an initialised torch.distributed group."""
    import torch.distributed as dist

    def ex(key: str, payload: bytes) -> list[bytes]:
        out = [None] * dist.get_world_size()
        dist.all_gather_object(out, payload)
        return out

    return ex


def from_env(device=None, timeout: float | None = None, nvls: bool | None = None) -> NVLinkGroup:
    """NVLinkGroup from RANK / WORLD_SIZE / STORE_ADDR (the launcher) or torchrun's env."""
    t = timeout if timeout is not None else float(os.environ.get("DTRAIN_TIMEOUT", "60"))
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = torch.device(device) if device is not None else torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if "STORE_ADDR" in os.environ:
        from ..utils.store import Store
        store = Store(os.environ["STORE_ADDR"], t)
        return NVLinkGroup(rank, world, dev, store_exchange(store, rank, world, os.environ.get("DTRAIN_PREFIX", "")),
                           timeout=t, nvls=nvls)
    import torch.distributed as dist
    if not dist.is_initialized():
        raise RuntimeError("no STORE_ADDR and torch.distributed is not initialised")
    return NVLinkGroup(rank, world, dev, torch_exchange(), timeout=t, nvls=nvls)
