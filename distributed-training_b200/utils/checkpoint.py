"""Sharded, atomic, SHA-256-checked checkpoints (on-disk layout of dtrain/checkpoint.py).

Layout under ``root``::

    step_000100/rank0.npz ... rank{W-1}.npz   one uncompressed .npz per rank
    step_000100/manifest.json                {"step", "world", "shards": {"rank{r}.npz": sha256}}
    LATEST                                   name of the newest complete step directory

Protocol: every rank writes its shard to ``rank{r}.npz.tmp``, fsyncs and renames;
barrier; rank 0 hashes every shard, writes the manifest (tmp + fsync + rename +
directory fsync) and then atomically replaces ``LATEST``; barrier.  A crash at
any point leaves ``LATEST`` on the previous complete checkpoint.  ``load``
checks the world size and the shard's checksum.  Files written here load with
the reference's ``dtrain.checkpoint.load`` and vice versa.

Device tensors in ``state`` are copied to host first (fp32 masters, never bf16:
``.npz`` has no bf16 and the working copy is re-derived from the masters).
"""
from __future__ import annotations

import hashlib
import io
import json
import os

import numpy as np

_CHUNK = 1 << 20


def sha256_file(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while True:
            b = f.read(_CHUNK)
            if not b:
                break
            h.update(b)
    return h.hexdigest()


def _sync_dir(path: str):
    fd = os.open(path, os.O_RDONLY)
    try:
        os.fsync(fd)
    finally:
        os.close(fd)


def _write_atomic(path: str, data: bytes):
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(data)
        f.flush()
        os.fsync(f.fileno())
    os.replace(tmp, path)


def _to_numpy(v):
    try:
        import torch
        if isinstance(v, torch.Tensor):
            v = v.detach()
            if v.dtype == torch.bfloat16:
                v = v.float()
            return v.cpu().numpy()
    except ImportError:  # pragma: no cover
        pass
    return np.asarray(v)


def _write_shard(root: str, step: int, rank: int, host_state: dict) -> str:
    d = os.path.join(root, f"step_{step:06d}")
    os.makedirs(d, exist_ok=True)
    payload = io.BytesIO()
    np.savez(payload, **host_state)
    _write_atomic(os.path.join(d, f"rank{rank}.npz"), payload.getvalue())
    return d


def _commit(root: str, step: int, rank: int, world: int, barrier) -> str:
    """Every rank's shard is on disk once all ranks reach the first barrier; rank 0 then
    hashes the shards into the manifest and moves LATEST (dtrain/checkpoint.py:52-68)."""
    name = f"step_{step:06d}"
    d = os.path.join(root, name)
    barrier()
    if rank == 0:
        manifest = {"step": step, "world": world,
                    "shards": {f"rank{r}.npz": sha256_file(os.path.join(d, f"rank{r}.npz")) for r in range(world)}}
        _write_atomic(os.path.join(d, "manifest.json"), json.dumps(manifest).encode())
        _sync_dir(d)
        _write_atomic(os.path.join(root, "LATEST"), name.encode())
        _sync_dir(root)
    barrier()
    return d


def save(root: str, step: int, rank: int, world: int, state: dict, barrier) -> str:
    _write_shard(root, step, rank, {k: _to_numpy(v) for k, v in state.items()})
    return _commit(root, step, rank, world, barrier)


class AsyncSaver:
    """Checkpoints whose shard files are written by a background thread.

    ``start`` copies the state to host memory on the calling thread (the training
    state may change right after) and writes ``rank{r}.npz`` in the background while
    training continues.  ``commit`` - called by the training thread at the next
    checkpoint and at the end of the run, in the same order on every rank - waits for
    the file and runs the same barrier / manifest / LATEST protocol as ``save``, so
    the collectives stay on the training thread.  A checkpoint is visible to
    ``latest``/``load`` only once committed: a crash before the commit resumes from
    the previous one.
    """

    def __init__(self):
        self._thread = None
        self._pending = None
        self._error: BaseException | None = None

    def start(self, root: str, step: int, rank: int, world: int, state: dict):
        import threading
        if self._pending is not None:
            raise RuntimeError("commit the previous checkpoint first")
        host = {k: _to_numpy(v) for k, v in state.items()}
        self._error = None

        def work():
            try:
                _write_shard(root, step, rank, host)
            except BaseException as e:  # noqa: BLE001 - re-raised by commit()
                self._error = e

        self._pending = (root, step, rank, world)
        self._thread = threading.Thread(target=work, name="dtb-ckpt-writer", daemon=True)
        self._thread.start()

    def commit(self, barrier) -> str | None:
        if self._pending is None:
            return None
        self._thread.join()
        root, step, rank, world = self._pending
        self._pending = self._thread = None
        if self._error is not None:
            raise self._error
        return _commit(root, step, rank, world, barrier)


def latest(root: str) -> str | None:
    p = os.path.join(root, "LATEST")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        return os.path.join(root, f.read().strip())


def load(d: str, rank: int, world: int) -> tuple[int, dict]:
    with open(os.path.join(d, "manifest.json")) as f:
        manifest = json.load(f)
    if manifest["world"] != world:
        raise ValueError(f"checkpoint was written by {manifest['world']} ranks, this job has {world}")
    shard = os.path.join(d, f"rank{rank}.npz")
    if sha256_file(shard) != manifest["shards"][f"rank{rank}.npz"]:
        raise ValueError(f"checksum mismatch in {shard}")
    with np.load(shard) as z:
        return manifest["step"], {k: z[k] for k in z.files}
