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


def save(root: str, step: int, rank: int, world: int, state: dict, barrier) -> str:
    name = f"step_{step:06d}"
    d = os.path.join(root, name)
    os.makedirs(d, exist_ok=True)
    payload = io.BytesIO()
    np.savez(payload, **{k: _to_numpy(v) for k, v in state.items()})
    _write_atomic(os.path.join(d, f"rank{rank}.npz"), payload.getvalue())
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
