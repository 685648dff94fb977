"""Training data: character-level text and iid synthetic tokens, batched deterministically.

The global batch of (step, micro-step) is a pure function of the seed
(dtrain/data.py:45-56): every rank takes its slice without communication, a
resumed run sees exactly the batches it would have seen, and one process can
reproduce the global batch of a W-rank job.  The random draws are the
reference's (``default_rng([seed, step, micro])``, start offsets via
``integers``), so batches are identical to the reference's for the same corpus.

``SyntheticData`` draws tokens iid uniform over the vocabulary from the same kind
of stateless generator, for benchmark configs that name a vocabulary but no corpus.
"""
from __future__ import annotations

import hashlib
import os
import tempfile
import urllib.request
from pathlib import Path

import numpy as np

TINY_SHAKESPEARE = "https://raw.githubusercontent.com/karpathy/char-rnn/master/data/tinyshakespeare/input.txt"
TINY_SHAKESPEARE_SHA256 = "86c4e6aa9db7c042ec79f339dcb96d42b0075e16b8fc2e86bf0ca57e2dc565ed"


def _fetch_verified(url: str, dest: str, sha256: str) -> None:
    """Download ``url`` to ``dest`` through a private temporary file in the same folder.

    The digest is computed while the bytes stream in; only a file whose digest
    matches is renamed into place (an atomic rename), so ranks that fetch the
    corpus at the same time never read a partial or unverified file.
    """
    folder = os.path.dirname(dest) or "."
    os.makedirs(folder, exist_ok=True)
    fd, tmp = tempfile.mkstemp(prefix=".fetch-", dir=folder)
    digest = hashlib.sha256()
    try:
        with os.fdopen(fd, "wb") as out, urllib.request.urlopen(url) as src:
            for block in iter(lambda: src.read(1 << 16), b""):
                digest.update(block)
                out.write(block)
        if digest.hexdigest() != sha256:
            raise ValueError(f"tiny shakespeare checksum mismatch: {digest.hexdigest()}")
        os.replace(tmp, dest)
    finally:
        if os.path.exists(tmp):
            os.remove(tmp)


def load_text(path: str | None = None, cache_dir: str = "data") -> str:
    """Text of ``path``; without one, tiny-shakespeare cached under ``cache_dir``
    (fetched and checksummed on first use)."""
    if not path:
        path = os.path.join(cache_dir, "tinyshakespeare.txt")
        if not os.path.isfile(path):
            _fetch_verified(TINY_SHAKESPEARE, path, TINY_SHAKESPEARE_SHA256)
    return Path(path).read_text(encoding="utf-8")


class CharData:
    """Character vocabulary (sorted) and a 90/10 train/validation split of the ids."""

    def __init__(self, text: str, val_fraction: float = 0.1):
        chars = sorted(set(text))
        self.vocab = len(chars)
        self.stoi = {c: i for i, c in enumerate(chars)}
        ids = np.fromiter((self.stoi[c] for c in text), dtype=np.int32, count=len(text))
        cut = int(len(ids) * (1 - val_fraction))
        self.train, self.val = ids[:cut], ids[cut:]


def global_batch(ids: np.ndarray, step: int, micro: int, global_bs: int, ctx: int, seed: int):
    rng = np.random.default_rng([seed, step, micro])
    starts = rng.integers(0, len(ids) - ctx - 1, size=global_bs)
    offs = np.arange(ctx)
    x = ids[starts[:, None] + offs[None, :]]
    y = ids[starts[:, None] + 1 + offs[None, :]]
    return x, y


def rank_batch(ids, step, micro, bs_per_rank, ctx, seed, rank, world):
    x, y = global_batch(ids, step, micro, bs_per_rank * world, ctx, seed)
    lo = rank * bs_per_rank
    return x[lo:lo + bs_per_rank], y[lo:lo + bs_per_rank]


class SyntheticData:
    """iid uniform tokens over ``vocab``; batches depend only on (seed, step, micro)."""

    def __init__(self, vocab: int):
        self.vocab = int(vocab)
        self.train = None

    def global_batch(self, step, micro, global_bs, ctx, seed):
        rng = np.random.default_rng([seed, step, micro, 0x53594E])
        toks = rng.integers(0, self.vocab, size=(global_bs, ctx + 1), dtype=np.int64)
        return toks[:, :-1], toks[:, 1:]

    def rank_batch(self, step, micro, bs_per_rank, ctx, seed, rank, world):
        x, y = self.global_batch(step, micro, bs_per_rank * world, ctx, seed)
        lo = rank * bs_per_rank
        return x[lo:lo + bs_per_rank], y[lo:lo + bs_per_rank]


def lr_at(step: int, a) -> float:
    """Linear warm-up to ``a.lr`` over ``a.warmup`` steps, then cosine to lr/10 (dtrain/train.py:63-69)."""
    if a.warmup and step < a.warmup:
        return a.lr * (step + 1) / a.warmup
    if not a.warmup:
        return a.lr
    t = (step - a.warmup) / max(1, a.steps - a.warmup)
    return a.lr * (0.1 + 0.9 * 0.5 * (1 + np.cos(np.pi * min(1.0, t))))
