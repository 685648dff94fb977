"""Distributed data parallel with gradient buckets and comm/compute overlap.

API and semantics of dtrain/ddp.py:40-110: ``DDP(model, pg, bucket_mb=1.0,
overlap=True, algo="ring")``, ``no_sync()``, ``finish()``, ``comm_wait_s``.

* Parameters are broadcast from rank 0 at construction.
* Buckets are built in reverse parameter order and closed as soon as their size
  reaches ``bucket_mb`` MiB (so one large tensor forms its own bucket).
* A grad-ready hook (torch's post-accumulate-grad hook, which fires once per
  parameter per backward, after the final gradient is in ``p.grad``) counts the
  bucket down; a complete bucket is all-reduced asynchronously while backward
  continues (``overlap=True``), or all buckets are reduced in ``finish()``.
* ``no_sync()`` skips communication on gradient-accumulation micro-steps.
* ``finish()`` zero-fills gradients of parameters that received none, waits
  for all reductions and leaves the averaged gradient in ``p.grad``.

GPU path (``pg`` is an ``NVLinkGroup``): the model's parameters and gradients
are moved into flat peer-mapped buffers, so every bucket is a contiguous slice
of the flat gradient that the backward kernels already wrote.  The bucket
all-reduce is one kernel (``csrc/comm.cu``) on the comm stream that reads the
peers' slices over NVLink, sums them in the fixed order, multiplies by 1/W and
writes the result in place - the reference's copy-in, all-reduce, scale and
copy-out (dtrain/ddp.py:73-110) collapse into that kernel.  ``finish()`` only
makes the compute stream wait for the comm stream; no host synchronisation.

Host path (``pg`` is a TCP ``ProcessGroup``): the reference algorithm on host
buffers, used by CPU ranks and the float64 oracle tests.
"""
from __future__ import annotations

import contextlib
import time

import numpy as np
import torch


class _Bucket:
    def __init__(self, params, lo=None, hi=None):
        self.params = params
        self.pending = len(params)
        self.work = None
        self.lo, self.hi = lo, hi          # flat-gradient range (GPU path)
        self.buf = None                    # host buffer (TCP path)
        self.offsets = []


class DDP:
    def __init__(self, model, pg, bucket_mb: float = 1.0, overlap: bool = True, algo: str = "ring",
                 method: str = "auto"):
        self.model, self.pg, self.overlap, self.algo, self.method = model, pg, overlap, algo, method
        self.params = list(model.parameters())
        self.gpu = getattr(pg, "backend", "tcp") == "nvlink"
        self.comm_wait_s = 0.0
        self._sync = True
        if self.gpu:
            self._init_gpu()
        else:
            for p in self.params:
                pg.broadcast(p.data.numpy(), root=0)
        limit = int(bucket_mb * (1 << 20))
        self.buckets: list[_Bucket] = []
        cur, size = [], 0
        for p in reversed(self.params):
            cur.append(p)
            size += p.numel() * p.element_size()
            if size >= limit:
                self.buckets.append(self._make_bucket(cur))
                cur, size = [], 0
        if cur:
            self.buckets.append(self._make_bucket(cur))
        self._where = {}
        for bi, b in enumerate(self.buckets):
            for pi, p in enumerate(b.params):
                self._where[id(p)] = (bi, pi)
        self._hooks = [p.register_post_accumulate_grad_hook(self._on_grad) for p in self.params]

    # -------------------------------------------------------------- set-up
    def _init_gpu(self):
        pg = self.pg
        n = sum(p.numel() for p in self.params)
        grad = pg.alloc(n, torch.float32)
        master = pg.alloc(n, torch.float32)
        flat = self.model.flatten(pg.device, grad_buffer=grad, master_buffer=master)
        # rank 0's parameters everywhere, with the bf16 working copy re-derived
        pg.broadcast(flat.master, root=0, cast_to=flat.work)
        self.flat = flat

    def _make_bucket(self, params) -> _Bucket:
        if self.gpu:
            idx = [self.flat.index[id(p)] for p in params]
            lo = min(self.flat.offsets[i] for i in idx)
            hi = max(self.flat.offsets[i] + self.flat.numels[i] for i in idx)
            return _Bucket(params, lo, hi)
        b = _Bucket(params)
        off = 0
        for p in params:
            b.offsets.append(off)
            off += p.numel()
        b.buf = np.zeros(off, dtype=self.params[0].detach().numpy().dtype)
        return b

    # ------------------------------------------------------------ interface
    @contextlib.contextmanager
    def no_sync(self):
        prev, self._sync = self._sync, False
        try:
            yield
        finally:
            self._sync = prev

    def _launch(self, b: _Bucket):
        if self.gpu:
            g = self.flat.grad[b.lo:b.hi]
            if self.overlap:
                b.work = self.pg.allreduce_async(g, self.algo, scale=1.0 / self.pg.world, method=self.method)
            else:
                self.pg.allreduce(g, self.algo, scale=1.0 / self.pg.world, method=self.method)
        else:
            if self.overlap:
                b.work = self.pg.allreduce_async(b.buf, self.algo)
            else:
                self.pg.allreduce(b.buf, self.algo)

    def _on_grad(self, p):
        if not self._sync:
            return
        bi, pi = self._where[id(p)]
        b = self.buckets[bi]
        if self.gpu:
            if not self.flat.owns_grad(p):
                self.flat.grad_view(p).copy_(p.grad)
        else:
            off = b.offsets[pi]
            b.buf[off:off + p.numel()] = p.grad.detach().reshape(-1).numpy()
        b.pending -= 1
        if b.pending == 0 and self.overlap:
            self._launch(b)

    def finish(self):
        """Complete gradient synchronisation; call after the last backward of a step."""
        t0 = time.perf_counter()
        if self.gpu and not self.overlap:
            self._finish_flat()
            self.comm_wait_s += time.perf_counter() - t0
            return
        for b in self.buckets:
            if b.pending:
                # parameters that got no gradient this step contribute zeros
                for pi, p in enumerate(b.params):
                    if p.grad is None:
                        if self.gpu:
                            self.flat.grad_view(p).zero_()
                        else:
                            off = b.offsets[pi]
                            b.buf[off:off + p.numel()] = 0
                    elif self.gpu and not self.flat.owns_grad(p):
                        self.flat.grad_view(p).copy_(p.grad)
                b.pending = 0
                if self.overlap:
                    self._launch(b)
            if not self.overlap:
                self._launch(b)
        for b in self.buckets:
            if b.work is not None:
                b.work.wait()
                b.work = None
        self.comm_wait_s += time.perf_counter() - t0
        if self.gpu:
            for p in self.params:
                if not self.flat.owns_grad(p):
                    p.grad = self.flat.grad_view(p)
        else:
            inv = 1.0 / self.pg.world
            for b in self.buckets:
                b.buf *= inv
                for pi, p in enumerate(b.params):
                    off = b.offsets[pi]
                    p.grad = torch.from_numpy(b.buf[off:off + p.numel()].reshape(tuple(p.shape)).copy())
        for b in self.buckets:
            b.pending = len(b.params)

    def _finish_flat(self):
        """GPU without overlap: every gradient already sits in the one peer-mapped flat
        buffer, so the whole buffer is averaged by a single all-reduce after the
        backward pass.  The buckets only matter for overlap; one collective pays the
        cross-rank synchronisation once instead of once per bucket, and no collective
        CTA competes with the backward kernels for SMs (measured faster than per-bucket
        overlap on B200: the comm CTAs that wait on peers steal SMs from the
        persistent GEMMs)."""
        for p in self.params:
            if p.grad is None:
                self.flat.grad_view(p).zero_()
            elif not self.flat.owns_grad(p):
                self.flat.grad_view(p).copy_(p.grad)
        self.pg.allreduce(self.flat.grad, self.algo, scale=1.0 / self.pg.world, method=self.method)
        for p in self.params:
            if not self.flat.owns_grad(p):
                p.grad = self.flat.grad_view(p)
        for b in self.buckets:
            b.pending = len(b.params)

    def remove_hooks(self):
        for h in self._hooks:
            h.remove()
        self._hooks = []
