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

``method="nvls"`` (a group made with ``nvls=True``) reduces the buckets in the
NVSwitch instead (multimem.ld_reduce / multimem.st): every rank still ends with the
same bits, in the switch's summation order rather than ``algo``'s.

GPU path (``pg`` is an ``NVLinkGroup``): the model's parameters and gradients
are moved into flat peer-mapped buffers, so every bucket is a contiguous slice
of the flat gradient that the backward kernels already wrote.  The bucket
all-reduce is one kernel (``csrc/comm.cu``) on the comm stream that reads the
peers' slices over NVLink, sums them in the fixed order, multiplies by 1/W and
writes the result in place - the reference's copy-in, all-reduce, scale and
copy-out (dtrain/ddp.py:73-110) collapse into that kernel.  The same kernel
publishes the sum of squares of what it reduced, so the gradient norm for
clipping (dtrain/train.py:155-158) costs no second pass: ``finish()`` makes the
compute stream wait for the comm stream and sums those partials in a fixed order
into ``sq_norm``; no host synchronisation.

Buckets reduced while backward is still running use lean 128-thread CTAs, which
fit beside the GEMM and attention CTAs on each SM instead of holding SMs those
persistent kernels need; buckets whose gradients come from the last backward
kernel (the embeddings, ``model.late_grad_params()``) have the GPU to themselves
and use full-width CTAs.  The launches are the same every step (the flag epochs
live on the device), so the whole forward + backward + bucket all-reduces can be
captured in one CUDA graph (``Trainer --cuda-graph``).

Host path (``pg`` is a TCP ``ProcessGroup``): the reference algorithm on host
buffers, used by CPU ranks and the float64 oracle tests.
"""
from __future__ import annotations

import contextlib
import os
import time

import numpy as np
import torch

# Upper bound on the CTAs of a bucket all-reduce that runs during backward
# (0: one per SM at most, sized by the bucket).
LEAN_BLOCKS = int(os.environ.get("DTB_DDP_LEAN_BLOCKS", "0"))


class _Bucket:
    def __init__(self, params, lo=None, hi=None):
        self.params = params
        self.pending = len(params)
        self.work = None
        self.lo, self.hi = lo, hi          # flat-gradient range (GPU path)
        self.buf = None                    # host buffer (TCP path)
        self.offsets = []
        # GPU launch plan: CTA count, lean or full-width CTAs, first sum-of-squares slot
        self.blocks, self.lean, self.sq_base = 0, False, 0
        self.index = 0


class DDP:
    def __init__(self, model, pg, bucket_mb: float = 1.0, overlap: bool = True, algo: str = "ring",
                 method: str = "auto"):
        self.model, self.pg, self.overlap, self.algo, self.method = model, pg, overlap, algo, method
        if method not in ("auto", "oneshot", "twoshot", "nvls"):
            raise ValueError(f"unknown DDP all-reduce method {method!r} (auto, oneshot, twoshot or nvls)")
        if method == "nvls" and getattr(pg, "world", 1) > 1 and not getattr(pg, "nvls", False):
            # checked here rather than at the first bucket launch, in the middle of backward
            raise ValueError("method='nvls' needs an NVLinkGroup made with nvls=True (DTB_NVLS=1)")
        self.params = list(model.parameters())
        self.gpu = getattr(pg, "backend", "tcp") == "nvlink"
        # one GPU: the flat buffer already holds the averaged gradient, nothing to launch
        self._single_gpu = self.gpu and pg.world == 1
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
            b.index = bi
            for pi, p in enumerate(b.params):
                self._where[id(p)] = (bi, pi)
        self._trace = None
        if self.gpu:
            self._plan_gpu()
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

    def _plan_gpu(self):
        """Per-bucket launch plan and the sum-of-squares pad: bucket b's CTAs own
        slots [b.sq_base, b.sq_base + b.blocks) of every rank's row; the single flat
        all-reduce of the no-overlap path owns the slots after the last bucket's."""
        pg = self.pg
        late = getattr(self.model, "late_grad_params", None)
        late_ids = {id(p) for p in late()} if callable(late) else {id(self.params[0])}
        cur = 0
        for b in self.buckets:
            nbytes = (b.hi - b.lo) * self.flat.grad.element_size()
            b.lean = self.overlap and not any(id(p) in late_ids for p in b.params)
            b.blocks = pg.collective_blocks(nbytes, lean=b.lean)
            if b.lean and LEAN_BLOCKS > 0:
                b.blocks = min(b.blocks, LEAN_BLOCKS)
            b.sq_base = cur
            cur += b.blocks
        self._sq_lo_buckets, self._sq_hi_buckets = 0, cur
        self._flat_blocks = pg.collective_blocks(self.flat.n * self.flat.grad.element_size(), lean=False)
        self._sq_lo_flat, self._sq_hi_flat = cur, cur + self._flat_blocks
        self._sq_stride = cur + self._flat_blocks
        # the two-shot and NVLS kernels publish the sums of squares; one-shot does not
        self.fused_norm = pg.world > 1 and self.method != "oneshot"
        self._sq_pad = pg.alloc(pg.world * self._sq_stride, torch.float64) if self.fused_norm else None
        # global sum of squares of the averaged gradient, written by finish()
        self.sq_norm = torch.zeros(1, dtype=torch.float64, device=pg.device)

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

    # ------------------------------------------------------------- tracing
    def enable_trace(self):
        """Record device timestamps (%globaltimer, ns) of every step: the step's start
        (``trace_begin``), each bucket's ready point on the compute stream and its
        all-reduce's start and end on the comm stream, and the join in ``finish()``.
        The stamps are kernels too, so they are captured with a CUDA graph and
        refreshed by every replay.  ``trace_report()`` reads the last step."""
        if self.gpu:
            self._trace = torch.zeros(3 * len(self.buckets) + 3, dtype=torch.int64, device=self.pg.device)

    def _stamp(self, slot: int):
        if self._trace is not None:
            from ..ops._ext import lib
            lib().stamp(self._trace, slot)

    def trace_begin(self):
        self._stamp(3 * len(self.buckets))

    def trace_report(self) -> dict | None:
        if self._trace is None:
            return None
        nb = len(self.buckets)
        t = self._trace.cpu().tolist()
        t0 = t[3 * nb]
        ms = lambda v: round((v - t0) / 1e6, 4) if v else None  # noqa: E731
        rep = {"join_ms": ms(t[3 * nb + 1])}
        if self.overlap:
            rows = [(ms(t[3 * i]), ms(t[3 * i + 1]), ms(t[3 * i + 2])) for i in range(nb)]
            rep["buckets_ready_start_end_ms"] = rows
            rep["backward_end_ms"] = max(r[0] for r in rows)
            rep["comm_busy_ms"] = round(sum(r[2] - r[1] for r in rows), 4)
            rep["exposed_after_backward_ms"] = round(rep["join_ms"] - rep["backward_end_ms"], 4)
        else:
            rep["backward_end_ms"] = ms(t[3 * nb + 2])
            rep["exposed_after_backward_ms"] = round(rep["join_ms"] - rep["backward_end_ms"], 4)
        return rep

    def _launch(self, b: _Bucket):
        if self.gpu:
            g = self.flat.grad[b.lo:b.hi]
            if self._trace is not None:
                self._stamp(3 * b.index)
                kw_trace = dict(stamps=(self._trace, 3 * b.index + 1, 3 * b.index + 2))
            else:
                kw_trace = {}
            if self.method == "oneshot":
                kw = dict(method="oneshot")
            else:
                kw = dict(method="nvls" if self.method == "nvls" else "twoshot", blocks=b.blocks, lean=b.lean,
                          sq=(self._sq_pad, b.sq_base, self._sq_stride) if self.fused_norm else None)
            if self.overlap:
                b.work = self.pg.allreduce_async(g, self.algo, scale=1.0 / self.pg.world, **kw, **kw_trace)
            else:
                self.pg.allreduce(g, self.algo, scale=1.0 / self.pg.world, **kw)
        else:
            if self.overlap:
                b.work = self.pg.allreduce_async(b.buf, self.algo)
            else:
                self.pg.allreduce(b.buf, self.algo)

    def _on_grad(self, p):
        if not self._sync or self._single_gpu:
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
        if self._single_gpu:
            for p in self.params:
                if p.grad is None:
                    self.flat.grad_view(p).zero_()
                elif not self.flat.owns_grad(p):
                    self.flat.grad_view(p).copy_(p.grad)
                    p.grad = self.flat.grad_view(p)
            return
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
                # the handle (and its event) is kept until the bucket's next launch:
                # inside a graph capture nothing may be destroyed mid-capture
                b.work.wait()
        self.comm_wait_s += time.perf_counter() - t0
        if self.gpu:
            self._stamp(3 * len(self.buckets) + 1)
            if self.fused_norm:
                self.pg.sq_total(self._sq_pad, self.sq_norm, self._sq_stride, self._sq_lo_buckets,
                                 self._sq_hi_buckets)
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
        """GPU without overlap (``overlap=False``): every gradient already sits in the
        one peer-mapped flat buffer, so the whole buffer is averaged by a single
        full-width all-reduce after the backward pass (which also yields the
        gradient's sum of squares)."""
        for p in self.params:
            if p.grad is None:
                self.flat.grad_view(p).zero_()
            elif not self.flat.owns_grad(p):
                self.flat.grad_view(p).copy_(p.grad)
        self._stamp(3 * len(self.buckets) + 2)
        if self.method == "oneshot":
            self.pg.allreduce(self.flat.grad, self.algo, scale=1.0 / self.pg.world, method="oneshot")
        else:
            self.pg.allreduce(self.flat.grad, self.algo, scale=1.0 / self.pg.world,
                              method="nvls" if self.method == "nvls" else "twoshot", blocks=self._flat_blocks,
                              sq=(self._sq_pad, self._sq_lo_flat, self._sq_stride) if self.fused_norm else None)
        self._stamp(3 * len(self.buckets) + 1)
        if self.fused_norm:
            self.pg.sq_total(self._sq_pad, self.sq_norm, self._sq_stride, self._sq_lo_flat, self._sq_hi_flat)
        for p in self.params:
            if not self.flat.owns_grad(p):
                p.grad = self.flat.grad_view(p)
        for b in self.buckets:
            b.pending = len(b.params)

    def remove_hooks(self):
        for h in self._hooks:
            h.remove()
        self._hooks = []
