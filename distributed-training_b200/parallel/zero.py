"""ZeRO-1 sharded AdamW (stage-1 state sharding, stage-2 style gradient reduce-scatter).

API of dtrain/zero.py:23-71: ``ZeroAdamW(model, pg, max_grad_norm=None, **adam)``
with ``step()``, ``state_bytes()``, ``state_dict()``, ``load_state_dict()``,
``flat``, ``opt``, ``last_grad_norm``.

All parameters live in one flat buffer (each parameter is a view into it); the
buffer is partitioned with ``partition(n, W)`` and rank r keeps the AdamW state
of partition r only.  Each step: reduce-scatter the gradient (this rank receives
the summed gradient of its partition), scale by 1/W, global-norm clip, AdamW on
the partition, all-gather the parameters.

GPU path (``NVLinkGroup``), one kernel per step on 2+ GPUs (``zero_rs_adamw``,
``fuse_rs=True``) doing what the two-kernel path (``fuse_rs=False``, and one GPU)
does in two launches with a kernel boundary as the grid-wide sync:

1. ``reduce_scatter`` kernel: the owner of each partition reads it from every
   peer over NVLink, sums in ring order, scales by 1/W, writes it in place and
   writes per-CTA sums of squares (fp64) into a peer-mapped slot;
2. ``zero_adamw_allgather`` kernel: every CTA sums all ranks' norm partials in a
   fixed order (identical global norm everywhere), applies the clip factor and
   AdamW to its slice of the partition - fp32 master plus bf16 working copy - and
   after a cross-GPU barrier pulls the peers' updated bf16 partitions straight
   into the working buffer the next forward's GEMMs read;
In the fused kernel a grid-wide cross-rank flag barrier separates 1 from 2 and
each CTA updates exactly the slice of the partition it reduced.

3. with ``gather_gemm`` (bf16 models on 2+ GPUs; off by default because the bulk
   gather in step 2 measured faster on B200, GPT-2-medium on 2 GPUs: 115.0 vs
   116.8 ms per step) step 2 pulls
   only the parameters that are not Linear weights (embeddings, LayerNorm,
   biases) and publishes a new generation number; each Linear weight is pulled
   by the first forward GEMM that reads it (``gemm_gather``): gather warps inside
   the GEMM copy the other ranks' partitions k-block by k-block into local memory
   while the tensor cores consume the k-blocks already in place.  Later forwards
   of the same step (gradient accumulation) see the generation already gathered
   and skip the copy.

The fp32 masters of other partitions are gathered only when needed
(``gather_params()``, e.g. before a checkpoint), which halves the all-gather
traffic compared with gathering fp32 every step.

Host path (TCP ``ProcessGroup``): the reference algorithm on host tensors.
"""
from __future__ import annotations

import math

import numpy as np
import torch

from ..ops.optim import AdamW, clip_scale
from .comm import partition


GS_GEN = 131     # gemm.cu: state word holding the generation the weights must reach
GS_SITES = 256   # gemm.cu: first per-weight "generation gathered" word


def keep_intervals(n: int, skip: list[tuple[int, int]]) -> list[tuple[int, int]]:
    """Complement of the (possibly unsorted, non-overlapping) ``skip`` intervals in [0, n)."""
    out, cur = [], 0
    for lo, hi in sorted(skip):
        if lo > cur:
            out.append((cur, lo))
        cur = max(cur, hi)
    if cur < n:
        out.append((cur, n))
    return out


class GatherPlan:
    """What the in-GEMM all-gather needs to know about the partitioned bf16 buffer:
    per weight (keyed by ``id(param)``) its site slot, flat offset and every
    rank's address of it, plus the shared int32 state words (``gemm.cu: GS_*``)."""

    def __init__(self, fp, weights, work_ptrs: list[int], rank: int):
        self.rank = rank
        self.nflat = fp.n
        self.sites = {}
        skip = []
        for s, w in enumerate(weights):
            off, k = fp.slot(fp.index[id(w)])
            self.sites[id(w)] = (s, off, [p + 2 * off for p in work_ptrs])
            skip.append((off, off + k))
        self.state = torch.zeros(GS_SITES + max(len(weights), 1), dtype=torch.int32, device=fp.device)
        self.gen_word = self.state[GS_GEN:GS_GEN + 1]
        keep = keep_intervals(fp.n, skip)
        self.keep = torch.tensor(keep if keep else [(0, 0)], dtype=torch.int64, device=fp.device).reshape(-1, 2)

    def mark_gathered(self):
        """Record (on the device) that every weight holds the current generation."""
        self.state[GS_SITES:GS_SITES + len(self.sites)].copy_(self.gen_word.expand(len(self.sites)))


class ZeroAdamW:
    def __init__(self, model, pg, max_grad_norm: float | None = None, gather_master: bool | None = None,
                 gather_gemm: bool = False, fuse_rs: bool = True, **adam):
        self.pg = pg
        self.model = model
        self.params = list(model.parameters())
        self.gpu = getattr(pg, "backend", "tcp") == "nvlink"
        n = sum(p.numel() for p in self.params)
        self.n = n
        if self.gpu:
            fused = getattr(getattr(model, "c", None), "fused", False)
            fp = model.flatten(pg.device, grad_buffer=pg.alloc(n, torch.float32),
                               master_buffer=pg.alloc(n, torch.float32),
                               work_buffer=pg.alloc(n, torch.bfloat16) if fused else None)
            pg.broadcast(fp.master, root=0, cast_to=fp.work)
            self.fp = fp
            self.flat = fp.master
            self.gflat = fp.grad
            self._sq_parts = pg.alloc(128, torch.float64)
            self._sq_total = torch.zeros(1, dtype=torch.float64, device=pg.device)
            self.gather_master = (not fused) if gather_master is None else gather_master
            self.fuse_rs = fuse_rs
            self.plan = None
            if fused and gather_gemm and pg.world > 1 and hasattr(model, "gemm_weights"):
                self.plan = GatherPlan(fp, model.gemm_weights(), self._ptrs_of(fp.work), pg.rank)
                fp.gather = self.plan
        else:
            dtype = self.params[0].dtype
            self.flat = torch.empty(n, dtype=dtype)
            off = 0
            with torch.no_grad():
                for p in self.params:
                    k = p.numel()
                    self.flat[off:off + k].copy_(p.detach().reshape(-1))
                    p.data = self.flat[off:off + k].view(p.shape)
                    off += k
            pg.broadcast(self.flat.numpy(), root=0)
            self.gflat = torch.empty(n, dtype=dtype)
            self.fp = None
        self.bounds = partition(n, pg.world)
        lo, hi = self.bounds[pg.rank], self.bounds[pg.rank + 1]
        self.shard = self.flat[lo:hi]
        self.opt = AdamW([self.shard], **adam)
        self.max_grad_norm = max_grad_norm
        self._last_norm = 0.0

    @property
    def last_grad_norm(self) -> float:
        if self.gpu:
            return math.sqrt(float(self._sq_total.item()))
        return self._last_norm

    def step(self):
        if self.gpu:
            self._step_gpu()
        else:
            self._step_host()

    def _step_gpu(self):
        pg, fp = self.pg, self.fp
        # gradients that landed outside the flat buffer (or none at all)
        for p in self.params:
            if p.grad is None:
                fp.grad_view(p).zero_()
            elif not fp.owns_grad(p):
                fp.grad_view(p).copy_(p.grad)
        W = pg.world
        nparts = pg._rs_blocks()
        from ..ops._ext import lib
        sq_ptrs = [b.ptrs for b in pg.buffers if b.contains(self._sq_parts) is not None][0]
        opt = self.opt
        if W > 1 and self.fuse_rs:
            # one kernel: reduce-scatter + norm exchange + clip + AdamW + all-gather
            opt.t += 1
            lib().zero_rs_adamw(
                pg._sigs, pg.rank, self._ptrs_of(self.gflat), sq_ptrs, self.flat, opt.m[0], opt.v[0],
                [self._ptrs_of(fp.work)[r] if fp.work is not None else 0 for r in range(W)],
                self._ptrs_of(self.flat), self.n, opt.lr, opt.b1, opt.b2, opt.eps, opt.wd, opt.t, 1.0 / W,
                float(self.max_grad_norm or 0.0), self._sq_total, bool(self.gather_master), pg.timeout, nparts,
                self.plan.keep if self.plan is not None else None,
                self.plan.gen_word if self.plan is not None else None)
            pg._issued()
            return
        if W > 1:
            pg.reduce_scatter(self.gflat, scale=1.0 / W, sq_parts=self._sq_parts)
        else:
            from ..ops import kernels as K
            # single rank: partials = the plain squared norm, in slot 0
            self._sq_parts.zero_()
            K.grad_sqnorm(self.gflat, self._sq_parts[:1])
            nparts = 1
        opt.t += 1
        lib().zero_adamw_allgather(
            pg._sigs, pg.rank, sq_ptrs, nparts, self.flat, self.gflat, opt.m[0], opt.v[0],
            [self._ptrs_of(fp.work)[r] if fp.work is not None else 0 for r in range(W)],
            self._ptrs_of(self.flat), self.n, opt.lr, opt.b1, opt.b2, opt.eps, opt.wd, opt.t,
            float(self.max_grad_norm or 0.0), self._sq_total, bool(self.gather_master), pg.timeout, 0,
            self.plan.keep if self.plan is not None else None,
            self.plan.gen_word if self.plan is not None else None)
        pg._issued()

    def _ptrs_of(self, t: torch.Tensor):
        buf, off = self.pg._locate(t)
        return [p + off for p in buf.ptrs]

    def _step_host(self):
        off = 0
        for p in self.params:
            k = p.numel()
            if p.grad is None:
                self.gflat[off:off + k] = 0
            else:
                self.gflat[off:off + k] = p.grad.reshape(-1)
            off += k
        g = self.pg.reduce_scatter(self.gflat.numpy())
        g *= 1.0 / self.pg.world
        g64 = g.astype(np.float64)
        sq = np.array([float(np.dot(g64, g64))])
        self.pg.allreduce(sq)
        self._last_norm = float(np.sqrt(sq[0]))
        if self.max_grad_norm:
            g *= clip_scale(sq[0], self.max_grad_norm)
        self.opt.step([torch.from_numpy(g)])
        self.pg.all_gather(self.flat.numpy())

    def gather_params(self):
        """Make ``flat`` hold every partition's current fp32 parameters on every rank
        (and the bf16 working copy every partition's weights, which the forward GEMMs
        would otherwise pull on their next call)."""
        if self.gpu and not self.gather_master and self.pg.world > 1:
            self.pg.all_gather(self.flat)
        if self.gpu and self.plan is not None:
            self.pg.all_gather(self.fp.work)
            self.plan.mark_gathered()

    def state_bytes(self) -> int:
        return self.opt.state_bytes()

    def state_dict(self):
        return self.opt.state_dict()

    def load_state_dict(self, s):
        self.opt.load_state_dict(s)
        if self.fp is not None:
            self.fp.refresh_work()
