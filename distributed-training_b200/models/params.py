"""Flat parameter / gradient buffers shared by the model, DDP, ZeRO and the optimizer.

All parameters of a model live in one contiguous fp32 ``master`` buffer in
parameter order (the layout the reference's ZeRO uses, dtrain/zero.py:29-35, and
the ``params`` array of its checkpoints, dtrain/train.py:175-179); each
``nn.Parameter`` becomes a view into it.  For bf16 compute there is a parallel
bf16 ``work`` buffer the GEMMs read, and one fp32 ``grad`` buffer that the
backward kernels write into directly.  The grad buffer may live in symmetric
(peer-mapped) memory so DDP / ZeRO collectives run on it in place, with no
bucket copies.

Gradient hand-off to autograd: ``grad_dest(p)`` returns a *fresh* view of p's
slot when ``p.grad`` is None.  Autograd's AccumulateGrad then adopts that view as
``p.grad`` without copying (it steals a gradient tensor nobody else references),
and the post-accumulate-grad hooks fire as usual.  When ``p.grad`` already
exists (gradient accumulation) a new tensor is returned and autograd adds it.
"""
from __future__ import annotations

import torch


class FlatParams:
    def __init__(self, params, device, *, grad_buffer: torch.Tensor | None = None,
                 master_buffer: torch.Tensor | None = None, work_buffer: torch.Tensor | None = None,
                 with_work: bool = True, master_dtype: torch.dtype = torch.float32):
        self.params = list(params)
        self.device = torch.device(device)
        self.numels = [p.numel() for p in self.params]
        self.offsets = []
        off = 0
        for k in self.numels:
            self.offsets.append(off)
            off += k
        self.n = off
        self.index = {id(p): i for i, p in enumerate(self.params)}
        if master_buffer is None:
            master_buffer = torch.empty(self.n, dtype=master_dtype, device=self.device)
        assert master_buffer.numel() >= self.n and master_buffer.dtype == master_dtype
        self.master = master_buffer[: self.n]
        with torch.no_grad():
            for p, o, k in zip(self.params, self.offsets, self.numels):
                self.master[o:o + k].copy_(p.detach().reshape(-1))
                p.data = self.master[o:o + k].view(p.shape)
        self.work = None
        # set by ZeRO-1 on GPUs: forward GEMMs all-gather their weights in-kernel
        self.gather = None
        if with_work:
            if work_buffer is None:
                work_buffer = torch.empty(self.n, dtype=torch.bfloat16, device=self.device)
            self.work = work_buffer[: self.n]
            self.refresh_work()
        if grad_buffer is None:
            grad_buffer = torch.zeros(self.n, dtype=master_dtype, device=self.device)
        self.set_grad_buffer(grad_buffer)

    # ------------------------------------------------------------------ views
    def slot(self, i: int):
        return self.offsets[i], self.numels[i]

    def work_view(self, p) -> torch.Tensor:
        o, k = self.slot(self.index[id(p)])
        return self.work[o:o + k].view(p.shape)

    def grad_view(self, p) -> torch.Tensor:
        """A fresh view (new TensorImpl) of p's gradient slot."""
        o, k = self.slot(self.index[id(p)])
        return self.grad[o:o + k].view(p.shape)

    def grad_dest(self, p) -> torch.Tensor:
        """Where a backward kernel should write p's gradient (see module docstring)."""
        if p.grad is None:
            return self.grad_view(p)
        return torch.empty(p.shape, dtype=self.grad.dtype, device=self.device)

    def owns_grad(self, p) -> bool:
        g = p.grad
        return g is not None and g.data_ptr() == self.grad_view(p).data_ptr()

    # --------------------------------------------------------------- updates
    def set_grad_buffer(self, buf: torch.Tensor):
        assert buf.numel() >= self.n and buf.dtype == self.master.dtype
        self.grad = buf[: self.n]
        for p in self.params:
            p.grad = None

    def refresh_work(self):
        """Re-derive the bf16 working copy from the fp32 masters."""
        if self.work is None:
            return
        if self.master.is_cuda:
            from ..ops import kernels as K
            K.cast_f32_bf16(self.master, self.work)
        else:
            self.work.copy_(self.master)

    def flat_grad_from_params(self, out: torch.Tensor | None = None) -> torch.Tensor:
        """Gather p.grad (zeros where None) into the flat grad buffer, skipping slots already in place."""
        g = self.grad if out is None else out
        for p, o, k in zip(self.params, self.offsets, self.numels):
            if p.grad is None:
                g[o:o + k].zero_()
            elif not (out is None and self.owns_grad(p)):
                g[o:o + k].copy_(p.grad.reshape(-1))
        return g
