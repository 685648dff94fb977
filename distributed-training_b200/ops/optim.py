"""AdamW over flat tensors, and global-norm clipping.

API of dtrain/optim.py:7-52: ``AdamW(params, lr, betas, eps, weight_decay)`` with
``step(grads)``, ``state_dict()``, ``load_state_dict()``, ``state_bytes()``, and
``clip_scale(total_sq_norm, max_norm)``.  Parameters are updated in place, so
ZeRO can run the optimizer on a shard view of the flat master buffer.

Two code paths with the same formula and order of operations
(m = b1 m + (1-b1) g; v = b2 v + (1-b2) g^2; p -= lr*wd*p; p -= lr*(m/b1t)/(sqrt(v/b2t)+eps)):

* fp32 CUDA tensors -> the fused ``adamw_step`` kernel (one pass over p, g, m, v,
  also refreshing the bf16 working copy; the clip factor is computed on the device
  from a device-resident squared norm, so nothing waits on the host);
* anything else (CPU, float64) -> elementwise torch ops in exactly the reference's
  order, which makes float64 runs bit-identical to the NumPy reference.
"""
from __future__ import annotations

import math

import numpy as np
import torch


def clip_scale(total_sq_norm: float, max_norm: float) -> float:
    """Factor that brings the global L2 norm down to ``max_norm`` (1.0 if already below)."""
    n = math.sqrt(float(total_sq_norm))
    return 1.0 if n <= max_norm or n == 0 else max_norm / (n + 1e-6)


def _to_tensor(x):
    if isinstance(x, np.ndarray):
        return torch.from_numpy(x)
    return x


class AdamW:
    def __init__(self, params, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, work=None):
        self.params = [_to_tensor(p) for p in params]
        self.lr, self.b1, self.b2, self.eps, self.wd = lr, betas[0], betas[1], eps, weight_decay
        self.m = [torch.zeros_like(p) for p in self.params]
        self.v = [torch.zeros_like(p) for p in self.params]
        self.work = list(work) if work is not None else [None] * len(self.params)
        self.t = 0

    def _fused_ok(self, p, g) -> bool:
        return (p.is_cuda and p.dtype == torch.float32 and g is not None and g.dtype == torch.float32
                and p.is_contiguous() and g.is_contiguous())

    def step(self, grads, sq_norm: torch.Tensor | None = None, max_norm: float = 0.0):
        """One update.  ``grads`` is a list aligned with the params (None skips one).

        With ``sq_norm`` (a device fp64 scalar, sum of squared gradients) and
        ``max_norm`` > 0 the gradients are clipped on the device.
        """
        self.t += 1
        b1t = 1 - self.b1 ** self.t
        b2t = 1 - self.b2 ** self.t
        for i, (p, g) in enumerate(zip(self.params, grads)):
            if g is None:
                continue
            g = _to_tensor(g)
            m, v = self.m[i], self.v[i]
            if self._fused_ok(p, g):
                from . import kernels as K
                K.adamw_step(p, g, m, v, self.work[i], self.lr, self.b1, self.b2, self.eps, self.wd, self.t,
                             sq_norm, max_norm)
                continue
            if sq_norm is not None and max_norm:
                g = g * clip_scale(float(sq_norm.reshape(-1)[0]), max_norm)
            with torch.no_grad():
                m.mul_(self.b1)
                m.add_((1 - self.b1) * g)
                v.mul_(self.b2)
                v.add_((1 - self.b2) * (g * g))
                p.sub_(self.lr * (self.wd * p))
                p.sub_(self.lr * (m / b1t) / (torch.sqrt(v / b2t) + self.eps))
                if self.work[i] is not None:
                    self.work[i].copy_(p)

    def state_bytes(self) -> int:
        return sum(a.numel() * a.element_size() for a in self.m) + sum(a.numel() * a.element_size() for a in self.v)

    def state_dict(self):
        return {"t": self.t, "m": [a.clone() for a in self.m], "v": [a.clone() for a in self.v]}

    def load_state_dict(self, s):
        self.t = int(s["t"])
        with torch.no_grad():
            for dst, src in zip(self.m, s["m"]):
                dst.copy_(_to_tensor(np.asarray(src)) if isinstance(src, np.ndarray) else src)
            for dst, src in zip(self.v, s["v"]):
                dst.copy_(_to_tensor(np.asarray(src)) if isinstance(src, np.ndarray) else src)
