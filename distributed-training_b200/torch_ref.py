"""Reference module name ``dtrain.torch_ref``: the plain-torch mirror of the GPT.

``TorchGPT.from_dtrain(model)`` copies a GPT (this package's or the reference's
NumPy one) into a module that always runs the reference math in torch ops
(dtrain/torch_ref.py:22-74): same parameter order, (in, out) weights, explicit
masked-softmax attention, tanh GELU, mean cross-entropy.  It is the cross-check
model for equivalence tests and the model of the torch/NCCL baseline.
"""
from __future__ import annotations

import numpy as np
import torch

from .models.gpt import GPT, GPTConfig


class TorchGPT(GPT):
    def __init__(self, cfg, named_arrays):
        c = GPTConfig(vocab=cfg.vocab, ctx=cfg.ctx, dim=cfg.dim, heads=cfg.heads, layers=cfg.layers,
                      dtype=str(np.dtype(named_arrays[0][1].dtype)) if not isinstance(named_arrays[0][1], torch.Tensor)
                      else str(named_arrays[0][1].dtype).replace("torch.", ""))
        super().__init__(c, seed=0)
        own = dict(self.named_parameters())
        with torch.no_grad():
            for name, arr in named_arrays:
                src = arr.detach() if isinstance(arr, torch.Tensor) else torch.from_numpy(np.array(arr, copy=True))
                own[name].data = src.clone().to(own[name].device)
        self.names = [n for n, _ in named_arrays]

    @classmethod
    def from_dtrain(cls, model):
        cfg = model.c
        named = [(n, p.data if hasattr(p, "data") else p) for n, p in model.named_parameters()]
        return cls(cfg, named)

    def forward(self, idx, targets=None):
        if not isinstance(idx, torch.Tensor):
            idx = torch.as_tensor(np.asarray(idx, dtype=np.int64))
        if targets is not None and not isinstance(targets, torch.Tensor):
            targets = torch.as_tensor(np.asarray(targets, dtype=np.int64))
        return self.forward_reference(idx.long(), None if targets is None else targets.long())

    def flat_params(self) -> np.ndarray:
        return np.concatenate([p.detach().cpu().numpy().reshape(-1) for p in self.parameters()])

    def flat_grads(self) -> np.ndarray:
        return np.concatenate([p.grad.detach().cpu().numpy().reshape(-1) for p in self.parameters()])
