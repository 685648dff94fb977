"""Reference module name ``dtrain.autograd``.

The autograd engine is PyTorch's; this module keeps the reference's names:
``Tensor``, ``no_grad``, the grad-ready hook and the functional ops.
"""
from .ops.functional import (Tensor, causal_attention, cross_entropy, embedding, gelu,  # noqa: F401
                             layer_norm, linear, no_grad, register_grad_ready_hook, relu)
