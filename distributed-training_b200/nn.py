"""Reference module name ``dtrain.nn``: modules and the GPT model (torch.nn based)."""
from torch.nn import Module  # noqa: F401

from .models.gpt import GPT, Block, GPTConfig, LayerNorm, Linear  # noqa: F401
from .models.params import FlatParams  # noqa: F401
