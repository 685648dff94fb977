"""Reference module name ``dtrain.optim``."""
from .ops.optim import AdamW, clip_scale  # noqa: F401
