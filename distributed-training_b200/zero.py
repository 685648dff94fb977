"""Reference module name ``dtrain.zero``."""
from .parallel.zero import ZeroAdamW  # noqa: F401
