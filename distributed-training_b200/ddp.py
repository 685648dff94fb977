"""Reference module name ``dtrain.ddp``."""
from .parallel.ddp import DDP  # noqa: F401
