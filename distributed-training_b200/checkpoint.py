"""Reference module name ``dtrain.checkpoint``."""
from .utils.checkpoint import latest, load, save, sha256_file  # noqa: F401
