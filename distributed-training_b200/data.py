"""Reference module name ``dtrain.data``."""
from .utils.data import (CharData, SyntheticData, global_batch, load_text, lr_at,  # noqa: F401
                         rank_batch)
