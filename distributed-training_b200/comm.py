"""Reference module name ``dtrain.comm``: stores, process groups, collectives.

Host/TCP backend: ``ProcessGroup`` (``parallel/comm.py``); GPU backend over
NVLink / NVSwitch: ``NVLinkGroup`` (``parallel/nvlink.py``).
"""
from .parallel.comm import ProcessGroup, Work, init_from_env, partition  # noqa: F401
from .parallel.nvlink import NVLinkGroup, SymmetricBuffer, from_env, store_exchange, torch_exchange  # noqa: F401
from .utils.store import CommError, Store, StoreServer  # noqa: F401
