"""Import name for the package in ``distributed-training_b200/``.

The package directory name is not a Python identifier, so this module binds it
to the import name ``dtrain_b200``: ``import dtrain_b200`` and
``python -m dtrain_b200.train`` load the package from that directory.
"""
import importlib.util as _ilu
import os as _os
import sys as _sys

_DIR = _os.path.join(_os.path.dirname(_os.path.abspath(__file__)), "distributed-training_b200")
_spec = _ilu.spec_from_file_location(__name__, _os.path.join(_DIR, "__init__.py"), submodule_search_locations=[_DIR])
_mod = _ilu.module_from_spec(_spec)
_sys.modules[__name__] = _mod
_spec.loader.exec_module(_mod)
