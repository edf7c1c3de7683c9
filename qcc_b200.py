"""Import shim: exposes the package directory ``qwen-contextual-compression_b200/``
under the importable name ``qcc_b200`` (a hyphenated directory cannot be
imported directly).  ``import qcc_b200`` replaces this module with the package.
"""
import importlib.util as _util
import sys as _sys
from pathlib import Path as _Path

_ROOT = _Path(__file__).resolve().parent / "qwen-contextual-compression_b200"
_spec = _util.spec_from_file_location(__name__, _ROOT / "__init__.py", submodule_search_locations=[str(_ROOT)])
_module = _util.module_from_spec(_spec)
_sys.modules[__name__] = _module
_spec.loader.exec_module(_module)
