"""Import shim: exposes the package directory `flashmaxsim.jl_b200/` (whose name
is not a Python identifier) as the importable package `flashmaxsim_b200`."""
import importlib.util as _ilu
import sys as _sys
from pathlib import Path as _Path

_dir = _Path(__file__).resolve().parent / "flashmaxsim.jl_b200"
_spec = _ilu.spec_from_file_location(__name__, _dir / "__init__.py",
                                     submodule_search_locations=[str(_dir)])
_mod = _ilu.module_from_spec(_spec)
_sys.modules[__name__] = _mod
_spec.loader.exec_module(_mod)
