"""Import shim: the rldx_b200 package lives in the directory `rldx-1_b200/` (a name that is not a
valid Python identifier).  `import rldx_b200` from the repository root loads that directory as
the package `rldx_b200`."""

import importlib.util as _util
import sys as _sys
from pathlib import Path as _Path

_DIR = _Path(__file__).resolve().parent / "rldx-1_b200"
_spec = _util.spec_from_file_location(__name__, _DIR / "__init__.py",
                                      submodule_search_locations=[str(_DIR)])
_mod = _util.module_from_spec(_spec)
_sys.modules[__name__] = _mod
_spec.loader.exec_module(_mod)
