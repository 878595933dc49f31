"""Import shim: the package lives in the directory ``kernelbench-harbor_b200/``,
whose name is not a Python identifier.  Importing this module loads that
directory as the package ``kernelbench_harbor_b200`` and replaces this shim in
``sys.modules``, so ``import kernelbench_harbor_b200.ops`` etc. work as usual."""
import importlib.util as _ilu
import os as _os
import sys as _sys

_PKG_DIR = _os.path.join(_os.path.dirname(_os.path.abspath(__file__)), "kernelbench-harbor_b200")
_spec = _ilu.spec_from_file_location(__name__, _os.path.join(_PKG_DIR, "__init__.py"),
                                     submodule_search_locations=[_PKG_DIR])
_mod = _ilu.module_from_spec(_spec)
_sys.modules[__name__] = _mod
_spec.loader.exec_module(_mod)
