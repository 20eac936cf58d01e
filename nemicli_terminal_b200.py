"""Import name of the package kept in the directory `nemicli-terminal_b200/` (a directory name
Python cannot import directly): `import nemicli_terminal_b200` loads that directory as the package."""
import importlib.util as _util
import os as _os
import sys as _sys

_dir = _os.path.join(_os.path.dirname(_os.path.abspath(__file__)), "nemicli-terminal_b200")
_spec = _util.spec_from_file_location(__name__, _os.path.join(_dir, "__init__.py"), submodule_search_locations=[_dir])
_mod = _util.module_from_spec(_spec)
_sys.modules[__name__] = _mod
_spec.loader.exec_module(_mod)
