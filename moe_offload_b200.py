"""Import shim: the package lives in the directory `moe-offload_b200/`, whose name is not
a valid Python identifier. `import moe_offload_b200` loads that directory as the package
of this name (submodules resolve inside it)."""
import importlib.util
import os
import sys

_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "moe-offload_b200")
_spec = importlib.util.spec_from_file_location(
    __name__, os.path.join(_DIR, "__init__.py"), submodule_search_locations=[_DIR])
_mod = importlib.util.module_from_spec(_spec)
sys.modules[__name__] = _mod
_spec.loader.exec_module(_mod)
