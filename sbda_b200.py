"""Import shim: makes ``import sbda_b200`` load the package directory
``staged-binary-local-diffusion-attention_b200/`` (whose name is not a Python
identifier)."""

import importlib.util
import os
import sys

_PKG_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)),
                        "staged-binary-local-diffusion-attention_b200")
_spec = importlib.util.spec_from_file_location(
    __name__, os.path.join(_PKG_DIR, "__init__.py"), submodule_search_locations=[_PKG_DIR])
_module = importlib.util.module_from_spec(_spec)
sys.modules[__name__] = _module
_spec.loader.exec_module(_module)
