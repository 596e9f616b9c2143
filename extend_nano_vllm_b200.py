"""Import shim: makes the package directory ``extend-nano-vllm_b200/`` (whose
name is not a Python identifier) importable as ``extend_nano_vllm_b200``.

Importing this module loads the package from that directory and replaces
itself in ``sys.modules`` with it, so ``import extend_nano_vllm_b200`` and
``from extend_nano_vllm_b200.moe import ExpertParallelMoE`` both work.
"""

import importlib.util as _util
import os as _os
import sys as _sys

_PKG_DIR = _os.path.join(_os.path.dirname(_os.path.abspath(__file__)), "extend-nano-vllm_b200")
_spec = _util.spec_from_file_location(
    __name__, _os.path.join(_PKG_DIR, "__init__.py"), submodule_search_locations=[_PKG_DIR])
_module = _util.module_from_spec(_spec)
_sys.modules[__name__] = _module
_spec.loader.exec_module(_module)
