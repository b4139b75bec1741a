"""Import name for the package directory ``fp4-fused-attention-sm120_b200/``.

A directory name with dashes cannot be imported directly, so this module
loads that package's ``__init__.py`` and registers it as ``fp4attn_b200``.
"""
import importlib.util
import pathlib
import sys

_PKG_DIR = pathlib.Path(__file__).resolve().parent / "fp4-fused-attention-sm120_b200"
_spec = importlib.util.spec_from_file_location(
    __name__, _PKG_DIR / "__init__.py", submodule_search_locations=[str(_PKG_DIR)])
_mod = importlib.util.module_from_spec(_spec)
sys.modules[__name__] = _mod
_spec.loader.exec_module(_mod)
