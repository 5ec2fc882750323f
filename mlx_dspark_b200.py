"""Import shim: the package lives in the hyphenated directory ``mlx-dspark_b200/``.

``import mlx_dspark_b200`` (from the repository root) loads that directory as the package
``mlx_dspark_b200`` so its modules import as ``mlx_dspark_b200.skinny_qmm`` etc.
"""

import importlib.util
import os
import sys

_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "mlx-dspark_b200")
_spec = importlib.util.spec_from_file_location(
    "mlx_dspark_b200", os.path.join(_DIR, "__init__.py"), submodule_search_locations=[_DIR])
_mod = importlib.util.module_from_spec(_spec)
sys.modules["mlx_dspark_b200"] = _mod
_spec.loader.exec_module(_mod)
