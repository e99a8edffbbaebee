"""Import shim for the ``gaussian-splats_b200/`` package directory.

The package directory name contains a dash, which ``import`` cannot spell.
Importing ``gaussian_splats_b200`` runs this file, which loads
``gaussian-splats_b200/__init__.py`` as the package of that name and replaces
itself in ``sys.modules``, so ``import gaussian_splats_b200.rasterize`` and
friends resolve inside the directory.
"""

import importlib.util
import os
import sys

_PACKAGE_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "gaussian-splats_b200")
_spec = importlib.util.spec_from_file_location(
    __name__,
    os.path.join(_PACKAGE_DIR, "__init__.py"),
    submodule_search_locations=[_PACKAGE_DIR],
)
_module = importlib.util.module_from_spec(_spec)
sys.modules[__name__] = _module
_spec.loader.exec_module(_module)
