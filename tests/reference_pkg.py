"""Import of the reference package itself, for the tests of ``tropnn_b200.register`` (test helper).

The reference is looked for as an installed ``tropnn`` package under ``baseline/_ref`` at the
repository root (``pip install --no-deps --target baseline/_ref <reference source>``), or under
the directory named by the ``TROPNN_REFERENCE`` environment variable. Tests that need it skip
when neither holds it.
"""

from __future__ import annotations

import importlib
import os
import sys
from pathlib import Path
from types import ModuleType

import pytest

REPO = Path(__file__).resolve().parent.parent


def reference_root() -> Path | None:
    for root in (os.environ.get("TROPNN_REFERENCE"), str(REPO / "baseline" / "_ref")):
        if root and (Path(root) / "tropnn" / "__init__.py").is_file():
            return Path(root)
    return None


def import_reference() -> ModuleType:
    """The reference ``tropnn`` package with ``backend="b200"`` registered on its layers."""
    root = reference_root()
    if root is None:
        pytest.skip("the reference package is not installed under baseline/_ref (or TROPNN_REFERENCE)")
    if str(root) not in sys.path:
        sys.path.append(str(root))
    tropnn = importlib.import_module("tropnn")
    import tropnn_b200

    tropnn_b200.register(tropnn)
    return tropnn
