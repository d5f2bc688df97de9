from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))
os.environ.setdefault("PYTHONDONTWRITEBYTECODE", "1")


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU and the built kernel library")


def pytest_collection_modifyitems(config: pytest.Config, items: list[pytest.Item]) -> None:
    # GPU tests fail loudly (rather than skip) when selected without a GPU, so a
    # `-m gpu` run on a machine without one never passes silently.
    del config, items
