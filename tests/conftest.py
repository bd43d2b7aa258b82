"""Shared pytest setup: the ``gpu`` marker, import paths, and loaders for the oracle and the product package."""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG_DIR = ROOT / "mlx-flashvsr-swift_b200"
for p in (ROOT, ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def load_product():
    """Import the product package (its directory name is not a Python identifier) as ``fvsr_b200``."""
    if "fvsr_b200" in sys.modules:
        return sys.modules["fvsr_b200"]
    spec = importlib.util.spec_from_file_location("fvsr_b200", PKG_DIR / "__init__.py",
                                                  submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["fvsr_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle as o
    o.lib()
    return o


@pytest.fixture(scope="session")
def fvsr():
    mod = load_product()
    mod.build()          # in-tree nvcc build; a no-op when the library is newer than its sources
    return mod
