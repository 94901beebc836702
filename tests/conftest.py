"""Shared pytest setup: the `gpu` marker and loaders for the package and oracle.

The package directory is ``bare-metal-llm-engine_b200/`` (not an importable
identifier), so it is loaded under the module name ``bmle_b200``.
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG_DIR = ROOT / "bare-metal-llm-engine_b200"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def load_package():
    if "bmle_b200" in sys.modules:
        return sys.modules["bmle_b200"]
    spec = importlib.util.spec_from_file_location(
        "bmle_b200", PKG_DIR / "__init__.py", submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["bmle_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def pkg():
    return load_package()


@pytest.fixture(scope="session")
def dev():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
