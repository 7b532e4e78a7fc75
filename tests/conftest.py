"""Shared pytest set-up: the ``gpu`` marker, package import and CUDA fixtures."""
from __future__ import annotations

import importlib
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

PKG = "emmy-hackathon-2026_b200"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


def pkg(name: str | None = None):
    """Import the backend package (or one of its submodules)."""
    return importlib.import_module(PKG if name is None else f"{PKG}.{name}")


@pytest.fixture(scope="session")
def torch_cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.fixture(scope="session")
def ctx(torch_cuda):
    runtime = pkg("runtime")
    torch_cuda.cuda.init()
    context = runtime.Context(0)
    yield context
    context.close()


def golden_cases(families=None, payload_only=True):
    import json
    manifest = json.loads((GOLDEN / "manifest.json").read_text())
    rows = [c for c in manifest["cases"] if (not payload_only or c["payload"])]
    if families is not None:
        rows = [c for c in rows if c["family"] in families]
    return rows
