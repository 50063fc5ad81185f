"""Shared test helpers.

``-m gpu`` tests need a B200 and the built ``libmoe_b200.so``; everything
else runs on CPU.  The product package lives in a directory whose name is not
a Python identifier, so it is loaded by path under the name ``moe_b200``.
The CPU checker (``oracle/``) is test infrastructure and is imported here.
"""
import importlib.util
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_DIR = ROOT / "accelerating-moe-inference_b200"
ORACLE_DIR = ROOT / "oracle"
GOLDEN_DIR = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built CUDA library")


def load_pkg():
    name = "moe_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, PKG_DIR / "__init__.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def load_oracle():
    if str(ORACLE_DIR) not in sys.path:
        sys.path.insert(0, str(ORACLE_DIR))
    import oracle  # noqa: E402
    return oracle


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def ref_elementwise_failures(y, y_ref, tol=3e-3) -> int:
    """The reference's own validation rule (src/main.cpp:326-344): an element
    fails if abs > tol and rel > tol, or if it is NaN."""
    y = np.asarray(y, np.float64)
    y_ref = np.asarray(y_ref, np.float64)
    ad = np.abs(y - y_ref)
    rd = ad / np.maximum(np.abs(y_ref), 1e-30)
    return int(np.count_nonzero(((ad > tol) & (rd > tol)) | np.isnan(y)))


@pytest.fixture(scope="session")
def pkg():
    return load_pkg()


@pytest.fixture(scope="session")
def orc():
    o = load_oracle()
    return o.Oracle()
