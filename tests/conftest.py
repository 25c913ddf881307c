"""Shared fixtures.  GPU tests are marked ``gpu``; everything else runs on CPU."""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_package():
    """Import spaceslug-main_b200/ under the module name ``spaceslug_b200``."""
    if "spaceslug_b200" in sys.modules:
        return sys.modules["spaceslug_b200"]
    root = ROOT / "spaceslug-main_b200"
    spec = importlib.util.spec_from_file_location("spaceslug_b200", root / "__init__.py",
                                                  submodule_search_locations=[str(root)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["spaceslug_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


load_package()


@pytest.fixture(scope="session")
def pkg():
    return load_package()


@pytest.fixture(scope="session")
def built_library(pkg):
    from spaceslug_b200 import build
    return build.build()


@pytest.fixture(scope="session")
def session(built_library):
    from spaceslug_b200.backend import BackendSession
    return BackendSession(built_library)


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def golden():
    return {name: np.load(GOLDEN / f"{name}.npz") for name in ("ref_generators", "ref_q4gemm_256", "cfg_tiny")}


@pytest.fixture(scope="session")
def golden_rows():
    """Reference outputs on sampled rows of BASELINE configs[2]-[4] (make_config_rows.py)."""
    return dict(np.load(GOLDEN / "cfg_rows.npz"))


def cuda_ok() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


@pytest.fixture(scope="session")
def cuda(session):
    if not cuda_ok():
        pytest.fail("a gpu-marked test ran without a CUDA device")
    import torch
    torch.cuda.init()
    return torch.device("cuda:0")
