"""Shared test set-up: the `gpu` marker, the package (loaded by path: its directory name has dots) and the oracle."""
import importlib.util
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
PKG_DIR = ROOT / "llama3.x.c_b200"


def load_package():
    if "llama3x_b200" in sys.modules:
        return sys.modules["llama3x_b200"]
    spec = importlib.util.spec_from_file_location("llama3x_b200", PKG_DIR / "__init__.py",
                                                  submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["llama3x_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def load_engine():
    """The engine mirror, llama3.x.c_b200/engine.py, as llama3x_b200.engine."""
    load_package()
    return importlib.import_module("llama3x_b200.engine")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def kc():
    """The sm_100a library, initialised on cuda:0 (GPU tests only)."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("a gpu-marked test ran without a GPU")
    mod = load_package()
    torch.cuda.set_device(0)
    mod.init()
    return mod


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.lib()
    return O
