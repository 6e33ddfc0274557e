# SPDX-License-Identifier: MIT
import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "qwen.haiku_b200")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def load_pkg():
    """Import the package from its dotted directory name as `qwen_haiku_b200`."""
    name = "qwen_haiku_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(
        name, os.path.join(PKG_DIR, "__init__.py"), submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def qh():
    return load_pkg()


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def ref():
    from oracle.oracle import Ref
    if not Ref.available():
        pytest.skip("oracle/_ref/libqhref.so not built (reference sources absent)")
    return Ref()


@pytest.fixture(scope="session")
def cuda(qh):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch
