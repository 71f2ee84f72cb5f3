"""Shared fixtures: the product library (through its ctypes host mirror) and
the oracle. GPU tests are marked ``gpu``; everything else runs on CPU."""
import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

PKG_DIR = os.path.join(ROOT, "i.sam3.opencl_b200")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")


def load_product():
    """Import i.sam3.opencl_b200/sam3_b200.py (the directory name is not a
    Python identifier, so it is loaded by path)."""
    name = "sam3_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(PKG_DIR, "sam3_b200.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def sb():
    return load_product()


@pytest.fixture(scope="session")
def ob():
    from oracle import binding
    return binding


@pytest.fixture(scope="session")
def cb(sb):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    be = sb.Backend(0)
    yield be
    be.sync()
    be.close()
