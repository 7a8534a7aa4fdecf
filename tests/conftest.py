import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")
REF_TREE = os.environ.get("LLMVHDL_REF", "/root/reference")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA path)")


def load_package():
    """Register llm.vhdl_b200/ (a directory name with a dot) as module llmvhdl_b200."""
    if "llmvhdl_b200" in sys.modules:
        return sys.modules["llmvhdl_b200"]
    pkg = os.path.join(ROOT, "llm.vhdl_b200")
    spec = importlib.util.spec_from_file_location(
        "llmvhdl_b200", os.path.join(pkg, "__init__.py"), submodule_search_locations=[pkg])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["llmvhdl_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def pkg():
    return load_package()


@pytest.fixture(scope="session")
def synth(pkg):
    import llmvhdl_b200.synth as S
    return S


@pytest.fixture(scope="session")
def golden():
    return np.load(os.path.join(GOLDEN, "mv4i_golden.npz"))


@pytest.fixture(scope="session")
def ref_tree():
    if not os.path.isdir(os.path.join(REF_TREE, "sim")):
        pytest.skip("llm.vhdl reference tree not present")
    return REF_TREE


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    torch.cuda.init()
    return torch
