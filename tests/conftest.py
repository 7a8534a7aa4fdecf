import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")
# the llm.vhdl tree: $LLMVHDL_REF, else the directory `reference` beside this repository
REF_TREE = os.environ.get("LLMVHDL_REF") or os.path.normpath(os.path.join(ROOT, "..", "reference"))


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


class _DevArray:
    """A raw device allocation seen through __cuda_array_interface__."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(int(s) for s in shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 2, "strides": None}


_SIGNED = {np.dtype(np.uint16): np.int16, np.dtype(np.uint32): np.int32, np.dtype(np.uint64): np.int64}


def device_view(torch, ptr, shape, dtype):
    """A torch tensor aliasing `shape` elements of `dtype` at device address ptr
    (unsigned 16/32/64-bit are viewed as the signed type of the same width)."""
    dt = np.dtype(dtype)
    dt = np.dtype(_SIGNED.get(dt, dt))
    return torch.as_tensor(_DevArray(ptr, shape, dt.str), device="cuda")


def device_read(torch, ptr, shape, dtype):
    """Copy device memory at ptr into a new numpy array of `dtype`."""
    torch.cuda.synchronize()
    return device_view(torch, ptr, shape, dtype).cpu().numpy().view(np.dtype(dtype)).copy()


def split(n, world, rank, align=1):
    """Contiguous [start, start+count) of n items for `rank`, in units of
    `align` (the last ranks take the remainder): a row-parallel K-slice."""
    units = (n + align - 1) // align
    per, extra = units // world, units % world
    u0 = rank * per + min(rank, extra)
    u1 = u0 + per + (1 if rank < extra else 0)
    s, e = u0 * align, min(n, u1 * align)
    return s, max(0, e - s)

