import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def load_pkg():
    """Imports the package directory sam3.cpp_b200/ as module `sam3_b200`."""
    name = "sam3_b200"
    if name in sys.modules:
        return sys.modules[name]
    pkg = os.path.join(ROOT, "sam3.cpp_b200")
    spec = importlib.util.spec_from_file_location(name, os.path.join(pkg, "__init__.py"),
                                                  submodule_search_locations=[pkg])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def s3b():
    return load_pkg()


@pytest.fixture(scope="session")
def engine(s3b):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()
    e = s3b.Engine(0)
    # run the engine on torch's stream so inputs made by torch are ready and
    # in-place outputs are not raced by torch's own reference computations
    e.set_stream(torch.cuda.current_stream().cuda_stream)
    yield e
    e.set_stream(None)
    e.close()
