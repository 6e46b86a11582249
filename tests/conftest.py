"""Shared fixtures.  The package directory is named ``mlip.cpp_b200`` (not an
importable identifier), so it is loaded here under the module name
``mlipcpp_b200``."""
import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def load_package():
    if "mlipcpp_b200" in sys.modules:
        return sys.modules["mlipcpp_b200"]
    pkg_dir = os.path.join(ROOT, "mlip.cpp_b200")
    spec = importlib.util.spec_from_file_location(
        "mlipcpp_b200", os.path.join(pkg_dir, "__init__.py"), submodule_search_locations=[pkg_dir])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["mlipcpp_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


load_package()
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (runs the sm_100a kernels)")


@pytest.fixture(scope="session")
def gguf_dir(tmp_path_factory):
    return tmp_path_factory.mktemp("gguf")


@pytest.fixture(scope="session")
def model_file(gguf_dir):
    """model_file(name, seed, nc=False, **hypers) -> path of a seeded
    random-init "pet" GGUF (nc: non-conservative heads, see
    workloads.random_pet_weights)."""
    from mlipcpp_b200 import workloads as wl
    cache = {}

    def make(name="tiny", seed=0, nc=False, **over):
        key = (name, seed, repr(nc), tuple(sorted(over.items())))
        if key not in cache:
            import dataclasses
            h = dataclasses.replace(wl.HYPERS[name], **over)
            path = os.path.join(str(gguf_dir), f"{name}_{seed}_{len(cache)}.gguf")
            wl.write_pet_gguf(path, h, seed=seed, nc_heads=nc)
            cache[key] = path
        return cache[key]
    return make


def nl_equal(a, b):
    """Bitwise equality of two NeighborList dicts; returns the first
    differing field or None."""
    for k in ("centers", "neighbors", "cell_shifts", "edge_vectors", "distances"):
        x, y = np.asarray(a[k]), np.asarray(b[k])
        if x.shape != y.shape:
            return k + " (shape)"
        if x.dtype == np.float32:
            x, y = x.view(np.uint32), y.view(np.uint32)
        if not np.array_equal(x, y):
            return k
    return None
