import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "hnsw-vector-db_b200")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU (run with -m gpu)")


def _make(args):
    subprocess.run(["make", "-s", "-j8"] + args, check=True)


@pytest.fixture(scope="session", autouse=True)
def built_libraries():
    """Builds the checkers and the GPU library in place when they are missing."""
    import oracle
    if not os.path.exists(oracle.ORACLE_LIB) or (
            not os.path.exists(oracle.REF_LIB) and os.path.isdir(os.path.join(oracle.REFERENCE_SRC, "src"))):
        oracle.build(ref=True)
    if not (os.path.exists(os.path.join(PKG, "lib", "libvdbgpu.so"))
            and os.path.exists(os.path.join(PKG, "lib", "libvdbsynth.so"))):
        _make(["-C", PKG])
    if not os.path.exists(oracle.REF_GPUINDEX_LIB) and os.path.isdir(os.path.join(oracle.REFERENCE_SRC, "src")):
        oracle.build(ref=True)
    yield


def golden(name):
    return dict(np.load(os.path.join(GOLDEN, name + ".npz"), allow_pickle=False))


@pytest.fixture(scope="session")
def ctx():
    import vdb_b200
    return vdb_b200.Context(0)
