import os
import subprocess
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, HERE)
sys.path.insert(0, ROOT)
GOLDEN = os.path.join(HERE, "golden")
# the DRANZER source tree the checker builds from, where it is present
REF_TREE = os.environ.get("DRANZER_REF", "/root/reference")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA path through the C ABI)")


@pytest.fixture(scope="session")
def oracle():
    from _native_oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def dz():
    """The product package, built in-tree if its library is missing."""
    import dranzer_b200
    from dranzer_b200 import _native
    if not os.path.exists(_native.LIB_PATH):
        from dranzer_b200 import build
        build.build()
    _native.lib()
    return dranzer_b200


@pytest.fixture(scope="session")
def gpu(dz):
    if not dz.available():
        pytest.fail("no usable B200: the gpu-marked tests need one (there is no CPU fallback)")
    return dz


def golden(name):
    return np.load(os.path.join(GOLDEN, name), allow_pickle=False)


@pytest.fixture(scope="session")
def ref():
    from _native_oracle import REF_SO, RefHarness
    if not os.path.exists(REF_SO):
        if os.path.isdir(os.path.join(REF_TREE, "src")):
            subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "ref", f"REF={REF_TREE}"], check=True)
        else:
            pytest.skip("reference build not present (tests/golden pins the oracle instead)")
    return RefHarness()


@pytest.fixture(scope="session")
def bridge(dz):
    """The reference's objects with the reference-side binding of the device
    path linked in (oracle/dz_bridge.c, oracle/_ref/libdzref_bridge.so)."""
    from _native_oracle import BRIDGE_SO, RefHarness
    if not os.path.exists(BRIDGE_SO):
        if os.path.isdir(os.path.join(REF_TREE, "src")):
            subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "ref", "bridge", f"REF={REF_TREE}"],
                           check=True)
        else:
            pytest.skip("reference build not present")
    return RefHarness(BRIDGE_SO)
