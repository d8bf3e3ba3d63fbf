"""Shared fixtures.  GPU tests are marked `gpu`; everything else runs on CPU."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def golden(name: str) -> str:
    return os.path.join(GOLDEN, name)


@pytest.fixture(scope="session")
def oracle():
    """The C restatement of the reference decode path (built on demand)."""
    subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "oracle"], check=True,
                   stdout=subprocess.DEVNULL)
    import oracle as O
    return O.Oracle()


@pytest.fixture(scope="session")
def reference():
    """The reference library built from its own sources (skips when absent)."""
    import oracle as O
    if not O.Reference.available():
        pytest.skip("oracle/_ref/libslate_ref.so not built (reference tree unavailable)")
    return O.Reference()


@pytest.fixture(scope="session")
def sb():
    """The product library binding (fails loudly if the .so is missing)."""
    import slate_b200
    return slate_b200


@pytest.fixture(scope="session")
def workdir(tmp_path_factory):
    return tmp_path_factory.mktemp("slate_b200")
