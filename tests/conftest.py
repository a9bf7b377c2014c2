import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests", "golden"),
                os.path.join(ROOT, "tests"), os.path.join(ROOT, "bitmamba.c_b200", "python")]


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a)")


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle
    oracle.build(ref=False)
    return oracle


@pytest.fixture(scope="session")
def sampler_lib():
    """The product library; built here when missing (nvcc cross-compiles)."""
    import bmsampler
    if not os.path.exists(bmsampler.LIB_PATH):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "bitmamba.c_b200")], check=True)
    return bmsampler


@pytest.fixture(scope="session")
def gpu_ctx(sampler_lib):
    ctx = sampler_lib.Context(0)
    yield ctx
    ctx.close()
