"""Test configuration: the `gpu` marker and import paths.

CPU tests (`-m "not gpu"`) cover the oracle against the reference's golden
vectors, host-side logic and the C ABI's exported symbols. GPU tests
(`-m gpu`) are the parity tests proper: the CUDA path against the oracle and
the golden fixtures, through the C ABI.
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("", "vllm-lite_b200", os.path.join("baseline", "_ref")):
    p = os.path.join(ROOT, sub)
    if os.path.isdir(p) and p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libvllt.so")


def have_vllmlite() -> bool:
    try:
        import vllmlite.engine  # noqa: F401
        return True
    except Exception:
        return False


needs_vllmlite = pytest.mark.skipif(not have_vllmlite(), reason="vllm-lite (the host engine) is not importable")


@pytest.fixture(scope="session")
def host_library(tmp_path_factory):
    """libvllt built for the host (tests/host_build.py), once per session;
    instrumented for ThreadSanitizer when VLLT_HOST_TSAN=1 (the race check of
    tests/test_race_check_host.py runs the host tests that way)."""
    from tests.host_build import build_library_host

    lib = build_library_host(str(tmp_path_factory.mktemp("libvllt_host")))
    if lib is None:
        pytest.skip("g++ is not available")
    return lib
