"""Test configuration: marker registration, import paths, on-demand builds.

CPU tests (``-m "not gpu"``) cover the oracle against the reference's golden
vectors, the host logic and the C ABI surface. GPU tests (``-m gpu``) are the
parity tests of the CUDA path through the C ABI.
"""
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "astc-kv_b200", ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session", autouse=True)
def _built():
    """Build the oracle, the host emulator and (if stale) the CUDA library."""
    subprocess.run(["make", "-s", "-C", str(ROOT / "oracle")], check=True)
    subprocess.run(["make", "-s", "-C", str(ROOT / "tests" / "emu")], check=True)
    from astc_kv_cuda import build
    if build._stale():
        if os.environ.get("AKV_NO_BUILD"):
            pytest.exit("libakv_cuda.so is stale or missing and AKV_NO_BUILD is set", returncode=3)
        build.build()
    yield


def gpu_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


@pytest.fixture
def cuda():
    if not gpu_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    import torch
    return torch.device("cuda:0")
