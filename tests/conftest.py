"""Shared test setup: import paths, the ``gpu`` marker, fixture locations."""
import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(REPO / "emmy-hackathon-2026_b200"))
sys.path.insert(0, str(REPO))

GOLDEN = REPO / "tests" / "golden"
PROBLEMS = sorted(p for p in (GOLDEN / "problems").iterdir() if p.is_dir())
FIXTURES = sorted(p for p in (GOLDEN / "fixtures").iterdir() if p.is_dir())
# the reference checkout (only the tests that regenerate or compare against it
# use it): EMMY_REFERENCE_ROOT, else a "reference" folder beside this repository
REFERENCE = Path(os.environ.get("EMMY_REFERENCE_ROOT") or REPO.parent / "reference")
# every launch the tests make through harness.run gets 64 KiB guard regions
# around each buffer and fails on a byte written out of place (an output's
# neighbourhood or an input): the memory-safety check in place of
# compute-sanitizer, which is closed on the GPU pool
os.environ.setdefault("EMMY_GUARD_BYTES", str(64 * 1024))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def native_lib():
    from emmy_b200 import native
    native.build()
    return native.lib()


def gpu_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
