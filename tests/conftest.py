import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def reference_root() -> Path | None:
    """The reference checkout named by KS_REFERENCE_ROOT, or None when the
    variable is unset or names no directory (tests that need the
    reference's own files then skip)."""
    v = os.environ.get("KS_REFERENCE_ROOT")
    if not v or not Path(v).is_dir():
        return None
    return Path(v)


def reference_file(rel: str) -> Path:
    """A file of the reference checkout; skips the calling test when the
    checkout (KS_REFERENCE_ROOT) or the file is absent."""
    root = reference_root()
    if root is None:
        pytest.skip("set KS_REFERENCE_ROOT to the reference checkout to run this test")
    f = root / rel
    if not f.exists():
        pytest.skip(f"{rel} not in the reference checkout")
    return f
