import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def ref_modules():
    """The reference's own C++ built from source (oracle/_ref); skip when absent."""
    ref_dir = ROOT / "oracle" / "_ref"
    if not any(ref_dir.glob("imi_ref*.so")):
        pytest.skip("oracle/_ref not built (needs the reference checkout)")
    sys.path.insert(0, str(ref_dir))
    import imi_ref  # noqa: E402
    import AdpIMI_Index  # noqa: E402
    return imi_ref, AdpIMI_Index
