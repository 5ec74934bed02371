import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "sana.cpp_b200"), os.path.join(ROOT, "oracle"), os.path.dirname(__file__)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def reference_root() -> str:
    """The reference tree: SANA_REFERENCE_ROOT, else BASELINE.json's reference_path."""
    root = os.environ.get("SANA_REFERENCE_ROOT")
    if root:
        return root
    try:
        import json
        with open(os.path.join(ROOT, "BASELINE.json")) as f:
            return json.load(f).get("reference_path", "")
    except (OSError, ValueError):
        return ""


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the CUDA path through the C ABI")
    config.addinivalue_line("markers", "slow: long-running CPU check")


@pytest.fixture(scope="session")
def oracle():
    from oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle import Reference
    if not Reference.available():
        pytest.skip("reference build (oracle/_ref) not present")
    return Reference()
