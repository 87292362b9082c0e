import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "solattn-amd_b200", ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))



def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: requires an NVIDIA B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: large-configuration parity case")


def pytest_collection_modifyitems(config, items):
    import torch
    has_gpu = torch.cuda.is_available() and torch.cuda.get_device_capability(0) == (10, 0)
    skip = pytest.mark.skip(reason="NVIDIA B200 (sm_100a) GPU required")
    for item in items:
        if "gpu" in item.keywords and not has_gpu:
            item.add_marker(skip)
