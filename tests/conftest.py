import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: full-size workloads")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


def golden_cases():
    """The loss fixtures (the sampler's, norm's and attention's are read by their own tests)."""
    return sorted(p.stem for p in GOLDEN.glob("*.npz")
                  if p.stem != "sample_token" and not p.stem.startswith(("norm_", "attn_")))
