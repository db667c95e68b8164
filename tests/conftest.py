"""Test configuration: puts the package directory on sys.path and registers markers.

`-m "not gpu"` runs everywhere (no CUDA device needed); `-m gpu` needs a B200.
"""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
for entry in (ROOT / "laya-cuda_b200", ROOT):
    if str(entry) not in sys.path:
        sys.path.insert(0, str(entry))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and the built library")
    config.addinivalue_line("markers", "slow: long-running CPU test")
