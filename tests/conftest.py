"""pytest configuration: the `gpu` marker and the repo root on sys.path.

Tests marked `gpu` need a B200 and the built `lazykv_b200/liblkv_sm100.so`; everything else runs
on CPU. Run the CPU suite with `-m "not gpu"` and the parity suite with `-m gpu`.
"""

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a) and the built kernel library")
