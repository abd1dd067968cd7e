"""Shared fixtures and markers.

Markers: ``gpu`` (needs a CUDA device with the sm_100a kernels) and ``slow``.
CPU tests cover the oracle against the golden vectors, the C++ ledger
against the oracle and the reference's known answers, and the C ABI surface.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: longer-running CPU test")


@pytest.fixture(scope="session", autouse=True)
def _native_library() -> None:
    """Build libpagedkv.so once if it is missing or stale (nvcc is available here)."""
    from pagedcore_b200 import build

    if not build.up_to_date() and os.environ.get("PKV_SKIP_BUILD") != "1":
        build.build()


@pytest.fixture(scope="session")
def rope_golden() -> np.ndarray:
    return np.load(GOLDEN / "rope_table.npz")["table"]


@pytest.fixture(scope="session")
def attention_golden() -> dict[str, np.ndarray]:
    with np.load(GOLDEN / "attention_cfg1.npz") as data:
        return {name: data[name] for name in data.files}


@pytest.fixture(scope="session")
def append_golden() -> dict:
    return json.loads((GOLDEN / "append_cfg2.json").read_text())


@pytest.fixture(scope="session")
def append_small_golden() -> dict[str, np.ndarray]:
    with np.load(GOLDEN / "append_small.npz") as data:
        return {name: data[name] for name in data.files}


SMALL_CASE = dict(seed=7, num_blocks=48, churn_count=200, prompt_count=3, decode_rows=8, max_prompt=64, churn_tokens=15)


def parity_report(test: str, **fields) -> None:
    """Append one JSON line of a parity test's measured margins to $PKV_PARITY_REPORT, if set.

    The assertions stay in the tests; this only records how close each case
    came to its bound (worst error over the tolerance, argmax flips, gaps).
    """
    path = os.environ.get("PKV_PARITY_REPORT")
    if not path:
        return
    with open(path, "a") as sink:
        sink.write(json.dumps({"test": test, **fields}) + "\n")


def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("requires a CUDA device")
    return torch.device("cuda:0")
