"""Shared test set-up.

Markers: `gpu` (needs a CUDA device; the parity tests proper, calling the C-ABI library through
flash_lab) and `slow`. Without a CUDA device the gpu tests are skipped, as in the reference's own
conftest (tests/conftest.py:13-19 of tfan2437/flash-attention-lab).
"""

import os
import pathlib
import sys

import pytest
import torch

ROOT = pathlib.Path(__file__).resolve().parents[1]
PACKAGE_DIR = ROOT / "flash-attention-lab_b200"
for path in (str(ROOT), str(PACKAGE_DIR)):
    if path not in sys.path:
        sys.path.insert(0, path)

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs the sm_100a kernels)")
    config.addinivalue_line("markers", "slow: long-running case")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip_gpu = pytest.mark.skip(reason="needs a CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip_gpu)


@pytest.fixture(autouse=True)
def _seed():
    torch.manual_seed(0)


@pytest.fixture(autouse=True, scope="session")
def _no_tf32():
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False


@pytest.fixture(scope="session")
def flash_ops():
    """torch.ops.flash_lab, failing loudly if a GPU is present but the library did not load."""
    from flash_lab import ops

    if not ops.HAS_EXTENSION:
        pytest.fail(f"CUDA is available but the sm_100a library did not load: "
                    f"{ops.EXTENSION_ERROR}")
    return torch.ops.flash_lab


os.environ.setdefault("FLASH_LAB_STRICT", "1")
