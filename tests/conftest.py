import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    # Build the oracle (and, where the reference sources exist, its compiled
    # reference twin) and the CUDA library if they are missing; both builds
    # are incremental.
    from oracle import oracle as oracle_lib

    if not oracle_lib.available():
        oracle_lib.build(ref=True)
    from distributed_graph_flow_b200 import build as dgfx_build

    if not (ROOT / "distributed_graph_flow_b200" / "libdgfx.so").exists():
        dgfx_build.build()


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch
