import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; runs the CUDA path through the C ABI")


@pytest.fixture(scope="session")
def oracle():
    import oracle as orc
    orc.build()
    return orc


@pytest.fixture(scope="session")
def backend():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA")
    from ocelotl_b200.build import build
    build()
    from ocelotl_b200 import CudaKernelBackend
    return CudaKernelBackend(0)


def pytest_terminal_summary(terminalreporter):
    import json
    import os
    from tests.tolerance import RECORDED
    if not RECORDED:
        return
    terminalreporter.section("achieved parity errors (asserted metric first)")
    for name in sorted(RECORDED):
        terminalreporter.write_line(f"{name}: " + ", ".join(f"{k}={v:.3g}" for k, v in RECORDED[name].items()))
    path = os.environ.get("OCL_PARITY_LOG")
    if path:
        with open(path, "w") as f:
            json.dump(RECORDED, f, indent=1, sort_keys=True)
