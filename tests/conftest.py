import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs 2+ GPUs")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from lumenrl_b200.ops.ext import ext
    ext()  # fail loudly if the extension is missing on a GPU box
    if os.environ.get("LRL_SEGV_BACKTRACE"):    # a file path for the native stack on SIGSEGV
        ext().install_segv_backtrace(os.environ["LRL_SEGV_BACKTRACE"])
    return torch.device("cuda", 0)
