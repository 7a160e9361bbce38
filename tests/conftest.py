import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built liboxg_b200.so")


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import oracle
    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def cuda_ctx():
    """One library context on cuda:0 for the whole GPU session (bound to torch's stream)."""
    import torch
    from oxidized_gpt_oss_b200 import abi
    from oxidized_gpt_oss_b200.mxfp4 import context
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return context(None)
