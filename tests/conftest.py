import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")
    config.addinivalue_line("markers", "multigpu: needs two or more CUDA devices")
    config.addinivalue_line("markers", "slow: full-size configuration, minutes of CPU oracle time")
    config.addinivalue_line("markers", "cpu: runs without a GPU (oracle, host logic, C-ABI surface)")


@pytest.fixture(scope="session")
def ncm():
    import nanocamelid_b200 as n
    n.lib()
    return n


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle as o
    o.lib()
    return o


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    return torch


# Small llama shape used by the parity tests (fast on the CPU oracle).
TINY = dict(emb=256, layers=2, heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=1024, ctx=128)
