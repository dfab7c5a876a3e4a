import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def pkg():
    import __graft_entry__

    return __graft_entry__.load_package()


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle

    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def cuda_dev():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a visible CUDA device")
    return torch.device("cuda:0")


def state_rel_err(got, ref) -> float:
    """Norm-wise relative error max|got-ref| / max|ref| (the 1e-3 state bar)."""
    ref = ref.float().cpu()
    denom = ref.abs().max().item()
    return (got.float().cpu() - ref).abs().max().item() / (denom if denom > 0 else 1.0)
