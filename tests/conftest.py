import sys
from pathlib import Path

import pytest

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
sys.path.insert(0, str(Path(__file__).resolve().parent))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (run with -m gpu on the GPU box)")
    config.addinivalue_line("markers", "slow: long-running (full 7B-size parity)")


@pytest.fixture(scope="session")
def cuda_ok():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return True


def pytest_terminal_summary(terminalreporter):
    """How many engine epochs were compared with the oracle, and every
    permitted near-tie divergence among them (row: step)."""
    try:
        from scenario import EPOCH_LOG
    except ImportError:
        return
    if not EPOCH_LOG:
        return
    rows = sum(entry[1] for entry in EPOCH_LOG)
    near = sum(entry[3] for entry in EPOCH_LOG)
    diverged = [(entry[0], entry[2]) for entry in EPOCH_LOG if entry[2]]
    count = sum(len(d) for _, d in diverged)
    terminalreporter.write_line(
        f"oracle parity: {len(EPOCH_LOG)} epochs, {rows} active rows compared, {near} near-tie row-steps "
        f"(oracle top-2 margin < 2e-2), {count} permitted near-tie divergence(s)"
        + (f": {diverged}" if diverged else ""))
