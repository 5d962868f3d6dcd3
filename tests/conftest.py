import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


def load_samrs():
    """The product package lives in the directory `sam-rs_b200` (not an identifier), so import it by name."""
    return importlib.import_module("sam-rs_b200")


@pytest.fixture(scope="session")
def samrs():
    return load_samrs()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def pytest_terminal_summary(terminalreporter):
    """Worst parity numbers per I/O dtype over the run: the plain max|got-ref|/max|ref| and the error beyond
    half an ulp of the I/O dtype (the f16/bf16 bar), with the test each came from."""
    from tests.helpers import PARITY_LOG
    if not PARITY_LOG:
        return
    tr = terminalreporter
    tr.write_line("parity vs the CPU oracle (worst case per I/O dtype; bar 1e-4 f32, 3e-3 f16/bf16 beyond half an ulp):")
    for dt in ("f32", "f16", "bf16"):
        rows = [r for r in PARITY_LOG if r[1] == dt]
        if not rows:
            continue
        wp = max(rows, key=lambda r: r[2])
        we = max(rows, key=lambda r: r[3])
        tr.write_line(f"  {dt:4s} {len(rows):3d} checks: plain max|got-ref|/max|ref| {wp[2]:.2e} "
                      f"({wp[0].split('::')[-1][:48]}); beyond half an ulp {we[3]:.2e}")
