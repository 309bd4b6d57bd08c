import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a) and the built extension")


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    """Print the parity record of the GPU tests (exact-token rates, near-tie
    slack, state differences), which passing tests would otherwise hide."""
    from tests.gpu_helpers import PARITY_LOG

    if not PARITY_LOG:
        return
    terminalreporter.section("parity record (GPU vs oracle / reference)")
    for line in PARITY_LOG:
        terminalreporter.write_line(line)
