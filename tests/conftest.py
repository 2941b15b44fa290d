"""pytest configuration: the `gpu` marker selects the parity tests that need a B200."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (sm_100a); run with -m gpu")
    config.addinivalue_line("markers", "slow: CPU test that runs for more than ~20 s")
