"""pytest plugin for the child run of tests/test_gpu_reference_suite.py:
seeds torch's generators once at session start, so the reference's test
files, which draw unseeded torch.randn inputs (torch seeds itself randomly
per process), see the same inputs on every run.  The files themselves are
not changed.  Test infrastructure only."""
import torch


def pytest_sessionstart(session):
    torch.manual_seed(0)
