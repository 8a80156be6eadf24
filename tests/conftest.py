import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

# The C oracle's attention over all host threads: the same arithmetic per
# output element as the reference's single thread (tests/test_oracle_ops.py
# checks bit equality), which the timed CPU baseline in bench.py keeps.
os.environ.setdefault("LAYA_ORACLE_THREADED_ATTENTION", "1")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")
