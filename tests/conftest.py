import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

# The C oracle's faster traversals (register-tiled GEMM, attention over all
# host threads): the same operation sequence per output element as the
# reference's (tests/test_oracle_ops.py checks bit equality); the timed CPU
# baseline in bench.py keeps the reference's own traversal.
os.environ.setdefault("LAYA_ORACLE_FAST", "1")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")
