import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
TESTS = os.path.dirname(os.path.abspath(__file__))
if TESTS not in sys.path:
    sys.path.insert(0, TESTS)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: large shapes (seconds of CPU oracle time)")


def pytest_sessionstart(session):
    """A fresh checkout has no built library: compile the in-tree sm_100a
    library (the same nvcc recipe as __graft_entry__.build()) before the tests
    that load it.  Nothing here substitutes for it -- without nvcc and without
    the .so, the tests that need it fail."""
    from decode_opt_b200 import build as dg_build
    if os.path.exists(dg_build.LIB_PATH) or not os.path.exists(dg_build.nvcc()):
        return
    dg_build.build_library()
