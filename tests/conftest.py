"""pytest configuration: the `gpu` marker and import paths.

Tests marked ``gpu`` need a B200 (sm_100) and the in-tree libbfp200.so; the
rest run on any CPU.  Tests call the product through its C ABI (bfp200 over
ctypes) and check it against the oracle package and the committed golden
fixtures in tests/golden/.
"""
import os
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (REPO, os.path.join(REPO, "tinyllm-fpga_b200"), os.path.join(REPO, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built libbfp200.so")
