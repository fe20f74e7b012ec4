"""pytest configuration: the `gpu` marker and import paths.

CPU tests (`-m "not gpu"`) cover the oracle against golden vectors, the host
logic and the C-ABI library's exports. GPU tests (`-m gpu`) are the parity
tests proper: CUDA path through the C ABI vs the oracle.
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "ssd-llm_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "tc_only: a case run on the tensor-core kernel only")
