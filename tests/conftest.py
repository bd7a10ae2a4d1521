import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; runs the CUDA kernels through the C ABI")


@pytest.fixture(scope="session")
def nbl_ctx():
    """One nbl_ctx on cuda:0 for the whole GPU session (kernels on torch's current stream)."""
    import torch
    import nibble_b200 as nb
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    ctx = nb.Context(0)
    yield ctx
    ctx.close()


def pytest_sessionstart(session):
    """Builds what the tests load (cached by content stamps): the CPU oracle, and the CUDA library when nvcc
    is present. On a GPU box the in-tree .so files built elsewhere are used as they are."""
    import shutil
    import oracle
    if not os.path.exists(oracle.ORACLE_SO):
        oracle.build(with_ref=False)
    if shutil.which("nvcc") or os.path.exists("/usr/local/cuda/bin/nvcc"):
        from nibble_b200 import build as nb_build
        try:
            nb_build.build()
        except Exception as e:  # a stale/broken build must not hide behind an old .so
            raise pytest.UsageError(f"building libnibble_cuda.so failed: {e}")
