import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; run with -m gpu")
    config.addinivalue_line("markers", "slow: full-size (8192^3 and larger) parity cases")


def _cuda_ok() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_ok():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this container (GPU tests run under -m gpu on a B200)")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def zx():
    """The product library, built in-tree; GPU tests fail (not skip) if it cannot load."""
    from zoxide_b200 import build as _b

    _b.build()
    import zoxide_b200

    zoxide_b200.lib()
    return zoxide_b200


@pytest.fixture(scope="session")
def zxo():
    import oracle

    oracle.build()
    return oracle


@pytest.fixture(params=[1, 2, 3, 4, 5, 6], ids=["1sm", "2sm", "2sm256", "2sm512", "2sm480", "2sm464"])
def policy(request, zx):
    """Run a GPU case on every tile path: one-SM 128x256 tiles, two-SM CTA pairs with the
    automatic tile width (256 or 224), two-SM pairs forced to 256-wide tiles, and two-SM pairs
    with 256 x 512, 256 x 480 and 256 x 464 tiles (K-major B; the MN-major layout falls back to
    the 256-wide pair path)."""
    zx.set_kernel_policy(request.param)
    yield request.param
    zx.set_kernel_policy(0)
