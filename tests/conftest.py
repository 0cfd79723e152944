import os
import sys

import pytest

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import common  # noqa: E402,F401  (puts oracle/ and the package on sys.path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and libsi_b200.so")


@pytest.fixture(scope="session")
def oc():
    import oracle as oracle_mod
    oracle_mod.build()
    return oracle_mod.Oracle()


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    from common import GOLDEN
    return dict(np.load(os.path.join(GOLDEN, "reference_golden.npz")))


@pytest.fixture(scope="session")
def ref():
    """The reference's own kernels; only where the reference checkout was built."""
    import oracle as oracle_mod
    if not os.path.exists(oracle_mod.LIB_REF):
        pytest.skip("oracle/_ref not built (reference checkout absent)")
    return oracle_mod.Reference()


@pytest.fixture(scope="session")
def si_ctx():
    """A libsi_b200 context on cuda:0 (GPU tests only)."""
    import sib200
    ctx = sib200.Context(0, max_positions=32768, rope_theta=1e6, head_dim=128)
    yield ctx
    ctx.close()
