import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
REF = os.path.join(ROOT, "baseline", "_ref")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running test")


@pytest.fixture(scope="session")
def reference():
    """The unmodified reference package (installed under baseline/_ref), or skip."""
    if not os.path.isdir(os.path.join(REF, "nanospec")):
        pytest.skip("reference not installed in baseline/_ref")
    if REF not in sys.path:
        sys.path.append(REF)
    import nanospec.config
    import nanospec.distributed
    import nanospec.dspark
    import nanospec.objective
    import nanospec.ops
    import nanospec.shard
    import nanospec.train
    return nanospec
