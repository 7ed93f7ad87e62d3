import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tiny-metal-nn_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")
    config.addinivalue_line("markers", "slow: long-running test")


def _ensure_ref():
    import ref_oracle
    if not ref_oracle.available("static"):
        try:
            import ref_build
            ref_build.build()
        except Exception as e:  # reference sources absent (GPU box)
            print("oracle/_ref unavailable:", e)


_ensure_ref()


@pytest.fixture(scope="session")
def ref():
    import ref_oracle
    if not ref_oracle.available("static"):
        pytest.skip("oracle/_ref (reference compiled here) not built")
    return ref_oracle
