import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))
sys.path.insert(0, str(Path(__file__).resolve().parents[1]))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running full-size case")

# The package directory (swin2sr-rs_b200) is not an identifier: register it as
# swin2sr_b200 once, so a test may import its submodules in any order.
from s2s_testlib import pkg  # noqa: E402

pkg()
