import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
for p in (REPO, REPO / "mlx-cross-entropy_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    # GPU tests are never skipped: without an sm_100 device they fail.
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) CUDA device")
