import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "siliceo-motor_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


def pytest_sessionstart(session):
    # The oracle is plain C++ and cheap to build; the engine library is built
    # by __graft_entry__.build() (nvcc), and must already exist.
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle")], check=True)


def cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def tmpdir_session(tmp_path_factory):
    return tmp_path_factory.mktemp("sm")


def preset_gguf(preset: int) -> str:
    """The seeded synthetic GGUF of a benchmark configuration, written once per
    machine into the cache directory bench.py uses (so the bench reuses it)."""
    import fcntl
    import tempfile

    import smotor
    d = os.environ.get("SM_CACHE_DIR", os.path.join(tempfile.gettempdir(), "smotor_cache"))
    os.makedirs(d, exist_ok=True)
    path = os.path.join(d, f"preset{preset}_seed0_v1.gguf")
    with open(path + ".lock", "w") as lk:
        fcntl.flock(lk, fcntl.LOCK_EX)
        if not os.path.exists(path):
            tmp = path + ".part"
            smotor.synth_write(smotor.synth_preset(preset), tmp)
            os.replace(tmp, path)
        fcntl.flock(lk, fcntl.LOCK_UN)
    return path
