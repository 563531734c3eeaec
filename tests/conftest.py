import json
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and the built library")


def golden_names():
    return sorted(json.loads((GOLDEN / "index.json").read_text()))


def load_golden(name):
    """Golden case produced by the reference's own prepare() (tests/golden/make_golden.py)."""
    z = np.load(GOLDEN / f"{name}.npz")
    m, n, k, seed = (int(v) for v in z["mnk"])
    return {
        "m": m, "n": n, "k": k, "seed": seed,
        "a": torch.from_numpy(z["a"]).view(torch.float8_e4m3fn),
        "b": torch.from_numpy(z["b"]).view(torch.float8_e4m3fn),
        "sa": torch.from_numpy(z["sa"]),
        "packed_sa": torch.from_numpy(z["packed_sa"]),
        "sb": torch.from_numpy(z["sb"]),
        "reference": torch.from_numpy(z["reference"]).view(torch.bfloat16),
    }


def _nvidia_device_present() -> bool:
    return any(Path(p).exists() for p in ("/dev/nvidiactl", "/dev/nvidia0"))


@pytest.fixture(scope="session")
def cuda_device():
    if not torch.cuda.is_available():
        if _nvidia_device_present():  # a GPU machine whose CUDA does not work: fail, do not skip
            pytest.fail("an NVIDIA device is present but CUDA is unavailable to torch", pytrace=False)
        pytest.skip("no CUDA device")
    cap = torch.cuda.get_device_capability(0)
    if cap != (10, 0):
        pytest.skip(f"needs sm_100 (B200), found sm_{cap[0]}{cap[1]}")
    # the library must be built and load; there is no fallback
    from fack_b200 import _lib
    _lib.load()
    return torch.device("cuda", 0)
