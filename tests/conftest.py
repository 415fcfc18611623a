from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
GOLDEN = REPO / "tests" / "golden"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built native library")


def load_golden(name: str) -> tuple[dict, dict]:
    """Returns (meta, arrays) of tests/golden/<name>.npz."""
    with np.load(GOLDEN / f"{name}.npz", allow_pickle=False) as z:
        arrays = {k: z[k] for k in z.files if k != "meta"}
        meta = json.loads(str(z["meta"]))
    return meta, arrays


def checksum(*tensors) -> np.ndarray:
    return np.array([float(t.double().sum()) for t in tensors] + [float(t.double().abs().sum()) for t in tensors])


def bf16_tolerance_check(out, ref, max_abs: float = 2e-2, mean_abs: float = 2e-3) -> None:
    """The north-star bar for 16-bit outputs: max-abs <= 2e-2 and mean-abs <= 2e-3
    against an fp32 (here fp64) reference."""
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert out.shape == ref.shape, (out.shape, ref.shape)
    assert np.isfinite(out).all(), "non-finite values in the output"
    err = np.abs(out - ref)
    assert err.max() <= max_abs, f"max-abs error {err.max():.3e} > {max_abs}"
    assert err.mean() <= mean_abs, f"mean-abs error {err.mean():.3e} > {mean_abs}"


@pytest.fixture(scope="session")
def native_lib():
    """The built library (builds it if missing: nvcc cross-compiles without a GPU)."""
    from aicas_b200 import _native
    from aicas_b200.build import build

    if not _native.library_path().exists():
        build()
    return _native.lib()


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    major, minor = torch.cuda.get_device_capability(0)
    if major != 10:
        pytest.skip(f"sm_100 device required (found sm_{major}{minor})")
    from aicas_b200 import _native

    _native.lib()  # the GPU tests must run the native path: fail loudly if it is missing
    return torch.device("cuda", 0)
