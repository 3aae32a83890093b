"""Shared test setup: import paths, the `gpu` marker, seeded input builders."""
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "rdna2-gfx1030-ai-handbook_b200"
GOLDEN = Path(__file__).resolve().parent / "golden"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and the CUDA library")


@pytest.fixture(scope="session")
def golden():
    return lambda name: np.load(GOLDEN / name)


def outlier_activations(rng, m, k, frac=0.01, gain=20.0):
    """N(0,1) activations with a fixed 1% of channels scaled x20 (BASELINE C1/C2)."""
    x = rng.standard_normal((m, k), dtype=np.float32)
    idx = rng.choice(k, size=max(1, int(round(frac * k))), replace=False)
    x[:, idx] *= gain
    return x
