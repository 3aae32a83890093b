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


# ---------------------------------------------------------------- 1-ULP rule
# Float outputs of the fp32-accumulating paths (W4A16, FP8, the dense 16-bit
# GEMM) are held to one unit in the last place of the output type, plus the
# error that fp32 accumulation itself may add: GAMMA_FP32 * sum_k |a_k * w_k|.
# GAMMA_FP32 = 2^-20 is sixteen fp32 roundings (u = 2^-24).  Products are
# exact in fp32 on these paths; only the sums round.  The full-output census of
# the B200 kernels measured at most 2^-22 * sum|a*w| (W4A16 at M = 2048), and
# the reference's own PyTorch CPU math needs the same term: no fp32
# accumulation keeps a near-zero output (|y| << sum|a*w|) inside one bare ulp.
# For a typical output (sum|a*w| / |y| ~ 40 at config 3) the term is 1/100 ulp.
GAMMA_FP32 = 2.0 ** -20
_PRECISION = {"bf16": (8, -126), "fp16": (11, -14), "fp32": (24, -126)}


def ulp_of(v, kind):
    """Spacing of the floating type `kind` ("bf16", "fp16", "fp32") at |v|
    (the subnormal spacing below the smallest normal)."""
    p, emin = _PRECISION[kind]
    e = np.floor(np.log2(np.maximum(np.abs(np.asarray(v, np.float64)), 2.0 ** emin)))
    return 2.0 ** (e - (p - 1))


def assert_within_ulp(got, ref, abs_products, kind, what=""):
    """|got - ref| <= ulp(got) + GAMMA_FP32 * abs_products, element-wise, with
    ref the f64 value of the same math and abs_products = sum |a*w| (scaled
    like ref).  Reports the worst offenders on failure."""
    got = np.asarray(got, np.float64)
    err = np.abs(got - ref)
    tol = ulp_of(got, kind) + GAMMA_FP32 * abs_products
    bad = err > tol
    if bad.any():
        idx = np.argsort((err - tol).ravel())[-3:]
        raise AssertionError(
            f"{what}: {int(bad.sum())} of {bad.size} outputs outside 1 ulp + 2^-20 sum|a*w|; worst "
            + "; ".join(f"got {got.ravel()[i]!r} ref {ref.ravel()[i]!r} sum|aw| {abs_products.ravel()[i]!r}"
                        for i in idx))
