"""The C-ABI library loads and exports every symbol include/*.h declares, and
its argument validation rejects bad calls before touching a GPU.  CPU only."""
import ctypes
import re
from pathlib import Path

import pytest

from conftest import ROOT

import rdna2_ops._native as nat

EINVAL = 1  # cudaErrorInvalidValue


def _declared_symbols():
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        names.update(re.findall(r"\b(b2_[a-z0-9_]+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    lib = nat.library()
    declared = _declared_symbols()
    assert declared, "no declarations found"
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_header():
    assert _declared_symbols() <= set(nat.SIGNATURES)


def test_version_and_error_strings():
    lib = nat.library()
    assert lib.b2_version() >= 1
    assert b"invalid argument" in lib.b2_error_string(EINVAL)


def _qgemm(**kw):
    args = dict(kind=0, a=16, lda=16, b=16, ldb=16, M=4, N=4, K=16, a_scale=16, b_scale=16,
                b_scale_count=4, bias=None, bias_dtype=0, epilogue=0, out=16, out_dtype=0,
                ldc=4, stream=None)
    args.update(kw)
    return nat.library().b2_qgemm(*args.values())


@pytest.mark.parametrize("bad", [
    dict(kind=7), dict(K=0), dict(K=131072), dict(lda=8), dict(ldb=24), dict(a=24),
    dict(ldc=3), dict(epilogue=9), dict(epilogue=3, out_dtype=0), dict(out_dtype=5),
    dict(b_scale_count=3), dict(a_scale=None), dict(M=-1), dict(bias=16, bias_dtype=4),
])
def test_qgemm_rejects_bad_arguments(bad):
    assert _qgemm(**bad) == EINVAL


def test_qgemm_empty_is_noop():
    assert _qgemm(M=0) == 0 and _qgemm(N=0) == 0


def test_act_quant_rejects_bad_arguments():
    lib = nat.library()
    ok = dict(x=16, dt=1, M=2, K=256, ldx=256, block=128, quant=0, q=16, ldq=256, s=16, st=None)
    for bad in (dict(block=96), dict(block=512), dict(dt=3), dict(dt=6), dict(quant=3), dict(ldx=100),
                dict(K=20000), dict(x=None)):
        a = dict(ok, **bad)
        assert lib.b2_act_quant(*a.values()) == EINVAL, bad


def test_quant_linear_workspace_and_validation():
    lib = nat.library()
    assert lib.b2_quant_linear_workspace_bytes(4096, 3072) >= 4096 * 3072 + 4096 * 4
    assert lib.b2_quant_linear_workspace_bytes(0, 16) == 0
    # misaligned workspace / too small / bad kind all fail before any launch
    base = [0, 16, 1, 4, 64, 64, 0, 16, 64, 8, 16, 8, None, 0, 0, 16, 1, 8]
    assert lib.b2_quant_linear(*base, 16, 10**6, None) == EINVAL          # not 256-aligned
    assert lib.b2_quant_linear(*base, 256, 8, None) == EINVAL             # too small
    assert lib.b2_quant_linear(2, *base[1:], 256, 10**6, None) == EINVAL  # bf16 kind


def test_repack_rejects_bad_arguments():
    lib = nat.library()
    assert lib.b2_repack(16, 4, 2, 2, 2, 1, 16, 2, None) == EINVAL
    assert lib.b2_repack(16, 1, 2, 4, 4, 1, 16, 2, None) == EINVAL
    assert lib.b2_repack(16, 1, 0, 4, 4, 1, 16, 16, None) == 0


def test_operators_refuse_cpu_tensors():
    torch = pytest.importorskip("torch")
    import rdna2_ops
    a = torch.zeros(4, 4, dtype=torch.int8)
    with pytest.raises(ValueError):
        rdna2_ops.int8_matmul(a, a)
    with pytest.raises(ValueError):
        rdna2_ops.act_quant(torch.zeros(2, 16))
