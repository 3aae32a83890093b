"""Install / verify / restore protocol of the Kitchen INT8 export replacement
(reference backend.py:148-204, comfy_int8.py:207-227) against a stand-in
comfy_kitchen.  CPU only: nothing here launches a kernel."""
import pytest

import fake_kitchen

torch = pytest.importorskip("torch")


@pytest.fixture()
def kitchen():
    k = fake_kitchen.install()
    yield k
    k.uninstall()


def _binding():
    from rdna2_ops.comfy_int8 import KitchenInt8Binding
    return KitchenInt8Binding()


def test_install_requires_accumulator_first(kitchen):
    b = _binding()
    mm = lambda a, w: None
    linear = lambda *a, **k: None
    with pytest.raises(RuntimeError, match="accumulator"):
        b.install_backend(mm, linear)
    kitchen.quant._int8_matmul_accumulate = mm
    b.install_backend(mm, linear)
    assert kitchen.eager.int8_linear is linear
    assert kitchen.registry.get_implementation("int8_linear", backend="eager") is linear
    b.install_backend(mm, linear)                       # idempotent with the same GEMM
    with pytest.raises(RuntimeError, match="different GEMM"):
        b.install_backend(lambda a, w: None, linear)
    b.disable_backend(linear)
    assert kitchen.eager.int8_linear is kitchen.quant.int8_linear
    b.disable_backend(linear)                           # no-op when not installed


def test_refuses_to_overwrite_foreign_patch(kitchen):
    b = _binding()
    mm = lambda a, w: None
    linear = lambda *a, **k: None
    kitchen.quant._int8_matmul_accumulate = mm
    b.install_backend(mm, linear)
    kitchen.eager.int8_linear = lambda *a, **k: "other"
    with pytest.raises(RuntimeError, match="changed"):
        b.disable_backend(linear)
    with pytest.raises(RuntimeError, match="changed"):
        b.install_backend(mm, linear)


def test_scoped_context_rejects_nesting(kitchen):
    b = _binding()
    mm = lambda a, w: None
    linear = lambda *a, **k: None
    kitchen.quant._int8_matmul_accumulate = mm
    with b.scoped(mm, linear):
        assert kitchen.eager.int8_linear is linear
        with pytest.raises(RuntimeError, match="Nested"):
            with b.scoped(mm, linear):
                pass
    assert kitchen.eager.int8_linear is kitchen.quant.int8_linear


def test_calling_before_install_raises():
    b = _binding()
    with pytest.raises(RuntimeError, match="Install"):
        b.int8_linear(torch.zeros(2, 16), torch.zeros(4, 16, dtype=torch.int8), torch.ones(4))


def test_stats_switch(monkeypatch):
    monkeypatch.setenv("MOSS_RDNA2_INT8_STATS", "1")
    b = _binding()
    w = torch.zeros(4, 16, dtype=torch.int8)
    b._record_layout(w)
    b._record_layout(w)
    st = b.get_stats()
    assert st["enabled"] and st["calls"] == 2 and st["weight_layouts"][0]["calls"] == 2
    assert st["weight_layouts"][0]["rhs_stride"] == (1, 16)
    b.reset_stats()
    assert b.get_stats()["calls"] == 0


def test_module_level_functions_exist():
    import rdna2_ops.comfy_int8 as c
    import MOSS_RDNA2_INT8.backend as be
    for mod in (c, be):
        for name in ("int8_linear", "install_backend", "disable_backend", "get_stats", "reset_stats"):
            assert callable(getattr(mod, name))
    assert callable(c.kitchen_int8_without_transpose_copy)
    assert be._binding is not c._binding                # independent state, as in the reference
