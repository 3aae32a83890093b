"""Research adapters (reference rdna2_ops/int8_gemm.py:217-330) on the CPU:
the scoped patch protocol (install, restore, refuse to restore over a
foreign change), the fallback of unaccelerated dtypes to the saved callables,
bridge discovery by source path, and the Qwen weight-scale dispatch.  Nothing
here launches a kernel."""
import importlib.util
import sys

import pytest

import fake_kitchen
import fake_qwen_bridge

torch = pytest.importorskip("torch")

from rdna2_ops import int8_gemm  # noqa: E402
from rdna2_ops._patch import scoped_patch  # noqa: E402


def test_scoped_patch_restores_and_detects_foreign_change():
    class Owner:
        f = staticmethod(lambda: "original")
    repl = lambda: "replacement"  # noqa: E731
    with scoped_patch(Owner, {"f": repl}, "owner export"):
        assert Owner.f is repl
    assert Owner.f() == "original"
    intruder = lambda: "intruder"  # noqa: E731
    with pytest.raises(RuntimeError, match="owner export changed"):
        with scoped_patch(Owner, {"f": repl}, "owner export"):
            Owner.f = intruder
    assert Owner.f is intruder          # a foreign value is never overwritten


def test_qwen_candidate_patches_both_wrappers_and_falls_back():
    bridge = fake_qwen_bridge
    saved = (bridge.triton_int8_linear, bridge.triton_int8_linear_per_row)
    x = torch.randn(3, 5, 64, dtype=torch.float16)
    w = torch.randint(-127, 128, (16, 64), dtype=torch.int8)
    ws = torch.rand(16) * 0.01 + 0.001
    with int8_gemm.qwen_int8_gemm_candidate(bridge) as stats:
        assert bridge.triton_int8_linear is not saved[0]
        assert bridge.triton_int8_linear_per_row is not saved[1]
        before = dict(fake_qwen_bridge.CALLS)
        # fp16 activations / compute dtype are not accelerated: the saved wrappers run
        y = bridge.triton_int8_linear_per_row(x, w, ws, compute_dtype=torch.float16)
        y2 = bridge.triton_int8_linear(x.float(), w, 0.01, compute_dtype=torch.float16)
        assert y.shape == (3, 5, 16) and y2.shape == (3, 5, 16)
        assert fake_qwen_bridge.CALLS["linear_per_row"] == before["linear_per_row"] + 1
        assert fake_qwen_bridge.CALLS["linear"] == before["linear"] + 1
    assert stats["fallbacks"] == 2 and stats["hits"] == 0
    assert (bridge.triton_int8_linear, bridge.triton_int8_linear_per_row) == saved


def test_qwen_bridge_discovered_by_source_path(tmp_path):
    src = tmp_path / "RDNA2-Qwen21-INT8" / "rocm_int8_kitchen_patch.py"
    src.parent.mkdir()
    src.write_text(open(fake_qwen_bridge.__file__).read())
    spec = importlib.util.spec_from_file_location("qwen_bridge_under_test", src)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    sys.modules["qwen_bridge_under_test"] = mod
    try:
        assert int8_gemm._loaded_qwen_bridge() is mod
        with int8_gemm.qwen_int8_gemm_candidate() as stats:
            assert mod.triton_int8_linear.__name__ == "linear"
        assert stats == {"hits": 0, "fallbacks": 0, "shapes": {}}
    finally:
        del sys.modules["qwen_bridge_under_test"]
    with pytest.raises(RuntimeError, match="Qwen patientx bridge"):
        int8_gemm._loaded_qwen_bridge()


def test_qwen_column_scale_dispatch():
    dev = torch.device("cpu")
    per_row = int8_gemm.qwen_column_scale(torch.arange(6, dtype=torch.float16).reshape(6, 1), 6, dev, True)
    assert per_row.dtype == torch.float32 and per_row.shape == (6,) and per_row.is_contiguous()
    one = int8_gemm.qwen_column_scale(torch.tensor([[0.25]]), 6, dev, False)
    assert one.shape == (1,) and float(one) == 0.25
    num = int8_gemm.qwen_column_scale(0.125, 6, dev, False)
    assert num.shape == (1,) and num.dtype == torch.float32 and float(num) == 0.125


def test_moss_candidate_falls_back_for_integer_inputs():
    kitchen = fake_kitchen.install()
    try:
        original = kitchen.eager.int8_linear
        with int8_gemm.moss_int8_gemm_candidate() as stats:
            assert kitchen.eager.int8_linear is not original
            out = kitchen.eager.int8_linear(torch.zeros(2, 8, dtype=torch.int32), None, None)
        assert out == "original" and stats["fallbacks"] == 1
        assert kitchen.eager.int8_linear is original
    finally:
        kitchen.uninstall()


def test_candidates_check_launch_keywords():
    with pytest.raises(ValueError):
        with int8_gemm.qwen_int8_gemm_candidate(fake_qwen_bridge, tile=(24, 64, 64)):
            pass
    with pytest.raises(ValueError):
        with int8_gemm.qwen_int8_gemm_candidate(fake_qwen_bridge, num_warps=2):
            pass
