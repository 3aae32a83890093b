#!/usr/bin/env python3
"""Generate golden vectors from the reference's own CPU-runnable code.

Run on a machine that has the reference checkout (its path in
--reference, or in the environment variable RDNA2_REFERENCE); the GPU hosts
only read the committed .npz output.

  python tests/golden/make_golden.py --reference PATH

What runs from the reference (unmodified, imported from its source tree):
  * rdna2_ops.int4_weight_gemm_v07.pack_int4_cpu / unpack_int4_cpu
    (int4_weight_gemm_v07.py:49-92), on the 17x19x384 smoke weights of
    bench_int4_v07.py:85-95 over every group/symmetry/layout/order;
  * int4_model_switches_v07.grouped_integer_reference (lines 19-34) with its
    GPU unpack swapped for the reference's CPU unpack;
  * production/MOSS_RDNA2_INT8/backend.py int8_linear + install_backend
    (lines 71-188) against a minimal stand-in of comfy_kitchen built from the
    call sites' names only (the real package is not vendored).  The stand-in
    quantizer is this repository's frozen row-quantizer contract, so this
    fixture pins the backend's GEMM/epilogue/bias order, not Kitchen's
    quantizer;
  * the bench_int8_gemm.py:181-203 known-answer recipe (INT64 oracle over an
    offset/padded A view, both B layouts, scalar and vector scales, bias)
    evaluated with torch on the CPU;
  * torch's own float8_e4m3fn/e5m2 casts over all 256 codes, the native side
    of the exhaustive decode check in bench_dtype_gemm_v06.py:232-245.
"""
import argparse
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent


def _fake_kitchen(quantize):
    """Stand-in comfy_kitchen modules exposing only the names backend.py uses."""
    root = types.ModuleType("comfy_kitchen")
    backends = types.ModuleType("comfy_kitchen.backends")
    eager = types.ModuleType("comfy_kitchen.backends.eager")
    quant = types.ModuleType("comfy_kitchen.backends.eager.quantization")
    registry_mod = types.ModuleType("comfy_kitchen.registry")

    def original_int8_linear(*args, **kwargs):
        raise RuntimeError("non-fp32 Kitchen path is not available offline")

    quant.int8_linear = original_int8_linear
    quant._int8_matmul_accumulate = None
    quant.quantize_int8_rowwise = quantize
    quant._apply_input_act = lambda x, act, w, eps: x
    quant._apply_residual = lambda y, r, s: y
    eager.int8_linear = original_int8_linear
    eager.quantization = quant

    class Registry:
        def get_implementation(self, name, backend):
            return eager.int8_linear

    registry_mod.registry = Registry()
    root.backends = backends
    backends.eager = eager
    mods = {"comfy_kitchen": root, "comfy_kitchen.backends": backends,
            "comfy_kitchen.backends.eager": eager,
            "comfy_kitchen.backends.eager.quantization": quant,
            "comfy_kitchen.registry": registry_mod}
    sys.modules.update(mods)
    return quant


def _row_quantize(x):
    """Frozen contract: s = absmax/127 (s := 1 if not > 0), q = clamp(rne(x/s))."""
    x = x.float()
    s = x.abs().amax(dim=-1, keepdim=True) / 127.0
    s = torch.where(s > 0, s, torch.ones_like(s))
    q = torch.round(x / s).clamp(-127, 127).to(torch.int8)
    return q, s


def _exact_matmul(a, b):
    return (a.to(torch.int64) @ b.to(torch.int64)).to(torch.int32)


def int8_known_answer(out):
    """bench_int8_gemm.py:181-203 recipe on the CPU with a seeded generator."""
    gen = torch.Generator().manual_seed(20261106)
    m, n, k = 37, 53, 79
    cases = {}
    for layout in ("weight_nk", "rhs_kn"):
        for scalar in (False, True):
            a_store = torch.randint(-128, 128, (m + 2, k + 3), dtype=torch.int8, generator=gen)
            a = a_store[1:1 + m, 1:1 + k]
            w = torch.randint(-128, 128, (n, k), dtype=torch.int8, generator=gen)
            sa = torch.rand(m, 1, generator=gen) * 0.02 + 0.001
            sb = torch.rand(1 if scalar else n, generator=gen) * 0.02 + 0.001
            bias = torch.randn(n, generator=gen)
            b = w.T if layout == "weight_nk" else w.T.contiguous()
            oracle_i64 = a.to(torch.int64) @ b.to(torch.int64)
            ref = oracle_i64.to(torch.float32) * (sa * sb.reshape(1, -1)) + bias
            key = f"{layout}_{'scalar' if scalar else 'vector'}"
            cases[key + "_a_store"] = a_store.numpy()
            cases[key + "_w"] = w.numpy()
            cases[key + "_sa"] = sa.numpy()
            cases[key + "_sb"] = sb.numpy()
            cases[key + "_bias"] = bias.numpy()
            cases[key + "_acc"] = oracle_i64.to(torch.int32).numpy()
            cases[key + "_ref"] = ref.numpy()
    np.savez_compressed(out / "int8_known_answer.npz", **cases)
    return len(cases) // 7


def moss_backend(ref_root, out):
    """Reference backend.int8_linear (fp32 path) with the stand-in Kitchen."""
    _fake_kitchen(_row_quantize)
    quant = sys.modules["comfy_kitchen.backends.eager.quantization"]
    sys.path.insert(0, str(ref_root / "rdna2-ops" / "production"))
    import MOSS_RDNA2_INT8.backend as backend  # noqa: E402  (reference source)
    quant._int8_matmul_accumulate = _exact_matmul
    backend.install_backend(_exact_matmul)
    gen = torch.Generator().manual_seed(20261105)
    cases = {}
    for idx, (m, n, k, with_bias, scalar) in enumerate(
            ((33, 40, 96, True, False), (64, 48, 256, False, False), (7, 24, 64, True, True))):
        x = torch.randn(m, k, generator=gen)
        x[:, : max(1, k // 100)] *= 20.0
        w = torch.randint(-127, 128, (n, k), dtype=torch.int8, generator=gen)
        ws = torch.rand(1 if scalar else n, generator=gen) * 0.01 + 0.001
        bias = torch.randn(n, generator=gen) * 0.02 if with_bias else None
        y = backend.int8_linear(x, w, ws, bias, out_dtype=torch.float32)
        cases[f"c{idx}_x"] = x.numpy()
        cases[f"c{idx}_w"] = w.numpy()
        cases[f"c{idx}_ws"] = ws.numpy()
        if bias is not None:
            cases[f"c{idx}_bias"] = bias.numpy()
        cases[f"c{idx}_y"] = y.numpy()
    backend.disable_backend()
    np.savez_compressed(out / "moss_backend_fp32.npz", **cases)
    return 3


def int4_packing(ref_root, out):
    sys.path.insert(0, str(ref_root / "rdna2-ops"))
    from rdna2_ops.int4_weight_gemm_v07 import pack_int4_cpu, unpack_int4_cpu  # reference
    import int4_model_switches_v07 as switches  # reference
    gen = torch.Generator().manual_seed(20261107)
    m, n, k = 17, 19, 384
    a = torch.randint(-128, 128, (m, k), dtype=torch.int8, generator=gen)
    a[0] = torch.arange(k).remainder(256).to(torch.int8)
    w = torch.randn((n, k), generator=gen) * .2
    w[0] = 0
    w[1] = torch.arange(k).remainder(16).float() - 8
    w[2] = torch.arange(k).remainder(15).float() - 7
    cases = {"a": a.numpy(), "w": w.numpy()}
    for g in (32, 64, 128):
        for sym in (True, False):
            for layout in ("nk", "kn"):
                for order in ("low", "high"):
                    key = f"g{g}_{'sym' if sym else 'aff'}_{layout}_{order}"
                    p = pack_int4_cpu(w, group_size=g, symmetric=sym, layout=layout, order=order)
                    cases[key + "_data"] = p.data.numpy()
                    cases[key + "_scales"] = p.scales.numpy()
                    cases[key + "_zeros"] = p.zeros.numpy()
                    cases[key + "_sums"] = p.sums.numpy()
                    qi = unpack_int4_cpu(p, floating=False)
                    cases[key + "_centered"] = qi.numpy()
                    cases[key + "_float"] = unpack_int4_cpu(p, floating=True).numpy()
                    cases[key + "_int_oracle"] = (a.to(torch.int64) @ qi.T.to(torch.int64)).numpy()
    # BASELINE-format affine g128 case at a slightly larger shape.
    wb = torch.randn((64, 512), generator=gen) * 0.02
    p = pack_int4_cpu(wb, group_size=128, symmetric=False, layout="nk", order="low")
    cases.update(big_w=wb.numpy(), big_data=p.data.numpy(), big_scales=p.scales.numpy(),
                 big_zeros=p.zeros.numpy(), big_sums=p.sums.numpy())
    # grouped_integer_reference (W4A8 grouped order) with the CPU unpack.
    switches.unpack_int4 = lambda packed, dtype: unpack_int4_cpu(packed, floating=False).to(dtype)
    a8 = torch.randint(-128, 128, (37, 384), dtype=torch.int8, generator=gen)
    sa = torch.rand(37, generator=gen) * .02 + .001
    wg = torch.randn((53, 384), generator=gen) * .01
    bias = torch.randn(53, generator=gen) * .01
    pg = pack_int4_cpu(wg, group_size=32, symmetric=False, layout="kn", order="low")
    y = switches.grouped_integer_reference(a8, pg, sa, bias)
    cases.update(grouped_a=a8.numpy(), grouped_sa=sa.numpy(), grouped_w=wg.numpy(),
                 grouped_bias=bias.numpy(), grouped_data=pg.data.numpy(),
                 grouped_scales=pg.scales.numpy(), grouped_zeros=pg.zeros.numpy(),
                 grouped_y=y.numpy())
    np.savez_compressed(out / "int4_packing.npz", **cases)
    return 24


def fp8_decode(out):
    codes = torch.arange(256, dtype=torch.int16).to(torch.uint8)
    np.savez_compressed(out / "fp8_decode.npz", codes=codes.numpy(),
                        e4m3=codes.view(torch.float8_e4m3fn).float().numpy(),
                        e5m2=codes.view(torch.float8_e5m2).float().numpy())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, default=os.environ.get("RDNA2_REFERENCE"))
    cfg = ap.parse_args()
    if cfg.reference is None:
        ap.error("give the reference checkout with --reference or RDNA2_REFERENCE")
    cfg.reference = Path(cfg.reference)
    sys.dont_write_bytecode = True
    torch.set_num_threads(2)
    print("int8 known-answer cases:", int8_known_answer(OUT))
    print("moss backend cases:", moss_backend(cfg.reference, OUT))
    print("int4 packing cases:", int4_packing(cfg.reference, OUT))
    fp8_decode(OUT)
    print("wrote", sorted(p.name for p in OUT.glob("*.npz")))


if __name__ == "__main__":
    main()
