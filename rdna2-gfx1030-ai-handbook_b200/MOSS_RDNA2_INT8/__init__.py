"""MOSS INT8 custom node for B200 (drop-in for the reference's
production/MOSS_RDNA2_INT8/__init__.py:1-64).

MOSS_RDNA2_INT8_PATCH=1 installs the B200 INT8 GEMM (rdna2_ops.int8_matmul)
as Kitchen's accumulator; MOSS_RDNA2_INT8_LAYOUT=view (default) also replaces
Kitchen's eager int8_linear export with this package's backend.int8_linear;
LAYOUT=legacy keeps only the accumulator.  MOSS_RDNA2_INT8_STATS=1 enables
the backend counters.  The device check requires an sm_100 GPU (the
reference checks gfx1030).  The reference's attention dispatch and
measurement hooks are not part of the quantized-linear path and are not
installed here.
"""
import logging
import os

NODE_CLASS_MAPPINGS = {}
NODE_DISPLAY_NAME_MAPPINGS = {}

if os.environ.get("MOSS_RDNA2_INT8_PATCH") == "1":
    layout = os.environ.get("MOSS_RDNA2_INT8_LAYOUT", "view")
    if layout not in {"legacy", "view"}:
        raise ValueError("MOSS_RDNA2_INT8_LAYOUT must be 'legacy' or 'view'")

    import torch

    if torch.version.cuda is None or not torch.cuda.is_available():
        raise RuntimeError("MOSS B200 patch requires a CUDA GPU")
    cap = torch.cuda.get_device_capability(0)
    if cap[0] != 10:
        raise RuntimeError("This INT8 patch targets sm_100 (B200), not sm_%d%d" % cap)

    import comfy_kitchen.backends.eager.quantization as ck_quant
    from rdna2_ops.int8_gemm import int8_matmul

    previous_accumulator = ck_quant._int8_matmul_accumulate
    try:
        ck_quant._int8_matmul_accumulate = int8_matmul
        if layout == "view":
            from . import backend

            backend.install_backend(int8_matmul)
    except Exception:
        ck_quant._int8_matmul_accumulate = previous_accumulator
        raise

    logging.getLogger("moss-b200").warning(
        "MOSS_RDNA2_INT8_PATCH active on sm_%d%d: tcgen05 INT8 GEMM, layout=%s%s",
        cap[0], cap[1], layout,
        " (fused prologue + GEMM + Kitchen epilogue, fp32/fp16/bf16)" if layout == "view"
        else " (original eager linear)",
    )
