"""Stand-in for the patientx Qwen bridge module (RDNA2-Qwen21-INT8/
rocm_int8_kitchen_patch.py, absent from the reference checkout), built from
the names the reference's adapter reads (rdna2_ops/int8_gemm.py:274-330):
two GEMM wrappers `triton_int8_linear` (scalar weight scale) and
`triton_int8_linear_per_row` (one scale per output row), whose module globals
hold the row quantizer `triton_quantize_rowwise`.  Test infrastructure only:
the wrappers compute in plain torch on whatever device the inputs live on."""
import torch

CALLS = {"linear": 0, "linear_per_row": 0, "quantize": 0}


def triton_quantize_rowwise(x):
    """Per-row symmetric INT8: scale = absmax / 127 (1 for an all-zero row),
    codes = round-half-even(x / scale) clamped to [-127, 127]; scale [M, 1]."""
    CALLS["quantize"] += 1
    x = x.float()
    amax = x.abs().amax(dim=1, keepdim=True)
    scale = torch.where(amax > 0, amax / 127.0, torch.ones_like(amax))
    codes = torch.clamp(torch.round(x / scale), -127, 127).to(torch.int8)
    return codes, scale


def _dequant_linear(x, weight, col_scale, bias, compute_dtype):
    codes, row_scale = triton_quantize_rowwise(x.reshape(-1, x.shape[-1]))
    acc = codes.double() @ weight.double().T
    y = (acc * row_scale.double() * col_scale.double()).to(compute_dtype)
    if bias is not None:
        y = y + bias.to(compute_dtype)
    return y.reshape(*x.shape[:-1], weight.shape[0])


def triton_int8_linear(x, weight, weight_scale, bias=None, compute_dtype=torch.float16):
    CALLS["linear"] += 1
    s = weight_scale if isinstance(weight_scale, torch.Tensor) else torch.tensor(float(weight_scale))
    return _dequant_linear(x, weight, s.to(x.device).reshape(1, -1), bias, compute_dtype)


def triton_int8_linear_per_row(x, weight, weight_scale, bias=None, compute_dtype=torch.float16):
    CALLS["linear_per_row"] += 1
    return _dequant_linear(x, weight, weight_scale.to(x.device).reshape(1, -1), bias, compute_dtype)
