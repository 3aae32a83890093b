"""ConvRot INT8 checkpoints loaded onto the GPU, and stale INT4 packs."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

import oracle  # noqa: E402
from conftest import outlier_activations  # noqa: E402

import rdna2_ops  # noqa: E402
from rdna2_ops import convrot_checkpoint as ck  # noqa: E402
from rdna2_ops import int4_weight_gemm_v07 as i4  # noqa: E402


def test_checkpoint_linear_matches_in_memory_and_oracle(tmp_path):
    rng = np.random.default_rng(20261106)
    n, k, m = 384, 1024, 77
    w = torch.from_numpy((rng.standard_normal((n, k)) * 0.02).astype(np.float32)).cuda()
    bias = torch.from_numpy((rng.standard_normal(n) * 0.02).astype(np.float32)).half().cuda()
    lin = ck.quantize_convrot(w, bias, rotation_block=128)
    path = tmp_path / "convrot_int8.safetensors"
    ck.save_int8_linears(path, {"blocks.0.mlp.up": lin})
    got = ck.load_int8_linears(path, device="cuda")["blocks.0.mlp.up"]
    assert got.weight.is_cuda and torch.equal(got.weight, lin.weight)
    x = torch.from_numpy(outlier_activations(rng, m, k)).cuda().half()
    y_disk = got(x, rotation_block=128, out_dtype=torch.float16)
    y_mem = rdna2_ops.w8a8_linear(x, lin.weight, lin.weight_scale, bias, rotation_block=128,
                                  out_dtype=torch.float16)
    assert torch.equal(y_disk.view(torch.int16), y_mem.view(torch.int16))
    # the stored weight is the oracle's rotated per-channel quantization
    wq_ref, sw_ref = oracle.quant_rows_int8(oracle.rotate_rows(w.cpu().numpy(), oracle.F32, 128))
    assert np.array_equal(got.weight.cpu().numpy(), wq_ref)
    assert np.array_equal(got.weight_scale.cpu().numpy().view(np.uint32), sw_ref.view(np.uint32))


def test_stale_int4_packs_are_rejected():
    torch.manual_seed(1)
    p = i4.pack_int4(torch.randn(256, 512, device="cuda") * 0.02, group_size=128, symmetric=False)
    a = torch.randn(4, 512, device="cuda").to(torch.bfloat16)
    pack16 = i4.prepare_w4a16(p, torch.bfloat16)
    pack8 = i4.prepare_w4a8(p)
    y = i4.int4_linear_a16(a, p, method="prepared", prepared=pack16)
    a8 = torch.randint(-127, 128, (4, 512), device="cuda", dtype=torch.int8)
    sa = torch.rand(4, device="cuda") * 0.01
    i4.int4_linear_a8(a8, p, sa, prepared=pack8)
    p.scales.mul_(2.0)                       # e.g. a requantization in place
    with pytest.raises(ValueError, match="stale"):
        i4.int4_linear_a16(a, p, method="prepared", prepared=pack16)
    with pytest.raises(ValueError, match="stale"):
        i4.int4_linear_a8(a8, p, sa, prepared=pack8)
    fresh = i4.prepare_w4a16(p, torch.bfloat16)
    y2 = i4.int4_linear_a16(a, p, method="prepared", prepared=fresh)
    assert not torch.equal(y, y2)
    assert torch.equal(y2, i4.int4_linear_a16(a, p))
