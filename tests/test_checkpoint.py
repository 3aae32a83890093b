"""ConvRot INT8 safetensors layout and INT4 pack invalidation (CPU).

The on-disk layout is the one the reference's benchmarks read
(rdna2-ops/bench_int4_v07.py:39-43, 193-200): `<name>.weight` int8 [N,K],
`<name>.weight_scale` fp32 [N] or scalar, optional `<name>.bias`.
"""
import hashlib

import pytest
import torch

from rdna2_ops import convrot_checkpoint as ck
from rdna2_ops import int4_weight_gemm_v07 as i4


def _linears(gen):
    a = ck.Int8Linear(torch.randint(-127, 128, (48, 64), generator=gen, dtype=torch.int8),
                      torch.rand(48, generator=gen) * 0.01,
                      torch.randn(48, generator=gen).half())
    b = ck.Int8Linear(torch.randint(-127, 128, (16, 32), generator=gen, dtype=torch.int8),
                      torch.tensor([0.125]))
    return {"layers.0.proj.qkv": a, "layers.0.proj.out": b}


def test_round_trip_bit_exact(tmp_path):
    gen = torch.Generator().manual_seed(20261105)
    lin = _linears(gen)
    extra = {"layers.0.norm.weight": torch.randn(64, generator=gen),
             "layers.1.fp8.weight": torch.randn(8, 8, generator=gen),
             "layers.1.fp8.weight_scale": torch.ones(8)}
    path = tmp_path / "model_int8_convrot.safetensors"
    ck.save_int8_linears(path, lin, extra=extra, metadata={"convrot_groupsize": "128"})
    got = ck.load_int8_linears(path, device="cpu")
    assert sorted(got) == sorted(lin)       # the float weight with a scale is not INT8: skipped
    for name, ref in lin.items():
        g = got[name]
        assert torch.equal(g.weight, ref.weight)
        assert torch.equal(g.weight_scale, ref.weight_scale.float().reshape(-1))
        assert (g.bias is None) == (ref.bias is None)
        if ref.bias is not None:
            assert torch.equal(g.bias, ref.bias)
    from safetensors import safe_open
    with safe_open(str(path), framework="pt") as f:
        assert f.metadata() == {"convrot_groupsize": "128"}
        assert torch.equal(f.get_tensor("layers.0.norm.weight"), extra["layers.0.norm.weight"])


def test_read_weight_matches_reference_reader(tmp_path):
    gen = torch.Generator().manual_seed(20261107)
    lin = _linears(gen)
    path = tmp_path / "m.safetensors"
    ck.save_int8_linears(path, lin)
    w, s, md = ck.read_weight(path, "layers.0.proj.qkv.weight")
    assert torch.equal(w, lin["layers.0.proj.qkv"].weight)
    assert torch.equal(s, lin["layers.0.proj.qkv"].weight_scale)
    assert md["tensor_sha256"] == hashlib.sha256(w.numpy().tobytes()).hexdigest()
    assert md["shape"] == [48, 64] and md["dtype"] == "torch.int8"
    with pytest.raises(KeyError):
        ck.read_weight(path, "missing.weight")
    with pytest.raises(ValueError):
        ck.read_weight(path, "layers.0.proj.qkv.weight_scale")
    sub = ck.load_int8_linears(path, device="cpu", names=["layers.0.proj.out"])
    assert list(sub) == ["layers.0.proj.out"]
    with pytest.raises(KeyError):
        ck.load_int8_linears(path, device="cpu", names=["nope"])


def test_validation_follows_the_backend():
    w = torch.zeros((4, 8), dtype=torch.int8)
    with pytest.raises(ValueError):
        ck.Int8Linear(w, torch.ones(3))
    with pytest.raises(TypeError):
        ck.Int8Linear(w.float(), torch.ones(4))
    with pytest.raises(TypeError):
        ck.Int8Linear(w, torch.ones(4, dtype=torch.int32))
    with pytest.raises(ValueError):
        ck.Int8Linear(w, torch.ones(4), torch.ones(5))
    ck.Int8Linear(w, torch.ones(1))
    ck.Int8Linear(w, torch.ones(4, 1))


def test_int4_pack_stamp_detects_in_place_updates():
    gen = torch.Generator().manual_seed(3)
    p = i4.pack_int4_cpu(torch.randn(16, 128, generator=gen), group_size=64, symmetric=False)
    pack = i4.W4A16Weight(torch.zeros(1), torch.zeros(1), p.n, p.k, p.group_size, torch.bfloat16,
                          ck.source_stamp(p))
    assert pack.is_current(p)
    ck.check_current(pack, p)
    p.data.add_(0)                       # any in-place write bumps the version
    assert not pack.is_current(p)
    with pytest.raises(ValueError, match="stale"):
        ck.check_current(pack, p)
    q = i4.pack_int4_cpu(torch.randn(16, 128, generator=gen), group_size=64, symmetric=False)
    assert not pack.is_current(q)        # a different pack
    legacy = i4.W4A8Weight(torch.zeros(1), torch.zeros(1), p.n, p.k, p.group_size)
    assert legacy.is_current(q)          # packs built without a stamp are not checked
