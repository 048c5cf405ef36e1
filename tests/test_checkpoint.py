"""The on-disk format of repacked layers and the repack exactness check (qwenfast_b200.checkpoint), on CPU with the
torch versions of the kernel-layout maps (the CUDA repack kernels produce the same bytes: tests/test_gpu_moe.py)."""
import os

import pytest
import torch

from qwenfast_b200 import checkpoint, formats, synthetic
from qwenfast_b200.ops import MoELayerWeights


def _cpu_layer(cfg):
    L = synthetic.make_moe_layer(cfg)
    wk13, sk13 = formats.repack_w4_torch(L["w13"], L["s13"], gated=True)
    wk2, sk2 = formats.repack_w4_torch(L["w2"], L["s2"], gated=False)
    sh = (formats.repack_bf16_torch(L["sh_gu"], True), formats.repack_bf16_torch(L["sh_d"], False)) if cfg.Is else (None, None)
    lw = MoELayerWeights(L["router"], wk13, sk13, wk2, sk2, L.get("w_gate"), sh[0], sh[1], cfg.H, cfg.I, cfg.E, cfg.Is)
    return L, lw


@pytest.fixture(scope="module")
def small():
    return _cpu_layer(synthetic.MoEConfig("ckpt", 256, 8, 128, 2, 3, 64, 5))


def test_repack_verifies_and_a_changed_byte_is_caught(small):
    L, lw = small
    checkpoint.verify_layer(lw, L, experts_per_block=3)
    bad = MoELayerWeights(**{**lw.__dict__, "w2": lw.w2.clone()})
    bad.w2[5, 17] ^= 0x10
    with pytest.raises(RuntimeError, match="w2 experts 5"):
        checkpoint.verify_layer(bad, L, experts_per_block=1)
    bad = MoELayerWeights(**{**lw.__dict__, "sh_w2": lw.sh_w2.clone()})
    bad.sh_w2[3] = torch.tensor(1.0, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="sh_d"):
        checkpoint.verify_layer(bad, L)


def test_save_load_round_trip(small, tmp_path):
    L, lw = small
    p = os.path.join(tmp_path, "layer.safetensors")
    checkpoint.save_layer(p, lw)
    got = checkpoint.load_layer(p, device="cpu")
    for n in ("router", "w13", "s13", "w2", "s2", "w_gate", "sh_w13", "sh_w2"):
        assert torch.equal(getattr(got, n).view(torch.uint8), getattr(lw, n).contiguous().view(torch.uint8)), n
    assert (got.H, got.I, got.E, got.Is) == (lw.H, lw.I, lw.E, lw.Is)
    checkpoint.verify_layer(got, L)


def test_load_rejects_tampering_and_other_formats(small, tmp_path):
    from safetensors.torch import load_file, save_file
    from safetensors import safe_open
    L, lw = small
    p = os.path.join(tmp_path, "layer.safetensors")
    checkpoint.save_layer(p, lw)
    with safe_open(p, framework="pt") as f:
        meta = f.metadata()
    t = load_file(p)
    t["s13"] = t["s13"].clone()
    t["s13"][0, 0] = torch.tensor(2.0, dtype=torch.bfloat16)
    q = os.path.join(tmp_path, "tampered.safetensors")
    save_file(t, q, metadata=meta)
    with pytest.raises(RuntimeError, match="s13 does not match"):
        checkpoint.load_layer(q, device="cpu")
    checkpoint.load_layer(q, device="cpu", verify=False)          # the digest check is what catches it
    save_file(load_file(p), q, metadata={**meta, "version": "0"})
    with pytest.raises(RuntimeError, match="not a"):
        checkpoint.load_layer(q, device="cpu")
    save_file(load_file(p), q, metadata={**meta, "I": "256"})
    with pytest.raises(RuntimeError, match="shape"):
        checkpoint.load_layer(q, device="cpu")


def test_layer_without_shared_expert(tmp_path):
    L, lw = _cpu_layer(synthetic.MoEConfig("ckpt0", 256, 4, 128, 2, 2, 0, 6))
    p = os.path.join(tmp_path, "l.safetensors")
    checkpoint.save_layer(p, lw)
    got = checkpoint.load_layer(p, device="cpu")
    assert got.Is == 0 and got.sh_w13 is None and got.w_gate is None
    checkpoint.verify_layer(got, L)
