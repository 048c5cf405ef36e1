"""Host logic of the SGLang overlay mirror (qwenfast_b200.overlay), on CPU: the load-time INT8 quantiser against the
reference's own function's outputs (bit-exact), the INT8 linear gate, and the MoE block gates (``why_not``,
``_a16_ok``, ``_a16_shared``) with the decline behaviour of serve/overlays/sglang/srt/qwenfast.py:1127-1171.
Nothing here launches a kernel: every gate is checked on CPU tensors up to its last ("device") condition."""
import os
from types import SimpleNamespace

import pytest
import torch

from conftest import GOLDEN
from qwenfast_b200 import overlay

BF = torch.bfloat16
REF = torch.load(os.path.join(GOLDEN, "reference_fns.pt"))


def test_w8_quant_matches_reference_function():
    for tag in ("w8_g128", "w8_g64"):
        r = REF[tag]
        p = overlay.w8_quant(r["w"], rows_per_chunk=7)        # chunking must not change anything
        assert p["kind"] == "w8" and p["G"] == r["G"] and p["shape"] == tuple(r["w"].shape)
        assert torch.equal(p["q"], r["q"]) and torch.equal(p["s"], r["s"]), tag


def _w8_entry(N=256, K=256):
    w = (torch.randn(N, K, generator=torch.Generator().manual_seed(0)) * 0.02).to(BF)
    return (overlay.w8_quant(w), 0, N)


def test_w8_route_gate_reasons():
    e = _w8_entry()
    x = torch.randn(4, 256).to(BF)
    assert overlay.w8_route(e, x, bias=torch.zeros(256)) == "bias"
    assert overlay.w8_route(e, torch.randn(65, 256).to(BF)) == "rows"
    assert overlay.w8_route(e, torch.randn(2, 3, 256).to(BF)) == "device"   # 6 rows: every host check passes
    assert overlay.w8_route(e, x.float()) == "dtype"
    assert overlay.w8_route(e, torch.randn(4, 512).to(BF)[:, ::2]) == "layout"
    e64 = (overlay.w8_quant(torch.randn(128, 192).to(BF)), 0, 128)
    assert e64[0]["G"] == 64 and overlay.w8_route(e64, torch.randn(3, 192).to(BF)) == "device"
    assert overlay.w8_route(e, x) == "device"                                 # CPU tensors never reach the kernel
    assert overlay.w8_route((e[0], 0, 200), x) == "device"                    # 200 rows: a multiple of 8 qualifies
    assert overlay.w8_route((e[0], 0, 204), x) == "shape"                     # output rows not a multiple of 8


def test_w8_linear_empty_rows():
    e = _w8_entry()
    y = overlay.w8_linear(e, torch.empty(0, 256, dtype=BF))
    assert y.shape == (0, 256)


class SiluAndMul:   # the activation class name the shared-expert gate looks for
    pass


def _block(H=256, E=32, topk=4, I=128, Is=64, **cfg_over):
    """An object with the attribute names of SGLang's Qwen2MoeSparseMoeBlock, CPU tensors, kernel-layout shapes."""
    cfg = SimpleNamespace(top_k=topk, renormalize=True, use_grouped_topk=False, num_fused_shared_experts=0,
                          custom_routing_function=None, correction_bias=None,
                          apply_routed_scaling_factor_on_output=False, scoring_func="softmax", output_format=None)
    for k, v in cfg_over.items():
        setattr(cfg, k, v)
    experts = SimpleNamespace(
        moe_runner_config=SimpleNamespace(inplace=False),
        w13_weight=torch.zeros(E, 2 * I * H // 8, dtype=torch.int32), w13_weight_scale=torch.zeros(E, 2 * I * H // 128, dtype=BF),
        w13_weight_scale_2=None, w2_weight=torch.zeros(E, H * I // 8, dtype=torch.int32),
        w2_weight_scale=torch.zeros(E, H * I // 128, dtype=BF), w2_weight_scale_2=torch.ones(E, dtype=BF))
    shared = SimpleNamespace(act_fn=SiluAndMul(), gate_up_proj=SimpleNamespace(weight=torch.zeros(2 * Is, H, dtype=BF), bias=None),
                             down_proj=SimpleNamespace(weight=torch.zeros(H, Is, dtype=BF), bias=None))
    return SimpleNamespace(
        topk=SimpleNamespace(topk_config=cfg, enable_waterfill=False, waterfill_balancer=None),
        gate=SimpleNamespace(weight=torch.zeros(E, H, dtype=BF), bias=None, quant_method=None),
        shared_expert=shared, enable_shared_expert_fusion=False, experts=experts,
        shared_expert_gate=SimpleNamespace(weight=torch.zeros(1, H, dtype=BF), bias=None))


def test_why_not_reasons_in_order():
    b = _block()
    x = torch.zeros(4, 256, dtype=BF)
    assert overlay.why_not(b, x) == "device"            # every host-side condition holds
    assert overlay.why_not(b, torch.zeros(65, 256, dtype=BF)) == "shape"
    assert overlay.why_not(b, torch.zeros(4, 320, dtype=BF)) == "shape"
    assert overlay.why_not(b, x.float()) == "dtype"
    assert overlay.why_not(b, x, lora_active=True) == "lora"
    assert overlay.why_not(_block(use_grouped_topk=True), x) == "topk"
    assert overlay.why_not(_block(top_k=17), x) == "topk"
    assert overlay.why_not(_block(scoring_func="sigmoid"), x) == "topk"
    b2 = _block()
    b2.enable_shared_expert_fusion = True
    assert overlay.why_not(b2, x) == "shared"
    b3 = _block()
    b3.experts.moe_runner_config.inplace = True
    assert overlay.why_not(b3, x) == "inplace"
    b4 = _block()
    b4.gate.weight = torch.zeros(30, 256, dtype=BF)     # experts % 16 != 0
    assert overlay.why_not(b4, x) == "gate"
    b5 = _block()
    b5.topk.enable_waterfill = True
    assert overlay.why_not(b5, x) == "waterfill"


def test_why_not_simulated_routing_env(monkeypatch):
    monkeypatch.setenv("SGLANG_SIMULATE_UNIFORM_EXPERTS", "1")
    assert overlay.why_not(_block(), torch.zeros(4, 256, dtype=BF)) == "simulate"


def test_dual_declines_to_the_stock_forward():
    b = _block()
    x = torch.zeros(4, 256, dtype=BF)
    assert overlay.dual(b, x, orig=lambda blk, h: ("stock", h.shape)) == ("stock", x.shape)
    with pytest.raises(RuntimeError, match="declined"):
        overlay.dual(b, x)


def test_a16_ok_shapes():
    x = torch.zeros(4, 256, dtype=BF)
    assert overlay._a16_ok(_block(), x)
    b = _block()
    b.experts.w13_weight = b.experts.w13_weight[:, :-1].contiguous()
    assert not overlay._a16_ok(b, x)
    b = _block()
    b.experts.w2_weight_scale_2 = torch.ones(3, dtype=BF)
    assert not overlay._a16_ok(b, x)
    b = _block()
    b.shared_expert_gate.bias = torch.zeros(1)
    assert not overlay._a16_ok(b, x)
    b = _block()
    b.experts._qf_a16 = (None,) * 6                      # an attached decode copy takes precedence
    assert not overlay._a16_ok(b, x)
    assert not overlay._a16_ok(_block(), torch.zeros(65, 256, dtype=BF))


def test_a16_shared_gate_on_host():
    b = _block()
    b.shared_expert.act_fn = object()                     # not SiluAndMul: the shared expert runs outside the kernel
    assert overlay._a16_shared(b) is None and b._qf_a16sh is None
    b = _block()
    assert overlay._a16_shared(b) is None                 # CPU weights: nothing is repacked here


def test_a16_ok_accepts_nvfp4_experts():
    """NVFP4 experts (E4M3 group-16 scales as uint8, the reference's format) qualify with their own scale shapes."""
    b = _block()
    E, H, I = 32, 256, 128
    b.experts.w13_weight_scale = torch.zeros(E, 2 * I * H // 16, dtype=torch.uint8)
    b.experts.w2_weight_scale = torch.zeros(E, H * I // 16, dtype=torch.uint8)
    x = torch.zeros(4, 256, dtype=BF)
    assert overlay._a16_format(b) == "nvfp4" and overlay._a16_ok(b, x)
    b.experts.w2_weight_scale = torch.zeros(E, H * I // 128, dtype=torch.uint8)   # int4-sized scales: no
    assert not overlay._a16_ok(b, x)
    assert overlay._a16_format(_block()) == "int4"


def test_tensor_cache_follows_the_tensors_lifetime():
    """The cache of converted weights (ops.tensor_cache): built once per live set of tensors, rebuilt for other
    tensors, dropped when the tensors are freed."""
    import gc
    from qwenfast_b200 import ops
    cache, calls = {}, []

    def build():
        calls.append(1)
        return len(calls)

    a, b = torch.zeros(4), torch.ones(4)
    assert ops.tensor_cache(cache, (a, b), build) == 1
    assert ops.tensor_cache(cache, (a, b), build) == 1 and len(calls) == 1
    c = torch.zeros(4)
    assert ops.tensor_cache(cache, (c, b), build) == 2 and len(cache) == 2
    del a
    gc.collect()
    assert len(cache) == 1
    del c
    gc.collect()
    assert cache == {}
