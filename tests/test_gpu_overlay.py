"""The overlay mirror (qwenfast_b200.overlay) on the GPU: each route of the reference's overlay for this path
(serve/overlays/sglang/srt/qwenfast.py) against the CPU oracle -- the INT8 linear's kernel and decline paths, the
W8A8 linear with more than 16 rows, and the decode MoE block's ``dual`` forward with the shared expert in the kernel,
passed in precomputed, and with experts outside the kernel's format (router kernel + the block's own experts)."""
from types import SimpleNamespace

import pytest
import torch

from oracle import moe_ref, w8_ref
from qwenfast_b200 import ops, overlay, synthetic
from qwenfast_b200.ops import MoELayerWeights

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def test_w8_linear_kernel_and_decline_paths(cuda):
    g = torch.Generator(device="cpu").manual_seed(3)
    w = (torch.randn(1280, 2048, generator=g) * 0.02).to(BF)
    p = overlay.w8_quant(w.to(cuda))
    q, s = w8_ref.w8_quant(w)
    assert torch.equal(p["q"].cpu(), q) and torch.equal(p["s"].cpu(), s)
    deq = w8_ref.w8g_dequant(q, s)
    for shape, rows, bias in (((2, 3, 2048), (0, 1280), None), ((5, 2048), (256, 768), None),
                              ((100, 2048), (0, 1280), None), ((4, 2048), (0, 1280), True)):
        x = torch.randn(*shape, generator=g).to(BF)
        b = (torch.randn(rows[1] - rows[0], generator=g) * 0.1).to(BF) if bias else None
        entry = (p, rows[0], rows[1])
        route = overlay.w8_route(entry, x.to(cuda), None if b is None else b.to(cuda))
        assert route == (None if x.numel() // 2048 <= 64 and b is None else ("rows" if b is None else "bias"))
        y = overlay.w8_linear(entry, x.to(cuda), None if b is None else b.to(cuda))
        truth = x.float().reshape(-1, 2048) @ deq[rows[0]:rows[1]].T
        if b is not None:
            truth = truth + b.float()
        assert y.shape == (*shape[:-1], rows[1] - rows[0])
        err = ((y.float().cpu().reshape(truth.shape) - truth).norm() / truth.norm()).item()
        assert err < 4e-3, (shape, rows, err)


def test_w8a8_linear_rows_beyond_16_are_exact(cuda):
    g = torch.Generator(device="cpu").manual_seed(4)
    q = torch.randint(-127, 128, (1024, 2048), generator=g, dtype=torch.int8)
    sw = torch.rand(1024, generator=g) * 1e-3 + 1e-4
    p = overlay.w8a8_prepare(q.to(cuda), sw.to(cuda))
    x = torch.randn(40, 2048, generator=g).to(BF)
    y = overlay.w8a8_linear(p, x.to(cuda))
    ref, _, _, _ = w8_ref.w8a8_ref(x, q, sw)
    assert torch.equal(y.cpu(), ref)
    b = (torch.randn(1024, generator=g) * 0.1).to(BF)
    yb = overlay.w8a8_linear(p, x.to(cuda), b.to(cuda))
    assert torch.equal(yb.cpu(), (ref.float() + b.float()).to(BF))


class SiluAndMul:   # the activation class name the shared-expert gate looks for
    pass


def _block(cfg, L, dev, shared_act=SiluAndMul, kernel_experts=True):
    lw = MoELayerWeights.from_canonical(L["router"].to(dev), L["w13"].to(dev), L["s13"].to(dev), L["w2"].to(dev),
                                        L["s2"].to(dev))
    topk_cfg = SimpleNamespace(top_k=cfg.topk, renormalize=True, use_grouped_topk=False, num_fused_shared_experts=0,
                               custom_routing_function=None, correction_bias=None,
                               apply_routed_scaling_factor_on_output=False, scoring_func="softmax", output_format=None)
    calls = []

    def stock_experts(h, topk_output):   # SGLang's FusedMoE stand-in: the oracle given the router kernel's routing
        calls.append(topk_output)
        C = {k: v.cpu() for k, v in L.items()}
        return moe_ref.moe_rounded(h.cpu(), topk_output.topk_ids.cpu(), topk_output.topk_weights.cpu(), C["w13"],
                                   C["s13"], C["w2"], C["s2"]).to(h.device)

    experts = SimpleNamespace(moe_runner_config=SimpleNamespace(inplace=False), calls=calls)
    if kernel_experts:
        experts.w13_weight, experts.w13_weight_scale, experts.w13_weight_scale_2 = lw.w13, lw.s13, None
        experts.w2_weight, experts.w2_weight_scale, experts.w2_weight_scale_2 = lw.w2, lw.s2, None
    shared = SimpleNamespace(act_fn=shared_act(), gate_up_proj=SimpleNamespace(weight=L["sh_gu"].to(dev), bias=None),
                             down_proj=SimpleNamespace(weight=L["sh_d"].to(dev), bias=None))

    def fwd_shared(h, apply_gate):
        out = moe_ref.shared_expert_bf16(h.cpu(), L["sh_gu"].cpu(), L["sh_d"].cpu())
        if apply_gate:
            gl = moe_ref.shared_gate_logits(h.cpu(), L["w_gate"].cpu())
            out = (torch.sigmoid(gl)[:, None] * out.float()).to(BF)
        return out.to(h.device)

    class Experts(SimpleNamespace):
        def __call__(self, h, topk_output):
            return stock_experts(h, topk_output)

    return SimpleNamespace(
        topk=SimpleNamespace(topk_config=topk_cfg, enable_waterfill=False, waterfill_balancer=None),
        gate=SimpleNamespace(weight=L["router"].to(dev), bias=None, quant_method=None),
        shared_expert=shared, enable_shared_expert_fusion=False, experts=Experts(**vars(experts)),
        shared_expert_gate=SimpleNamespace(weight=L["w_gate"].to(dev).view(1, -1), bias=None),
        _forward_shared_experts=fwd_shared), lw


@pytest.fixture(scope="module")
def cfg1_layer(cuda):
    cfg = synthetic.CONFIGS[1]
    return cfg, synthetic.make_moe_layer(cfg)


def test_dual_shared_expert_in_kernel(cuda, cfg1_layer):
    cfg, L = cfg1_layer
    block, lw = _block(cfg, L, cuda)
    x = synthetic.make_tokens(cfg, device=cuda)
    assert overlay.why_not(block, x) is None and overlay._a16_ok(block, x)
    out, sh = overlay.dual(block, x)
    out2, _ = overlay.dual(block, x)                     # the cached workspace and repacked shared weights again
    torch.cuda.synchronize()
    assert sh is None and torch.equal(out, out2)
    assert block._qf_a16sh is not None and block._qf_a16sh[2] == cfg.Is
    # the same launch as the library's layer-step on the same weights
    full = MoELayerWeights.from_canonical(L["router"].to(cuda), L["w13"].to(cuda), L["s13"].to(cuda),
                                          L["w2"].to(cuda), L["s2"].to(cuda), L["w_gate"].to(cuda),
                                          L["sh_gu"].to(cuda), L["sh_d"].to(cuda))
    bufs = ops.moe_workspace(cfg.M, cfg.H, cfg.I, cfg.topk, cfg.Is, cuda)
    ref_out, tw, ids, _ = ops.moe_layer_step(x, full, cfg.topk, bufs, ops.router_bufs(cuda), torch.empty_like(x))
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out)
    C = {k: v.cpu() for k, v in L.items()}
    ref = moe_ref.moe_rounded(x.cpu(), ids.cpu(), tw.cpu(), C["w13"], C["s13"], C["w2"], C["s2"], w_gate=C["w_gate"],
                              shared_w=(C["sh_gu"], C["sh_d"]))
    d = out.float().cpu() - ref.float()
    assert bool((d.abs() <= 2e-2 + 2.0 ** -6 * ref.float().abs()).all()) and (d.norm() / ref.float().norm()) <= 1e-2


def test_dual_precomputed_shared_and_stock_experts(cuda, cfg1_layer):
    cfg, L = cfg1_layer
    x = synthetic.make_tokens(cfg, device=cuda, seed=9)
    C = {k: v.cpu() for k, v in L.items()}
    # shared expert outside the kernel (activation not SiluAndMul): its ungated output is passed in
    block, _ = _block(cfg, L, cuda, shared_act=object)
    out, sh = overlay.dual(block, x)
    torch.cuda.synchronize()
    assert sh is None and block._qf_a16sh is None
    r = block._qf_topk                                   # the routing of that launch (fused router)
    shared = moe_ref.shared_expert_bf16(x.cpu(), C["sh_gu"], C["sh_d"])
    ref = moe_ref.moe_rounded(x.cpu(), r.topk_ids.cpu(), r.topk_weights.cpu(), C["w13"], C["s13"], C["w2"], C["s2"],
                              shared=shared, w_gate=C["w_gate"])
    d = out.float().cpu() - ref.float()
    assert bool((d.abs() <= 2e-2 + 2.0 ** -6 * ref.float().abs()).all()) and (d.norm() / ref.float().norm()) <= 1e-2
    # experts not in the kernel's format: the router kernel, then the block's own experts module
    block, _ = _block(cfg, L, cuda, kernel_experts=False)
    assert not overlay._a16_ok(block, x)
    w, ids, _ = ops.router_topk(x, L["router"].to(cuda), cfg.topk, True, *ops.router_bufs(cuda))
    routed, sh = overlay.dual(block, x)
    torch.cuda.synchronize()
    assert len(block.experts.calls) == 1
    t = block.experts.calls[0]
    assert torch.equal(t.topk_ids, ids) and torch.equal(t.topk_weights, w) and block._qf_topk is t
    assert routed.shape == x.shape and sh.shape == x.shape


def test_dual_nvfp4_experts(cuda):
    """The block with NVFP4 experts (the reference's format, repacked by formats.repack_nvfp4): ``dual`` runs the
    router op and then the NVFP4 MoE op, as the reference's dual does; the result equals that op called directly and
    the oracle within tolerance."""
    from oracle import nvfp4_ref
    from qwenfast_b200 import formats
    E, H, I, topk, M, Is = 64, 2048, 512, 10, 10, 512
    wp13, sf13, g13 = synthetic.make_nvfp4_experts(E, 2 * I, H, seed=1)
    wp2, sf2, g2 = synthetic.make_nvfp4_experts(E, H, I, seed=2)
    cfg = synthetic.MoEConfig("nvfp4-block", H, E, 128, topk, M, Is, 3)
    L = synthetic.make_moe_layer(cfg)                       # router, shared expert, gate
    block, _ = _block(cfg, {**L, "w13": L["w13"], "s13": L["s13"], "w2": L["w2"], "s2": L["s2"]}, cuda,
                      kernel_experts=False)
    wk13, sk13 = formats.repack_nvfp4(wp13.to(cuda), sf13.to(cuda), gated=True)
    wk2, sk2 = formats.repack_nvfp4(wp2.to(cuda), sf2.to(cuda), gated=False)
    gs13, gs2 = (1.0 / g13).to(BF).to(cuda), (1.0 / g2).to(BF).to(cuda)
    ex = block.experts
    ex.w13_weight, ex.w13_weight_scale, ex.w13_weight_scale_2 = wk13, sk13, gs13
    ex.w2_weight, ex.w2_weight_scale, ex.w2_weight_scale_2 = wk2, sk2, gs2
    x = synthetic.make_tokens(cfg, device=cuda, seed=4)
    assert overlay._a16_format(block) == "nvfp4" and overlay._a16_ok(block, x)
    out, sh = overlay.dual(block, x)
    torch.cuda.synchronize()
    r = block._qf_topk
    assert sh is None and not block.experts.calls
    w, ids, _ = ops.router_topk(x, block.gate.weight, topk, True, *ops.router_bufs(cuda))
    assert torch.equal(ids, r.topk_ids) and torch.equal(w, r.topk_weights)
    bufs = ops.moe_workspace(M, H, I, topk, Is, cuda)
    direct = torch.empty_like(x)
    shk = block._qf_a16sh
    ops.a16_moe_decode(x, ids, w, wk13, sk13, gs13, wk2, sk2, gs2, block.shared_expert_gate.weight.view(-1), None,
                       bufs["hbuf"], bufs["ybuf"], bufs["gl"], bufs["ctrl"], direct, 4, None, bufs["pbuf"], shk[0],
                       None, shk[1], None, bufs["shbuf"], fmt="nvfp4")
    torch.cuda.synchronize()
    assert torch.equal(out, direct)
    deq = lambda wp, sf: nvfp4_ref.dequant_nvfp4(wp, sf, 1.0)
    ref = moe_ref.moe_rounded(x.cpu(), ids.cpu(), w.cpu(), wp13, sf13, wp2, sf2, gs13=gs13.cpu(), gs2=gs2.cpu(),
                              dequant=deq, w_gate=L["w_gate"], shared_w=(L["sh_gu"], L["sh_d"]))
    d = out.float().cpu() - ref.float()
    assert bool((d.abs() <= 2e-2 + 2.0 ** -6 * ref.float().abs()).all()) and (d.norm() / ref.float().norm()) <= 1e-2
