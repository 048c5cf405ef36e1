"""``torch.ops.qwenfast_b200`` and the FusedMoE adapter on the GPU: each op gives bit for bit what the ctypes op of
``qwenfast_b200.ops`` gives on the same inputs (both launch the same kernels), a ``torch.compile``d decode step
(``aot_eager``, ``fullgraph=True``) equals the eager one, and ``QwenFastW4A16MoEMethod`` -- create_weights,
process_weights_after_loading, apply_weights on a stub layer -- equals the MoE kernel called directly and the CPU
oracle within the MoE tolerance, for one-launch decode batches and for batches above 64 tokens (chunked)."""
from types import SimpleNamespace

import pytest
import torch

from oracle import moe_ref, w8_ref
from qwenfast_b200 import formats, ops, synthetic, torch_ops
from qwenfast_b200.ops import MoELayerWeights

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


@pytest.fixture(scope="module")
def qops(cuda):
    return torch_ops.load()


@pytest.fixture(scope="module")
def cfg1(cuda):
    cfg = synthetic.CONFIGS[1]
    L = synthetic.make_moe_layer(cfg, device=cuda)
    lw = MoELayerWeights.from_canonical(L["router"], L["w13"], L["s13"], L["w2"], L["s2"], L["w_gate"], L["sh_gu"],
                                        L["sh_d"])
    return cfg, L, lw


def _a16_both(qops, x, ids, tw, lw, cfg, shared_in_kernel):
    bufs = ops.moe_workspace(64, cfg.H, cfg.I, cfg.topk, cfg.Is if shared_in_kernel else 0, x.device)
    none = bufs["none"]
    a = torch.empty_like(x)
    ops.a16_moe_decode(x, ids, tw, lw.w13, lw.s13, None, lw.w2, lw.s2, None, lw.w_gate if shared_in_kernel else None,
                       None, bufs["hbuf"], bufs["ybuf"], bufs["gl"], bufs["ctrl"], a, 4, None, bufs["pbuf"],
                       lw.sh_w13 if shared_in_kernel else None, None, lw.sh_w2 if shared_in_kernel else None, None,
                       bufs["shbuf"])
    b = torch.empty_like(x)
    qops.a16_moe_decode(x, ids, tw, lw.w13, lw.s13, none, lw.w2, lw.s2, none,
                        lw.w_gate if shared_in_kernel else none, none, bufs["hbuf"], bufs["ybuf"], bufs["gl"],
                        bufs["ctrl"], b, 4, bufs["none_i64"], bufs["pbuf"], lw.sh_w13 if shared_in_kernel else none,
                        none, lw.sh_w2 if shared_in_kernel else none, none, bufs["shbuf"])
    torch.cuda.synchronize()
    ops.check_moe_error(bufs["ctrl"])
    return a, b


@pytest.mark.parametrize("M,shared_in_kernel", [(10, True), (1, False), (64, True)])
def test_a16_moe_decode_op_equals_python_op(qops, cfg1, M, shared_in_kernel):
    cfg, L, lw = cfg1
    x = synthetic.make_tokens(cfg, M=M, device=L["router"].device, seed=M)
    tw, ids, _ = ops.router_topk(x, lw.router, cfg.topk, True, *ops.router_bufs(x.device))
    a, b = _a16_both(qops, x, ids, tw, lw, cfg, shared_in_kernel)
    assert torch.equal(a, b)


def test_router_and_layer_ops_equal_python_ops(qops, cfg1):
    cfg, L, lw = cfg1
    dev = L["router"].device
    x = synthetic.make_tokens(cfg, device=dev, seed=21)
    scratch, counter = ops.router_bufs(dev)
    w0, i0, l0 = ops.router_topk(x, lw.router, cfg.topk, True, scratch, counter)
    w1, i1, l1 = qops.router_topk(x, lw.router, cfg.topk, True, scratch, counter, True)
    torch.cuda.synchronize()
    assert torch.equal(w0, w1) and torch.equal(i0, i1) and torch.equal(l0, l1)
    bufs = ops.moe_workspace(64, cfg.H, cfg.I, cfg.topk, cfg.Is, dev)
    none = bufs["none"]
    out_py = torch.empty_like(x)
    tw_py = torch.empty(cfg.M, cfg.topk, dtype=torch.float32, device=dev)
    ids_py = torch.empty(cfg.M, cfg.topk, dtype=torch.int32, device=dev)
    lg_py = torch.empty(cfg.M, cfg.E, dtype=BF, device=dev)
    ops.a16_moe_decode(x, ids_py, tw_py, lw.w13, lw.s13, None, lw.w2, lw.s2, None, lw.w_gate, None, bufs["hbuf"],
                       bufs["ybuf"], bufs["gl"], bufs["ctrl"], out_py, 4, None, bufs["pbuf"], lw.sh_w13, None,
                       lw.sh_w2, None, bufs["shbuf"], router_w=lw.router, logits=lg_py)
    out_op = torch.empty_like(x)
    tw, ids, lg = qops.moe_layer_decode(x, lw.router, True, lw.w13, lw.s13, none, lw.w2, lw.s2, none, lw.w_gate, none,
                                        lw.sh_w13, lw.sh_w2, cfg.topk, bufs["hbuf"], bufs["ybuf"], bufs["gl"],
                                        bufs["ctrl"], bufs["pbuf"], bufs["shbuf"], out_op)
    torch.cuda.synchronize()
    ops.check_moe_error(bufs["ctrl"])
    assert torch.equal(out_py, out_op) and torch.equal(tw_py, tw) and torch.equal(ids_py, ids)
    assert torch.equal(lg_py, lg) and torch.equal(ids, i0) and torch.equal(tw, w0)


def test_int8_ops_equal_python_ops(qops, cuda):
    g = torch.Generator(device="cpu").manual_seed(12)
    w = (torch.randn(1536, 2048, generator=g) * 0.02).to(BF)
    q, s = w8_ref.w8_quant(w)
    q, s = q.to(cuda), s.to(cuda)
    for M in (1, 7, 16, 40):
        x = torch.randn(M, 2048, generator=g).to(BF).to(cuda)
        assert torch.equal(ops.w8g_gemm(x, q, s), qops.w8g_gemm(x, q, s, 0))
    wa, wb = torch.empty(1536, 2048, dtype=BF, device=cuda), torch.empty(1536, 2048, dtype=BF, device=cuda)
    ops.w8g_unpack(q, s, wa)
    qops.w8g_unpack(q, s, wb)
    assert torch.equal(wa, wb)
    qa = torch.randint(-127, 128, (1024, 2048), generator=g, dtype=torch.int8)
    sw = (torch.rand(1024, generator=g) * 1e-3 + 1e-4).to(cuda)
    qk = formats.repack_w8(qa.to(cuda))
    for M in (1, 9, 16):
        x = torch.randn(M, 2048, generator=g).to(BF).to(cuda)
        assert torch.equal(ops.w8a8_gemm(x, qk, sw), qops.w8a8_gemm(x, qk, sw))
    torch.cuda.synchronize()
    assert ops.w8g_take_status() == 0


def test_compiled_decode_step_equals_eager(qops, cfg1):
    """Router op, MoE op (in place, shared expert in the kernel) and a W8A16 projection as one ``torch.compile``d
    function (aot_eager, fullgraph): the same result as the same ops run eagerly."""
    cfg, L, lw = cfg1
    dev = L["router"].device
    g = torch.Generator(device="cpu").manual_seed(5)
    q, s = w8_ref.w8_quant((torch.randn(1024, cfg.H, generator=g) * 0.02).to(BF))
    q, s = q.to(dev), s.to(dev)
    bufs = ops.moe_workspace(64, cfg.H, cfg.I, cfg.topk, cfg.Is, dev)
    scratch, counter = ops.router_bufs(dev)
    none = bufs["none"]

    def step(x):
        tw, ids, _ = qops.router_topk(x, lw.router, cfg.topk, True, scratch, counter, True)
        out = torch.empty_like(x)
        qops.a16_moe_decode(x, ids, tw, lw.w13, lw.s13, none, lw.w2, lw.s2, none, lw.w_gate, none, bufs["hbuf"],
                            bufs["ybuf"], bufs["gl"], bufs["ctrl"], out, 4, bufs["none_i64"], bufs["pbuf"], lw.sh_w13,
                            none, lw.sh_w2, none, bufs["shbuf"])
        return out, qops.w8g_gemm(out, q, s, 0)

    x = synthetic.make_tokens(cfg, device=dev, seed=33)
    eager = step(x)
    compiled = torch.compile(step, backend="aot_eager", fullgraph=True)
    for _ in range(2):   # twice: the zero-kept counters are re-armed through the functionalized copies
        got = compiled(x)
        torch.cuda.synchronize()
        assert torch.equal(got[0], eager[0]) and torch.equal(got[1], eager[1])
    ops.check_moe_error(bufs["ctrl"])
    assert int(bufs["ctrl"][:ops._lib.QF_MOE_CTRL_MIRROR].abs().sum().item()) == 0


class _Layer(torch.nn.Module):
    pass


@pytest.mark.parametrize("M", [10, 100])
def test_fused_moe_adapter_on_a_stub_layer(cfg1, M):
    from qwenfast_b200.fused_moe import QwenFastW4A16MoEMethod
    cfg, L, lw = cfg1
    dev = L["router"].device
    method = QwenFastW4A16MoEMethod()
    layer = _Layer()
    method.create_weights(layer, cfg.E, cfg.H, cfg.I, params_dtype=BF)
    for name, key in (("w13_qweight", "w13"), ("w13_scales", "s13"), ("w2_qweight", "w2"), ("w2_scales", "s2")):
        p = getattr(layer, name)
        p.data = L[key].clone()   # the loader's copy into the created parameter
    method.process_weights_after_loading(layer)
    assert not hasattr(layer, "w13_qweight") and layer.w13_weight.dim() == 2
    assert torch.equal(layer.w13_weight, lw.w13) and torch.equal(layer.w2_weight_scale, lw.s2)
    x = synthetic.make_tokens(cfg, M=M, device=dev, seed=40 + M)
    tw, ids, _ = ops.router_topk(x[:64], lw.router, cfg.topk, True, *ops.router_bufs(dev))
    if M > 64:
        tw2, ids2, _ = ops.router_topk(x[64:], lw.router, cfg.topk, True, *ops.router_bufs(dev))
        tw, ids = torch.cat([tw, tw2]), torch.cat([ids, ids2])
    disp = SimpleNamespace(hidden_states=x, topk_output=SimpleNamespace(topk_ids=ids.long(), topk_weights=tw))
    got = method.apply_weights(layer, disp).hidden_states
    torch.cuda.synchronize()
    assert got.shape == x.shape and got.dtype == BF
    # the kernel called directly, one launch per 64 tokens, routed experts only
    bufs = ops.moe_workspace(64, cfg.H, cfg.I, cfg.topk, 0, dev)
    direct = torch.empty_like(x)
    for m0 in range(0, M, 64):
        sl = slice(m0, min(M, m0 + 64))
        ops.a16_moe_decode(x[sl], ids[sl], tw[sl], lw.w13, lw.s13, None, lw.w2, lw.s2, None, None, None, bufs["hbuf"],
                           bufs["ybuf"], bufs["gl"], bufs["ctrl"], direct[sl], 4, None, bufs["pbuf"], None, None,
                           None, None, bufs["shbuf"])
    torch.cuda.synchronize()
    assert torch.equal(got, direct)
    assert torch.equal(method.apply(layer, x, disp.topk_output), got)
    C = {k: v.cpu() for k, v in L.items()}
    ref = moe_ref.moe_rounded(x.cpu(), ids.cpu(), tw.cpu(), C["w13"], C["s13"], C["w2"], C["s2"])
    d = got.float().cpu() - ref.float()
    assert bool((d.abs() <= 2e-2 + 2.0 ** -6 * ref.float().abs()).all()) and (d.norm() / ref.float().norm()) <= 1e-2
    # the repack is exact: the canonical checkpoint tensors come back
    q13, s13 = formats.unpack_w4(layer.w13_weight, layer.w13_weight_scale, 2 * cfg.I, cfg.H, gated=True)
    assert torch.equal(q13, L["w13"]) and torch.equal(s13, L["s13"])
