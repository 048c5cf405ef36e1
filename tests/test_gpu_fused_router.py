"""The MoE launch with the router inside (C ABI qf_moe_layer_decode) vs the CPU oracle and vs the two-launch path.

Router part, by the protocol of the router tests (serve/qwenfast/test_router.py:41-43): the kernel's bf16 logits
within one bf16 ulp of the oracle's (or, where the dot product cancels, within 4 fp32 ulps of sum |x w|), top-k ids bit-exact given the kernel's own logits, weights within fp32
tolerance; on integer-valued inputs (exact logits, heavy ties) the ids equal the oracle's outright. Layer part: the
output is bit-identical to a16_moe_decode given the fused launch's own ids and weights (the same kernel after the
routing), and within the MoE tolerances of the oracle."""
import pytest
import torch

from qwenfast_b200._lib import QF_MOE_CTRL_MIRROR

from oracle import moe_ref, router_ref
from qwenfast_b200 import ops, synthetic
from qwenfast_b200.ops import MoELayerWeights

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def layer(cfg, dev, router=None):
    L = synthetic.make_moe_layer(cfg, device=dev)
    if router is not None:
        L["router"] = router.to(dev)
    lw = MoELayerWeights.from_canonical(L["router"], L["w13"], L["s13"], L["w2"], L["s2"], L.get("w_gate"),
                                        L.get("sh_gu"), L.get("sh_d"))
    return L, lw


def fused_step(x, lw, topk, renorm, Is):
    M, H = x.shape
    bufs = ops.moe_workspace(M, H, lw.I, topk, Is, x.device)
    out = torch.empty_like(x)
    _, tw, ids, lg = ops.moe_layer_step(x, lw, topk, bufs, None, out, renormalize=renorm)
    torch.cuda.synchronize()
    assert ops.moe_error_word(bufs["ctrl"]) == 0
    assert int(bufs["ctrl"][:QF_MOE_CTRL_MIRROR].abs().sum().item()) == 0, "control block (barrier counter included) must be re-armed"
    return out, tw, ids, lg, bufs


def check_router(x, lw, tw, ids, lg, topk, renorm, exact_logits=False):
    ref = router_ref.router_logits(x.cpu(), lw.router.cpu()).float()
    got = lg.float().cpu()
    if exact_logits:
        assert torch.equal(got, ref)
    else:
        # one bf16 ulp, or 4 fp32 ulps of sum_k |x w| where the sum cancels (the two fp32 summation orders differ)
        scale = (x.cpu().float().abs() @ lw.router.cpu().float().abs().T)
        tol = torch.maximum(ref.abs(), got.abs()) * 2.0 ** -7 + scale * 2.0 ** -21
        bad = ((got - ref).abs() > tol).nonzero()
        detail = [(int(t), int(e), float(ref[t, e]), float(got[t, e]), float(scale[t, e])) for t, e in bad[:8]]
        assert bad.shape[0] == 0, f"{bad.shape[0]} logits differ by more than one bf16 ulp: {detail}"
    ow, oids = router_ref.topk_from_logits(lg.cpu(), topk, renorm)
    assert torch.equal(ids.cpu(), oids), "top-k ids must be bit-exact given the kernel logits"
    torch.testing.assert_close(tw.cpu(), ow, rtol=3e-5, atol=1e-6)


def check_layer(x, lw, tw, ids, out, bufs, L, Is):
    ref2 = torch.empty_like(x)
    ops.a16_moe_decode(x, ids, tw, lw.w13, lw.s13, None, lw.w2, lw.s2, None, lw.w_gate, None, bufs["hbuf"],
                       bufs["ybuf"], bufs["gl"], bufs["ctrl"], ref2, 4, None, bufs["pbuf"], lw.sh_w13, None,
                       lw.sh_w2, None, bufs["shbuf"])
    torch.cuda.synchronize()
    assert torch.equal(out, ref2), "the fused launch must equal a16_moe_decode given its own routing"
    C = {k: v.cpu() for k, v in L.items()}
    kw = dict(w_gate=C["w_gate"], shared_w=(C["sh_gu"], C["sh_d"])) if Is else {}
    ref = moe_ref.moe_rounded(x.cpu(), ids.cpu(), tw.cpu(), C["w13"], C["s13"], C["w2"], C["s2"], **kw)
    d = out.float().cpu() - ref.float()
    tol = 2e-2 + 2.0 ** -6 * ref.float().abs()
    assert bool((d.abs() <= tol).all()) and (d.norm() / ref.float().norm()).item() <= 1e-2


@pytest.mark.parametrize("H,E,I,topk,M,Is", [(2048, 512, 128, 10, 10, 512), (2048, 512, 128, 10, 1, 0),
                                             (2048, 512, 128, 10, 64, 0), (4096, 256, 128, 8, 3, 0),
                                             (2048, 1024, 128, 16, 5, 0), (256, 16, 128, 4, 4, 0)])
@pytest.mark.parametrize("renorm", [True, False])
def test_fused_router_layer(cuda, H, E, I, topk, M, Is, renorm):
    cfg = synthetic.MoEConfig("t", H, E, I, topk, M, Is, H + E + M)
    L, lw = layer(cfg, cuda)
    x = synthetic.make_tokens(cfg, device=cuda)
    out, tw, ids, lg, bufs = fused_step(x, lw, topk, renorm, Is)
    check_router(x, lw, tw, ids, lg, topk, renorm)
    check_layer(x, lw, tw, ids, out, bufs, L, Is)


def test_fused_router_ties_kat(cuda):
    """Integer router weights and sparse +-1 tokens: exact integer logits with many ties (the case generator of
    serve/qwenfast/test_router3.py:25-28); ids must equal the oracle's router outright."""
    cfg = synthetic.MoEConfig("ties", 2048, 512, 128, 10, 8, 0, 3)
    g = torch.Generator(device="cpu").manual_seed(1234)
    w = torch.randint(-2, 3, (cfg.E, cfg.H), generator=g).float().to(BF)
    L, lw = layer(cfg, cuda, router=w)
    x = (torch.randint(-1, 2, (cfg.M, cfg.H), generator=g).float() * (torch.rand(cfg.M, cfg.H, generator=g) < 0.002))
    x = x.to(BF).to(cuda)
    for renorm in (True, False):
        out, tw, ids, lg, bufs = fused_step(x, lw, cfg.topk, renorm, 0)
        check_router(x, lw, tw, ids, lg, cfg.topk, renorm, exact_logits=True)
        _, oids, _ = router_ref.router_topk(x.cpu(), w, cfg.topk, renorm)
        assert torch.equal(ids.cpu(), oids)
        check_layer(x, lw, tw, ids, out, bufs, L, 0)


def test_fused_matches_two_launch_path_and_back_to_back(cuda):
    """Config 1: the fused layer-step equals the router_topk + a16_moe_decode path wherever the two routers' logits
    agree (they are the same up to fp32 summation order); repeated launches without a sync are bit-identical."""
    cfg = synthetic.CONFIGS[1]
    L, lw = layer(cfg, cuda)
    x = synthetic.make_tokens(cfg, device=cuda, seed=21)
    bufs = ops.moe_workspace(cfg.M, cfg.H, cfg.I, cfg.topk, cfg.Is, cuda)
    rb = ops.router_bufs(cuda)
    out_f = torch.empty_like(x)
    out_u = torch.empty_like(x)
    _, tw_f, ids_f, lg_f = ops.moe_layer_step(x, lw, cfg.topk, bufs, rb, out_f)
    _, tw_u, ids_u, lg_u = ops.moe_layer_step(x, lw, cfg.topk, bufs, rb, out_u, fused=False)
    torch.cuda.synchronize()
    if torch.equal(lg_f, lg_u):
        assert torch.equal(ids_f, ids_u) and torch.equal(tw_f, tw_u) and torch.equal(out_f, out_u)
    outs = []
    for _ in range(4):
        o = torch.empty_like(x)
        outs.append(ops.moe_layer_step(x, lw, cfg.topk, bufs, rb, o))
    torch.cuda.synchronize()
    for o, tw, ids, lg in outs:
        assert torch.equal(o, out_f) and torch.equal(ids, ids_f) and torch.equal(tw, tw_f) and torch.equal(lg, lg_f)
    assert int(bufs["ctrl"][:QF_MOE_CTRL_MIRROR].abs().sum().item()) == 0


def test_fused_host_io_matches_device_io(cuda):
    """x read from pinned host memory by the kernel (staged into x_stage) and out written to pinned host memory:
    the same bits as the all-device call; a second step with new host tokens sees the new tokens (no stale copy)."""
    cfg = synthetic.CONFIGS[1]
    L, lw = layer(cfg, cuda)
    bufs = ops.moe_workspace(cfg.M, cfg.H, cfg.I, cfg.topk, cfg.Is, cuda)
    xs = torch.empty(cfg.M, cfg.H, dtype=BF, device=cuda)
    xh = torch.empty(cfg.M, cfg.H, dtype=BF).pin_memory()
    oh = torch.empty(cfg.M, cfg.H, dtype=BF).pin_memory()
    for seed in (31, 32):
        x = synthetic.make_tokens(cfg, device=cuda, seed=seed)
        out_d = torch.empty_like(x)
        _, tw_d, ids_d, lg_d = ops.moe_layer_step(x, lw, cfg.topk, bufs, None, out_d)
        xh.copy_(x.cpu())
        _, tw_h, ids_h, lg_h = ops.moe_layer_step(xh, lw, cfg.topk, bufs, None, oh, x_stage=xs)
        torch.cuda.synchronize()
        assert ops.moe_error_word(bufs["ctrl"]) == 0
        assert torch.equal(xs, x)
        assert torch.equal(ids_h, ids_d) and torch.equal(tw_h, tw_d) and torch.equal(lg_h, lg_d)
        assert torch.equal(oh, out_d.cpu())
    assert int(bufs["ctrl"][:QF_MOE_CTRL_MIRROR].abs().sum().item()) == 0


def test_declined_fused_launch_takes_the_two_launch_path(cuda, monkeypatch):
    """When the fused layer-step's cooperative grid cannot be co-resident, qf_moe_layer_decode returns
    QF_ERR_UNSUPPORTED (nothing enqueued) and moe_layer_step runs router_topk + a16_moe_decode instead -- for device
    buffers and for pinned host x / out. The refusal is simulated at the library boundary (a full B200 always
    co-schedules the grid)."""
    from qwenfast_b200 import _lib
    cfg = synthetic.CONFIGS[1]
    L, lw = layer(cfg, cuda)
    x = synthetic.make_tokens(cfg, device=cuda, seed=41)
    bufs = ops.moe_workspace(cfg.M, cfg.H, cfg.I, cfg.topk, cfg.Is, cuda)
    rb = ops.router_bufs(cuda)
    ref = torch.empty_like(x)
    _, tw_r, ids_r, lg_r = ops.moe_layer_step(x, lw, cfg.topk, bufs, rb, ref, fused=False)
    torch.cuda.synchronize()
    lib = _lib.load()

    class Refusing:   # the library with a fused entry that declines, everything else forwarded
        def __getattr__(self, name):
            return getattr(lib, name)

        @staticmethod
        def qf_moe_layer_decode(*args):
            return _lib.QF_ERR_UNSUPPORTED

    monkeypatch.setattr(_lib, "load", lambda *a, **k: Refusing())
    out = torch.empty_like(x)
    _, tw, ids, lg = ops.moe_layer_step(x, lw, cfg.topk, bufs, rb, out)
    xs = torch.empty_like(x)
    xh = x.cpu().pin_memory()
    oh = torch.empty(cfg.M, cfg.H, dtype=BF).pin_memory()
    ops.moe_layer_step(xh, lw, cfg.topk, bufs, rb, oh, x_stage=xs)
    torch.cuda.synchronize()
    assert torch.equal(out, ref) and torch.equal(ids, ids_r) and torch.equal(tw, tw_r) and torch.equal(lg, lg_r)
    assert torch.equal(oh, ref.cpu())
    assert ops.moe_error_word(bufs["ctrl"]) == 0
