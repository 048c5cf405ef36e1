"""The persistent MoE kernel on NVFP4 experts -- the reference's own expert format (e2m1 codes, one E4M3 scale per 16 k,
a per-expert global value g applied as the multiplier 1/g) -- against the CPU oracle: the layer with the kernel's
rounding points (oracle.moe_ref.moe_rounded with the NVFP4 dequantisation of oracle.nvfp4_ref, which is pinned to
the reference's own deq) within the layer tolerance, and the reference's fp32 truth (oracle.nvfp4_ref.truth,
serve/qwenfast/test_a16moe.py:138-148) within relative L2 1e-2."""
import pytest
import torch

from oracle import moe_ref, nvfp4_ref, router_ref
from qwenfast_b200 import formats, ops, synthetic

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def _assert_close(out, ref, truth=None):
    out = out.float().cpu()
    d = out - ref.float()
    tol = 2e-2 + 2.0 ** -6 * ref.float().abs()
    rel = (d.norm() / ref.float().norm()).item()
    assert bool((d.abs() <= tol).all()) and rel <= 1e-2, (d.abs().max().item(), rel)
    if truth is not None:
        rel_t = ((out - truth).norm() / truth.norm()).item()
        assert rel_t <= 1e-2, rel_t


def _layer(E, H, I, seed):
    g = torch.Generator().manual_seed(seed)
    w13, s13 = nvfp4_ref.random_nvfp4((E, 2 * I, H), g)
    w2, s2 = nvfp4_ref.random_nvfp4((E, H, I), g)
    g13 = (torch.rand(E, generator=g) * 200 + 100)[:, None].repeat(1, 2)   # gate and up share the global value
    g2 = torch.rand(E, generator=g) * 200 + 100
    router = (torch.randn(E, H, generator=g) * 0.02).to(BF)
    return dict(w13=w13, s13=s13, w2=w2, s2=s2, g13=g13, g2=g2, router=router)


@pytest.mark.parametrize("E,H,I,topk,M,Is", [(16, 256, 128, 4, 4, 0), (64, 2048, 512, 10, 10, 512),
                                             (64, 2048, 512, 10, 1, 0), (32, 768, 256, 6, 40, 128)])
def test_nvfp4_layer(cuda, E, H, I, topk, M, Is):
    C = _layer(E, H, I, seed=E + H + M)
    g = torch.Generator().manual_seed(7 + M)
    x = torch.randn(M, H, generator=g).to(BF)
    w, ids, _ = router_ref.router_topk(x, C["router"], topk, True)
    ids, w = ids.int().contiguous(), w.float().contiguous()
    wk13, sk13 = formats.repack_nvfp4(C["w13"].to(cuda), C["s13"].to(cuda), gated=True)
    wk2, sk2 = formats.repack_nvfp4(C["w2"].to(cuda), C["s2"].to(cuda), gated=False)
    gs13 = (1.0 / C["g13"][:, 0]).to(BF)
    gs2 = (1.0 / C["g2"]).to(BF)
    kw, shw = {}, (None, None)
    if Is:
        sh_gu = (torch.randn(2 * Is, H, generator=g) * 0.02).to(BF)
        sh_d = (torch.randn(H, Is, generator=g) * 0.02).to(BF)
        w_gate = (torch.randn(H, generator=g) * 0.02).to(BF)
        shw = (formats.repack_bf16(sh_gu.to(cuda), gated=True), formats.repack_bf16(sh_d.to(cuda), gated=False))
        kw = dict(w_gate=w_gate, shared_w=(sh_gu, sh_d))
    bufs = ops.moe_workspace(M, H, I, topk, Is, cuda)
    outs = []
    for _ in range(2):
        out = torch.empty(M, H, dtype=BF, device=cuda)
        ops.a16_moe_decode(x.to(cuda), ids.to(cuda), w.to(cuda), wk13, sk13, gs13.to(cuda), wk2, sk2, gs2.to(cuda),
                           kw["w_gate"].to(cuda) if Is else None, None, bufs["hbuf"], bufs["ybuf"], bufs["gl"],
                           bufs["ctrl"], out, 4, None, bufs["pbuf"], shw[0], None, shw[1], None, bufs["shbuf"],
                           fmt="nvfp4")
        outs.append(out)
    torch.cuda.synchronize()
    assert ops.moe_error_word(bufs["ctrl"]) == 0
    assert torch.equal(outs[0], outs[1])
    deq = lambda wp, sf: nvfp4_ref.dequant_nvfp4(wp, sf, 1.0)
    ref = moe_ref.moe_rounded(x, ids, w, C["w13"], C["s13"], C["w2"], C["s2"], gs13=gs13, gs2=gs2, dequant=deq, **kw)
    truth = None
    if not Is:
        truth = nvfp4_ref.truth(x, ids, w, C["w13"], C["s13"], C["g13"], C["w2"], C["s2"], C["g2"])
    _assert_close(outs[0], ref, truth)


@pytest.mark.parametrize("M", [1, 10])
def test_nvfp4_fused_router_layer_step(cuda, M):
    """NVFP4 experts with the router inside the launch (qf_moe_layer_decode_nvfp4): the logits equal the standalone
    router's bit for bit (the same arithmetic), so ids, weights and the layer output equal the two-launch path
    (router_topk, then the NVFP4 MoE op); ids are the oracle's given the logits."""
    E, H, I, topk = 64, 2048, 512, 10
    C = _layer(E, H, I, seed=90 + M)
    g = torch.Generator().manual_seed(91 + M)
    x = torch.randn(M, H, generator=g).to(BF).to(cuda)
    wk13, sk13 = formats.repack_nvfp4(C["w13"].to(cuda), C["s13"].to(cuda), gated=True)
    wk2, sk2 = formats.repack_nvfp4(C["w2"].to(cuda), C["s2"].to(cuda), gated=False)
    gs13 = (1.0 / C["g13"][:, 0]).to(BF).to(cuda)
    gs2 = (1.0 / C["g2"]).to(BF).to(cuda)
    router = C["router"].to(cuda)
    bufs = ops.moe_workspace(M, H, I, topk, 0, cuda)
    tw = torch.empty(M, topk, dtype=torch.float32, device=cuda)
    ids = torch.empty(M, topk, dtype=torch.int32, device=cuda)
    lg = torch.empty(M, E, dtype=BF, device=cuda)
    out_f = torch.empty_like(x)
    ops.a16_moe_decode(x, ids, tw, wk13, sk13, gs13, wk2, sk2, gs2, None, None, bufs["hbuf"], bufs["ybuf"],
                       bufs["gl"], bufs["ctrl"], out_f, 4, None, bufs["pbuf"], None, None, None, None, bufs["shbuf"],
                       fmt="nvfp4", router_w=router, logits=lg)
    w2_, ids2, lg2 = ops.router_topk(x, router, topk, True, *ops.router_bufs(cuda))
    out_u = torch.empty_like(x)
    ops.a16_moe_decode(x, ids2, w2_, wk13, sk13, gs13, wk2, sk2, gs2, None, None, bufs["hbuf"], bufs["ybuf"],
                       bufs["gl"], bufs["ctrl"], out_u, 4, None, bufs["pbuf"], None, None, None, None, bufs["shbuf"],
                       fmt="nvfp4")
    torch.cuda.synchronize()
    assert ops.moe_error_word(bufs["ctrl"]) == 0
    assert torch.equal(lg, lg2)
    assert torch.equal(ids, ids2) and torch.equal(tw, w2_) and torch.equal(out_f, out_u)
    ow, oids = router_ref.topk_from_logits(lg.cpu(), topk, True)
    assert torch.equal(ids.cpu(), oids)


@pytest.mark.parametrize("M", [1, 10])
def test_nvfp4_split_phases_equal_whole_layer(cuda, M):
    """The reference's split phases on NVFP4 experts: phase 1 (gate logits, gate_up + SwiGLU) then phase 2 (down,
    weighting, combine with a precomputed shared term) give the bits of the one-launch layer (phase 4)."""
    E, H, I, topk = 64, 2048, 512, 10
    C = _layer(E, H, I, seed=70 + M)
    g = torch.Generator().manual_seed(71 + M)
    x = torch.randn(M, H, generator=g).to(BF).to(cuda)
    shared = (torch.randn(M, H, generator=g) * 0.05).to(BF).to(cuda)
    w_gate = (torch.randn(H, generator=g) * 0.02).to(BF).to(cuda)
    wk13, sk13 = formats.repack_nvfp4(C["w13"].to(cuda), C["s13"].to(cuda), gated=True)
    wk2, sk2 = formats.repack_nvfp4(C["w2"].to(cuda), C["s2"].to(cuda), gated=False)
    gs13 = (1.0 / C["g13"][:, 0]).to(BF).to(cuda)
    gs2 = (1.0 / C["g2"]).to(BF).to(cuda)
    w, ids, _ = ops.router_topk(x, C["router"].to(cuda), topk, True, *ops.router_bufs(cuda))
    outs = {}
    for phases in ((4,), (1, 2)):
        bufs = ops.moe_workspace(M, H, I, topk, 0, cuda)
        out = torch.empty_like(x)
        for phase in phases:
            ops.a16_moe_decode(x, ids, w, wk13, sk13, gs13, wk2, sk2, gs2, w_gate, shared, bufs["hbuf"],
                               bufs["ybuf"], bufs["gl"], bufs["ctrl"], out, phase, None, bufs["pbuf"], None, None,
                               None, None, bufs["shbuf"], fmt="nvfp4")
        torch.cuda.synchronize()
        assert ops.moe_error_word(bufs["ctrl"]) == 0
        outs[phases] = out
    assert torch.equal(outs[(4,)], outs[(1, 2)])
