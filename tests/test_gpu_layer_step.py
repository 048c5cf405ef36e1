"""ops.LayerStep (the prepared layer-step call) against ops.moe_layer_step: the same launch with the same arguments,
so the outputs are the same bits -- for device and pinned-host x / out, for several M on one workspace, on the
declined-fused path, and with an error reported through the workspace's host mirror."""
import pytest
import torch

from qwenfast_b200 import _lib, ops, synthetic
from qwenfast_b200.ops import LayerStep, MoELayerWeights

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def layer(cfg, dev):
    L = synthetic.make_moe_layer(cfg, device=dev)
    return MoELayerWeights.from_canonical(L["router"], L["w13"], L["s13"], L["w2"], L["s2"], L.get("w_gate"),
                                          L.get("sh_gu"), L.get("sh_d"))


def test_layer_step_equals_moe_layer_step(cuda):
    cfg = synthetic.CONFIGS[1]
    lw = layer(cfg, cuda)
    bufs = ops.moe_workspace(64, cfg.H, cfg.I, cfg.topk, cfg.Is, cuda)
    step = LayerStep(lw, cfg.topk, bufs)
    xs = torch.empty(64, cfg.H, dtype=BF, device=cuda)
    for M, seed in ((10, 51), (1, 52), (64, 53), (10, 54)):
        x = synthetic.make_tokens(cfg, M=M, device=cuda, seed=seed)
        ref = torch.empty_like(x)
        _, tw_r, ids_r, lg_r = ops.moe_layer_step(x, lw, cfg.topk, bufs, None, ref)
        tw_r, ids_r, lg_r = tw_r.clone(), ids_r.clone(), lg_r.clone()
        out = torch.empty_like(x)
        o, tw, ids, lg = step(x, out)
        torch.cuda.synchronize()
        assert o is out and tw.shape == (M, cfg.topk) and lg.shape == (M, cfg.E)
        assert torch.equal(out, ref) and torch.equal(ids, ids_r) and torch.equal(tw, tw_r) and torch.equal(lg, lg_r)
        # pinned host x / out through x_stage
        xh = x.cpu().pin_memory()
        oh = torch.empty(M, cfg.H, dtype=BF).pin_memory()
        step(xh, oh, x_stage=xs[:M])
        torch.cuda.synchronize()
        assert torch.equal(oh, ref.cpu())
        assert ops.moe_error_word(bufs["ctrl"]) == 0


def test_layer_step_checks_its_arguments(cuda):
    cfg = synthetic.CONFIGS[1]
    lw = layer(cfg, cuda)
    bufs = ops.moe_workspace(cfg.M, cfg.H, cfg.I, cfg.topk, cfg.Is, cuda)
    step = LayerStep(lw, cfg.topk, bufs)
    x = synthetic.make_tokens(cfg, device=cuda, seed=5)
    with pytest.raises(RuntimeError, match="x must be"):
        step(x.float(), torch.empty_like(x))
    with pytest.raises(RuntimeError, match="out must be"):
        step(x, torch.empty(cfg.M + 1, cfg.H, dtype=BF, device=cuda))
    with pytest.raises(RuntimeError, match="pinned host"):
        step(x.cpu(), torch.empty_like(x), x_stage=torch.empty_like(x))
    with pytest.raises(RuntimeError, match="topk"):
        LayerStep(lw, 0, bufs)
    bad = dict(bufs)
    del bad["pbuf"]
    with pytest.raises(RuntimeError, match="pbuf"):
        LayerStep(lw, cfg.topk, bad)


def test_layer_step_reports_a_mirrored_error_and_recovers(cuda):
    """An error word in the workspace's host mirror (set here on the host, as a launch that ran out of a bounded
    wait would leave it) makes the next call raise and reset the workspace; the call after that computes normally."""
    cfg = synthetic.CONFIGS[1]
    lw = layer(cfg, cuda)
    bufs = ops.moe_workspace(cfg.M, cfg.H, cfg.I, cfg.topk, cfg.Is, cuda)
    step = LayerStep(lw, cfg.topk, bufs)
    x = synthetic.make_tokens(cfg, device=cuda, seed=7)
    ref = torch.empty_like(x)
    ops.moe_layer_step(x, lw, cfg.topk, bufs, None, ref)
    torch.cuda.synchronize()
    bufs["err_host"][0] = _lib.QF_MOE_ERR_TIMEOUT
    with pytest.raises(RuntimeError, match="earlier launch"):
        step(x, torch.empty_like(x))
    assert int(bufs["err_host"][0]) == 0
    out = torch.empty_like(x)
    step(x, out)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


def test_layer_step_declined_fused_launch_takes_the_two_launch_path(cuda, monkeypatch):
    cfg = synthetic.CONFIGS[1]
    lw = layer(cfg, cuda)
    x = synthetic.make_tokens(cfg, device=cuda, seed=9)
    bufs = ops.moe_workspace(cfg.M, cfg.H, cfg.I, cfg.topk, cfg.Is, cuda)
    ref = torch.empty_like(x)
    _, tw_r, ids_r, _ = ops.moe_layer_step(x, lw, cfg.topk, bufs, ops.router_bufs(cuda), ref, fused=False)
    torch.cuda.synchronize()
    lib = _lib.load()

    class Refusing:   # the library with a fused entry that declines, everything else forwarded
        def __getattr__(self, name):
            return getattr(lib, name)

        @staticmethod
        def qf_moe_layer_decode(*args):
            return _lib.QF_ERR_UNSUPPORTED

    monkeypatch.setattr(_lib, "load", lambda *a, **k: Refusing())
    step = LayerStep(lw, cfg.topk, bufs)
    for _ in range(2):   # the first call is declined and remembered; the second goes straight to two launches
        out = torch.empty_like(x)
        _, tw, ids, _ = step(x, out)
        torch.cuda.synchronize()
        assert torch.equal(out, ref) and torch.equal(ids, ids_r) and torch.equal(tw, tw_r)
    assert step._fused is False
