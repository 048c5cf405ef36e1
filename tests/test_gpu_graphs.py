"""The decode ops under CUDA-graph capture and replay, the way the reference runs them (its verify step is one captured
graph: serve/qwenfast/test_a16moe.py:191-206 times graph replays). Each op is captured once on static buffers,
then replayed for several different inputs copied into those buffers; every replay must give the same bits as the
eager call on the same input (control words re-armed by the kernels, no host state baked into the graph)."""
import pytest
import torch

from qwenfast_b200._lib import QF_MOE_CTRL_MIRROR

from oracle import w8_ref
from qwenfast_b200 import formats, ops, synthetic
from qwenfast_b200.ops import MoELayerWeights

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def capture(fn):
    """Warm up on a side stream (launch attributes are cached there), then capture ``fn`` once."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g


@pytest.fixture(scope="module")
def layer(cuda):
    cfg = synthetic.CONFIGS[1]
    L = synthetic.make_moe_layer(cfg, device=cuda)
    lw = MoELayerWeights.from_canonical(L["router"], L["w13"], L["s13"], L["w2"], L["s2"], L["w_gate"], L["sh_gu"],
                                        L["sh_d"])
    return cfg, lw


@pytest.mark.parametrize("fused", [True, False])
def test_layer_step_graph_replays_equal_eager(cuda, layer, fused):
    """The layer-step (router inside the MoE launch, or router op + MoE op) captured once, replayed on new tokens."""
    cfg, lw = layer
    bufs = ops.moe_workspace(cfg.M, cfg.H, cfg.I, cfg.topk, cfg.Is, cuda)
    rb = ops.router_bufs(cuda)
    x = torch.empty(cfg.M, cfg.H, dtype=BF, device=cuda)
    out = torch.empty_like(x)
    res = {}

    def step():
        res["r"] = ops.moe_layer_step(x, lw, cfg.topk, bufs, rb, out, fused=fused)

    x.copy_(synthetic.make_tokens(cfg, device=cuda, seed=1))
    g = capture(step)
    for seed in (2, 3, 4):
        xs = synthetic.make_tokens(cfg, device=cuda, seed=seed)
        x.copy_(xs)
        g.replay()
        torch.cuda.synchronize()
        got = [t.clone() for t in res["r"]]
        eb = ops.moe_workspace(cfg.M, cfg.H, cfg.I, cfg.topk, cfg.Is, cuda)
        want = ops.moe_layer_step(xs, lw, cfg.topk, eb, ops.router_bufs(cuda), torch.empty_like(xs), fused=fused)
        torch.cuda.synchronize()
        for a, b in zip(got, want):
            assert torch.equal(a, b), seed
        assert ops.moe_error_word(bufs["ctrl"]) == 0
    assert int(bufs["ctrl"][:QF_MOE_CTRL_MIRROR].abs().sum().item()) == 0
    del g


def test_int8_gemms_graph_replays_equal_eager(cuda):
    g0 = torch.Generator(device="cpu").manual_seed(11)
    K, N, M = 2048, 4096, 10
    w = (torch.randn(N, K, generator=g0) * 0.02).to(BF)
    q, s = w8_ref.w8_quant(w)
    q, s = q.to(cuda), s.to(cuda)
    q8 = torch.randint(-127, 128, (N, K), generator=g0, dtype=torch.int8).to(cuda)
    qk = formats.repack_w8(q8)
    sw = (torch.rand(N, generator=g0) * 1e-3 + 1e-4).to(cuda)
    xq = torch.empty(16 * K, dtype=torch.int8, device=cuda)
    sx = torch.empty(M, dtype=torch.float32, device=cuda)
    fix = ops.w8a8_fixup(N, cuda)
    x = torch.empty(M, K, dtype=BF, device=cuda)
    res = {}

    def run():
        res["w8g"] = ops.w8g_gemm(x, q, s, 0, pdl=True)
        res["w8a8"] = ops.w8a8_gemm(x, qk, sw, xq=xq, sx=sx, fixup=fix)

    x.copy_(torch.randn(M, K, generator=g0).to(BF))
    graph = capture(run)
    for _ in range(3):
        xs = torch.randn(M, K, generator=g0).to(BF).to(cuda)
        x.copy_(xs)
        graph.replay()
        torch.cuda.synchronize()
        a, b = res["w8g"].clone(), res["w8a8"].clone()
        assert torch.equal(a, ops.w8g_gemm(xs, q, s, 0))
        assert torch.equal(b, ops.w8a8_gemm(xs, qk, sw))
        torch.cuda.synchronize()
    assert ops.w8a8_take_status() == 0
    assert int(fix.abs().sum().item()) == 0   # the split-K fixup buffer is left zero-filled after every replay
    del graph
