"""The torch custom operators (``torch.ops.qwenfast_b200``) and the FusedMoE quant-method adapter, without a GPU:
every op is registered with a CUDA and a Meta kernel, the Meta kernels give the reference's output shapes, every
in-place op can be functionalized, a function calling the ops traces as one graph under ``torch.compile``
(``aot_eager``, ``fullgraph=True``) on meta tensors, and the adapter's ``create_weights`` lays out the canonical
checkpoint parameters (compressed_tensors_w4a4_nvfp4_moe.py:62-95 is the slot it fills)."""
from types import SimpleNamespace

import pytest
import torch

BF = torch.bfloat16


@pytest.fixture(scope="module")
def qops(lib):
    from qwenfast_b200 import build, torch_ops
    build.build_torch_ops()
    return torch_ops.load()


def test_ops_registered_with_cuda_and_meta_kernels(qops):
    import torch._higher_order_ops.auto_functionalize as af
    from qwenfast_b200 import torch_ops
    for name in torch_ops.OP_NAMES:
        full = f"qwenfast_b200::{name}"
        assert torch._C._dispatch_has_kernel_for_dispatch_key(full, "CUDA"), name
        assert torch._C._dispatch_has_kernel_for_dispatch_key(full, "Meta"), name
        op = getattr(qops, name).default
        if op._schema.is_mutable:   # in-place ops return nothing aliased, so compile can functionalize them
            assert af.can_auto_functionalize(op), name


def _meta_layer(M=5, H=2048, E=512, I=512, topk=10, Is=512):
    d = "meta"
    t = lambda *s, dt=BF: torch.empty(*s, dtype=dt, device=d)   # noqa: E731
    return dict(x=t(M, H), router=t(E, H), w13=t(E, 2 * I * H // 8, dt=torch.int32), s13=t(E, 2 * I * H // 128),
                w2=t(E, H * I // 8, dt=torch.int32), s2=t(E, H * I // 128), wg=t(H), none=t(0),
                shw13=t(2 * Is * H), shw2=t(H * Is), hbuf=t(1 << 20), ybuf=t(1 << 20), gl=t(4096, dt=torch.float32),
                ctrl=t(2048, dt=torch.int32), pbuf=t(4096, dt=torch.float32), shbuf=t(1 << 16),
                none_i64=t(0, dt=torch.int64), ids=t(M, topk, dt=torch.int32), tw=t(M, topk, dt=torch.float32),
                scratch=t(64 * 1024, dt=torch.float32), counter=t(1, dt=torch.int32))


def test_meta_kernels_give_the_reference_shapes(qops):
    L = _meta_layer()
    tw, ids, logits = qops.router_topk(L["x"], L["router"], 10, True, L["scratch"], L["counter"], True)
    assert (tw.shape, tw.dtype, ids.shape, ids.dtype, logits.shape, logits.dtype) == \
        ((5, 10), torch.float32, (5, 10), torch.int32, (5, 512), BF)
    tw, ids, logits = qops.moe_layer_decode(L["x"], L["router"], True, L["w13"], L["s13"], L["none"], L["w2"], L["s2"],
                                            L["none"], L["wg"], L["none"], L["shw13"], L["shw2"], 10, L["hbuf"],
                                            L["ybuf"], L["gl"], L["ctrl"], L["pbuf"], L["shbuf"], torch.empty_like(L["x"]))
    assert (tw.shape, ids.shape, logits.shape) == ((5, 10), (5, 10), (5, 512))
    x = torch.empty(7, 6144, dtype=BF, device="meta")
    y = qops.w8g_gemm(x, torch.empty(1024, 6144, dtype=torch.int8, device="meta"),
                      torch.empty(1024, 48, dtype=BF, device="meta"))
    assert (y.shape, y.dtype) == ((7, 1024), BF)
    y = qops.w8a8_gemm(x, torch.empty(512, 6144, dtype=torch.int8, device="meta"),
                       torch.empty(512, dtype=torch.float32, device="meta"))
    assert (y.shape, y.dtype) == ((7, 512), BF)


def test_compile_traces_the_decode_step_as_one_graph(qops):
    """Router op -> MoE op (in place) -> W8A16 projection, under ``torch.compile(fullgraph=True)``: one graph, no
    break, output shapes from the Meta kernels."""
    graphs = []

    def counting_backend(gm, example_inputs):
        graphs.append(gm)
        from torch._dynamo.backends.common import aot_autograd
        from functorch.compile import make_boxed_func
        return aot_autograd(fw_compiler=lambda g, _: make_boxed_func(g.forward))(gm, example_inputs)

    L = _meta_layer()
    q8 = torch.empty(1024, 2048, dtype=torch.int8, device="meta")
    s8 = torch.empty(1024, 16, dtype=BF, device="meta")

    def step(x, router, w13, s13, w2, s2, wg, none, shw13, shw2, hbuf, ybuf, gl, ctrl, pbuf, shbuf, none_i64,
             scratch, counter):
        tw, ids, _ = qops.router_topk(x, router, 10, True, scratch, counter, True)
        out = torch.empty_like(x)
        qops.a16_moe_decode(x, ids, tw, w13, s13, none, w2, s2, none, wg, none, hbuf, ybuf, gl, ctrl, out, 4, none_i64,
                            pbuf, shw13, none, shw2, none, shbuf)
        return qops.w8g_gemm(out, q8, s8, 0)

    args = [L[k] for k in ("x", "router", "w13", "s13", "w2", "s2", "wg", "none", "shw13", "shw2", "hbuf", "ybuf",
                           "gl", "ctrl", "pbuf", "shbuf", "none_i64", "scratch", "counter")]
    y = torch.compile(step, backend=counting_backend, fullgraph=True)(*args)
    assert y.shape == (5, 1024) and y.dtype == BF
    assert len(graphs) == 1
    targets = {str(n.target) for n in graphs[0].graph.nodes if n.op == "call_function"}
    assert any("a16_moe_decode" in t for t in targets) and any("router_topk" in t for t in targets)


class _Layer(torch.nn.Module):
    pass


def test_adapter_create_weights_lays_out_the_checkpoint_parameters():
    from qwenfast_b200.fused_moe import QwenFastW4A16MoEMethod, _combine_input
    m = QwenFastW4A16MoEMethod()
    layer = _Layer()
    loader = object()
    m.create_weights(layer, num_experts=8, hidden_size=512, intermediate_size_per_partition=256,
                     params_dtype=BF, weight_loader=loader)
    shapes = {n: (tuple(p.shape), p.dtype) for n, p in layer.named_parameters()}
    assert shapes == {"w13_qweight": ((8, 512, 64), torch.int32), "w13_scales": ((8, 512, 4), BF),
                      "w2_qweight": ((8, 512, 32), torch.int32), "w2_scales": ((8, 512, 2), BF)}
    assert all(p.weight_loader is loader and not p.requires_grad for p in layer.parameters())
    with pytest.raises(RuntimeError, match="multiple"):
        m.create_weights(_Layer(), 8, 500, 256)
    with pytest.raises(RuntimeError, match="group-128"):
        QwenFastW4A16MoEMethod(group_size=64)
    ci = _combine_input(torch.zeros(2, 3))
    assert ci.hidden_states.shape == (2, 3)
    # the routed output needs the CUDA kernel: a CPU call fails loudly instead of falling back
    d = SimpleNamespace(hidden_states=torch.zeros(2, 512, dtype=BF),
                        topk_output=SimpleNamespace(topk_ids=torch.zeros(2, 4, dtype=torch.int32),
                                                    topk_weights=torch.zeros(2, 4)))
    with pytest.raises(RuntimeError, match="CUDA"):
        m.apply_weights(layer, d)
