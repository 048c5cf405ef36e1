"""The persistent W4A16 MoE kernel (+ shared expert + combine) vs the CPU oracle.

Tolerances: bf16 outputs within max-abs 2e-2 and relative L2 1e-2 of the fp32-accumulated
oracle that keeps the reference's bf16 rounding points (oracle.moe_ref.moe_rounded), and relative L2 1e-2 of the
all-fp32 truth (serve/qwenfast/test_a16moe.py:139-148). The routing fed to the oracle is the kernel router's own
ids and weights, so GEMM rounding in the router cannot flip an expert. Also checked, as in test_a16moe.py:163-178
and :235-237: batch invariance (rows together == rows one at a time, bit for bit), back-to-back launches equal to
synchronised ones, and the control block re-armed to zero after every launch."""
import os

import pytest
import torch

from qwenfast_b200._lib import QF_MOE_CTRL_MIRROR

from conftest import GOLDEN
from oracle import moe_ref
from qwenfast_b200 import formats, ops, synthetic
from qwenfast_b200.ops import MoELayerWeights

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def assert_close_to_oracle(out, ref_rounded, ref_truth=None, label=""):
    """max-abs 2e-2, widened elementwise by two bf16 ulps of the reference value (one output rounding step already
    exceeds 2e-2 once |out| >= 4), and relative L2 1e-2 against the rounded oracle. Against the all-fp32 truth:
    relative L2 1e-2 and max-abs <= max(2e-2, floor + one bf16 step of max|truth|), where floor = max|rounded oracle -
    truth| is what the reference's own rounding points already give (0.035 at config 1, up to 0.22 on the Zipf sweep
    where outputs reach |20|): no bf16-output kernel with those rounding points can meet a flat 2e-2 there. The
    measured max-abs against the truth is printed."""
    out = out.float().cpu()
    ref = ref_rounded.float()
    d = out - ref
    rel = (d.norm() / ref.norm()).item()
    tol = 2e-2 + 2.0 ** -6 * ref.abs()
    assert bool((d.abs() <= tol).all()) and rel <= 1e-2, (d.abs().max().item(), rel)
    if ref_truth is not None:
        tru = ref_truth.float()
        rel_t = ((out - tru).norm() / tru.norm()).item()
        max_t = (out - tru).abs().max().item()
        floor = (ref - tru).abs().max().item()
        bound = max(2e-2, floor + 2.0 ** -7 * tru.abs().max().item())
        print(f"[parity {label}] max|out-truth| {max_t:.4f} (reference rounding floor {floor:.4f}, bound {bound:.4f}), "
              f"rel-L2 {rel_t:.2e}, max|truth| {tru.abs().max().item():.2f}")
        assert rel_t <= 1e-2, rel_t
        assert max_t <= bound, (max_t, floor, bound)


def canon_cpu(L):
    return {k: v.cpu() for k, v in L.items()}


def layer_on(dev, L):
    return MoELayerWeights.from_canonical(L["router"].to(dev), L["w13"].to(dev), L["s13"].to(dev), L["w2"].to(dev),
                                          L["s2"].to(dev), L["w_gate"].to(dev) if "w_gate" in L else None,
                                          L["sh_gu"].to(dev) if "sh_gu" in L else None,
                                          L["sh_d"].to(dev) if "sh_d" in L else None)


def run_moe(x, ids, tw, lw, bufs, shared=None, gs13=None, gs2=None, use_shw=True, out=None):
    out = torch.empty_like(x) if out is None else out
    ops.a16_moe_decode(x, ids, tw, lw.w13, lw.s13, gs13, lw.w2, lw.s2, gs2, lw.w_gate, shared, bufs["hbuf"],
                       bufs["ybuf"], bufs["gl"], bufs["ctrl"], out, 4, None, bufs["pbuf"],
                       lw.sh_w13 if use_shw else None, None, lw.sh_w2 if use_shw else None, None, bufs["shbuf"])
    return out


@pytest.fixture(scope="module")
def cfg1(cuda):
    cfg = synthetic.CONFIGS[1]
    L = synthetic.make_moe_layer(cfg, device=cuda)
    lw = layer_on(cuda, L)
    return cfg, L, lw, canon_cpu(L)


def test_config0_against_golden(cuda):
    cfg = synthetic.CONFIGS[0]
    gold = torch.load(os.path.join(GOLDEN, "config0.pt"))
    L = synthetic.make_moe_layer(cfg)
    x = synthetic.make_tokens(cfg)
    from tests.golden.make_golden import checksum  # noqa: E402  (same checksum as the fixture writer)
    assert checksum(x, L["router"], L["w13"], L["s13"], L["w2"], L["s2"]) == gold["checksum"]
    lw = layer_on(cuda, L)
    bufs = ops.moe_workspace(cfg.M, cfg.H, cfg.I, cfg.topk, 0, cuda)
    out = run_moe(x.to(cuda), gold["ids"].to(cuda), gold["weights"].to(cuda), lw, bufs)
    torch.cuda.synchronize()
    assert_close_to_oracle(out, gold["out_rounded"], gold["out_truth"], "config0 golden")
    assert int(bufs["ctrl"][:QF_MOE_CTRL_MIRROR].abs().sum().item()) == 0


def test_config0_layer_step(cuda):
    cfg = synthetic.CONFIGS[0]
    L = synthetic.make_moe_layer(cfg)
    x = synthetic.make_tokens(cfg).to(cuda)
    lw = layer_on(cuda, L)
    bufs = ops.moe_workspace(cfg.M, cfg.H, cfg.I, cfg.topk, 0, cuda)
    rb = ops.router_bufs(cuda)
    out = torch.empty_like(x)
    _, tw, ids, _ = ops.moe_layer_step(x, lw, cfg.topk, bufs, rb, out)
    torch.cuda.synchronize()
    ref = moe_ref.moe_rounded(x.cpu(), ids.cpu(), tw.cpu(), L["w13"], L["s13"], L["w2"], L["s2"])
    assert_close_to_oracle(out, ref)


def test_config1_full_layer(cfg1, cuda):
    cfg, L, lw, C = cfg1
    x = synthetic.make_tokens(cfg, device=cuda)
    bufs = ops.moe_workspace(cfg.M, cfg.H, cfg.I, cfg.topk, cfg.Is, cuda)
    rb = ops.router_bufs(cuda)
    out = torch.empty_like(x)
    _, tw, ids, _ = ops.moe_layer_step(x, lw, cfg.topk, bufs, rb, out)
    torch.cuda.synchronize()
    assert ops.moe_error_word(bufs["ctrl"]) == 0
    xs, i_c, w_c = x.cpu(), ids.cpu(), tw.cpu()
    ref = moe_ref.moe_rounded(xs, i_c, w_c, C["w13"], C["s13"], C["w2"], C["s2"], w_gate=C["w_gate"],
                              shared_w=(C["sh_gu"], C["sh_d"]))
    tru = moe_ref.moe_truth(xs, i_c, w_c, C["w13"], C["s13"], C["w2"], C["s2"], w_gate=C["w_gate"],
                            shared_w=(C["sh_gu"], C["sh_d"]))
    assert_close_to_oracle(out, ref, tru, "config1 M=10")
    assert int(bufs["ctrl"][:QF_MOE_CTRL_MIRROR].abs().sum().item()) == 0


def test_config1_precomputed_shared(cfg1, cuda):
    cfg, L, lw, C = cfg1
    x = synthetic.make_tokens(cfg, device=cuda, seed=5)
    g = torch.Generator(device="cpu").manual_seed(5)
    shared = (torch.randn(cfg.M, cfg.H, generator=g) * 0.05).to(BF)
    w, ids, _ = ops.router_topk(x, lw.router, cfg.topk, True, *ops.router_bufs(cuda))
    bufs = ops.moe_workspace(cfg.M, cfg.H, cfg.I, cfg.topk, 0, cuda)
    out = run_moe(x, ids, w, lw, bufs, shared=shared.to(cuda), use_shw=False)
    torch.cuda.synchronize()
    ref = moe_ref.moe_rounded(x.cpu(), ids.cpu(), w.cpu(), C["w13"], C["s13"], C["w2"], C["s2"], shared=shared,
                              w_gate=C["w_gate"])
    assert_close_to_oracle(out, ref)


def test_batch_invariance_and_back_to_back(cfg1, cuda):
    """Back-to-back launches equal a synchronised one; rows give the same bits in any batch of the same gate_up
    split regime (test_a16moe.py:163-178): at config 1, M = 10 (one chain per gate_up tile) against two batches of
    5, and M = 2 (k halves) against single rows; across the regimes, within the oracle tolerance."""
    cfg, L, lw, C = cfg1
    x = synthetic.make_tokens(cfg, device=cuda, seed=11)
    w, ids, _ = ops.router_topk(x, lw.router, cfg.topk, True, *ops.router_bufs(cuda))
    bufs = ops.moe_workspace(cfg.M, cfg.H, cfg.I, cfg.topk, cfg.Is, cuda)
    ref = run_moe(x, ids, w, lw, bufs).clone()
    torch.cuda.synchronize()
    outs = [run_moe(x, ids, w, lw, bufs) for _ in range(5)]            # back to back, no sync

    def rows(r0, r1):
        return run_moe(x[r0:r1].contiguous(), ids[r0:r1].contiguous(), w[r0:r1].contiguous(), lw, bufs)

    assert not gate_up_split(10, cfg.I, cfg.topk) and not gate_up_split(5, cfg.I, cfg.topk)
    assert gate_up_split(2, cfg.I, cfg.topk) and gate_up_split(1, cfg.I, cfg.topk)
    halves = torch.cat([rows(0, 5), rows(5, 10)])
    pair = rows(0, 2)
    single = torch.cat([rows(r, r + 1) for r in range(cfg.M)])
    torch.cuda.synchronize()
    assert all(torch.equal(o, ref) for o in outs)
    assert torch.equal(halves, ref)
    assert torch.equal(single[:2], pair)
    oracle = moe_ref.moe_rounded(x.cpu(), ids.cpu(), w.cpu(), C["w13"], C["s13"], C["w2"], C["s2"],
                                 w_gate=C["w_gate"], shared_w=(C["sh_gu"], C["sh_d"]))
    assert_close_to_oracle(single, oracle)
    assert int(bufs["ctrl"][:QF_MOE_CTRL_MIRROR].abs().sum().item()) == 0


def gate_up_split(M, I, topk):
    """Whether a launch of M tokens splits its gate_up items into two k halves (every half fits one wave of the
    three pipelines per SM): the kernel's rule. Within one regime results are batch-invariant bit for bit; across
    the two the fp32 association of the gate_up sums differs (half + half vs one chain)."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    return 2 * (2 * I // 128) * M * topk <= 3 * sms


@pytest.mark.parametrize("M", [3, 20, 60])
def test_odd_shared_shape_and_workspace_reuse(cuda, M):
    """H = 768 and a shared expert of Is = 192 (six 32-k stages per split-K item and per down item), two and four
    token groups at M = 20 / 60. The rows are then run one at a time on the same workspace (sized for M rows: its
    zero-kept counters sit at the same place for every M): equal to the batch bit for bit where both launches
    make the same gate_up split choice, within the oracle tolerance where they do not (M = 60)."""
    cfg = synthetic.MoEConfig("odd-shared", 768, 32, 128, 4, M, 192, 40 + M)
    L = synthetic.make_moe_layer(cfg)
    lw = layer_on(cuda, L)
    x = synthetic.make_tokens(cfg, device=cuda)
    w, ids, _ = ops.router_topk(x, lw.router, cfg.topk, True, *ops.router_bufs(cuda))
    bufs = ops.moe_workspace(M, cfg.H, cfg.I, cfg.topk, cfg.Is, cuda)
    out = run_moe(x, ids, w, lw, bufs)
    single = torch.cat([run_moe(x[r:r + 1].contiguous(), ids[r:r + 1].contiguous(), w[r:r + 1].contiguous(), lw, bufs)
                        for r in range(M)])
    again = run_moe(x, ids, w, lw, bufs)
    torch.cuda.synchronize()
    assert ops.moe_error_word(bufs["ctrl"]) == 0
    C = canon_cpu(L)
    ref = moe_ref.moe_rounded(x.cpu(), ids.cpu(), w.cpu(), C["w13"], C["s13"], C["w2"], C["s2"], w_gate=C["w_gate"],
                              shared_w=(C["sh_gu"], C["sh_d"]))
    assert_close_to_oracle(out, ref)
    assert_close_to_oracle(single, ref)
    assert torch.equal(again, out)
    if gate_up_split(M, cfg.I, cfg.topk) == gate_up_split(1, cfg.I, cfg.topk):
        assert torch.equal(single, out)
    assert int(bufs["ctrl"][:QF_MOE_CTRL_MIRROR].abs().sum().item()) == 0


@pytest.mark.parametrize("M", [1, 2, 4, 8, 16, 32, 64])
def test_token_sweep_with_zipf_routing(cfg1, cuda, M):
    """Config-2 style routing skew: hot experts receive more than 16 tokens (several token groups)."""
    cfg, L, lw, C = cfg1
    g = torch.Generator(device="cpu").manual_seed(100 + M)
    router = synthetic.zipf_router(C["router"].float(), 1.1, g).to(BF)
    x = synthetic.make_tokens(cfg, M=M, device=cuda, seed=100 + M)
    w, ids, _ = ops.router_topk(x, router.to(cuda), cfg.topk, True, *ops.router_bufs(cuda))
    bufs = ops.moe_workspace(M, cfg.H, cfg.I, cfg.topk, cfg.Is, cuda)
    out = run_moe(x, ids, w, lw, bufs)
    torch.cuda.synchronize()
    assert ops.moe_error_word(bufs["ctrl"]) == 0
    ref = moe_ref.moe_rounded(x.cpu(), ids.cpu(), w.cpu(), C["w13"], C["s13"], C["w2"], C["s2"], w_gate=C["w_gate"],
                              shared_w=(C["sh_gu"], C["sh_d"]))
    tru = moe_ref.moe_truth(x.cpu(), ids.cpu(), w.cpu(), C["w13"], C["s13"], C["w2"], C["s2"], w_gate=C["w_gate"],
                            shared_w=(C["sh_gu"], C["sh_d"]))
    assert_close_to_oracle(out, ref, tru, f"config2 zipf M={M}")
    if M == 64:
        counts = torch.bincount(ids.cpu().flatten().long(), minlength=cfg.E)
        assert counts.max().item() > 16, "the skewed router should give some expert several token groups"


def test_global_scales_and_odd_shapes(cuda):
    """I = 384 (a half-size last k stage in the down projection), top-1 and top-16, per-expert global scales."""
    cfg = synthetic.MoEConfig("odd", 512, 32, 384, 16, 7, 0, 21)
    L = synthetic.make_moe_layer(cfg)
    lw = layer_on(cuda, L)
    g = torch.Generator(device="cpu").manual_seed(3)
    gs13 = (torch.rand(cfg.E, generator=g) + 0.5).to(BF)
    gs2 = (torch.rand(cfg.E, generator=g) + 0.5).to(BF)
    for topk in (1, 16):
        x = synthetic.make_tokens(cfg, device=cuda)
        w, ids, _ = ops.router_topk(x, lw.router, topk, True, *ops.router_bufs(cuda))
        bufs = ops.moe_workspace(cfg.M, cfg.H, cfg.I, topk, 0, cuda)
        out = run_moe(x, ids, w, lw, bufs, gs13=gs13.to(cuda), gs2=gs2.to(cuda))
        torch.cuda.synchronize()
        ref = moe_ref.moe_rounded(x.cpu(), ids.cpu(), w.cpu(), L["w13"], L["s13"], L["w2"], L["s2"], gs13=gs13,
                                  gs2=gs2)
        tru = moe_ref.moe_truth(x.cpu(), ids.cpu(), w.cpu(), L["w13"], L["s13"], L["w2"], L["s2"], gs13=gs13, gs2=gs2)
        assert_close_to_oracle(out, ref, tru, "odd shapes")


def test_duplicate_and_out_of_range_ids(cuda):
    """A token that names the same expert twice gets both slots; an out-of-range id is skipped by the kernel's own
    bounds check and reported in the control block (no memory access through it)."""
    cfg = synthetic.CONFIGS[0]
    L = synthetic.make_moe_layer(cfg)
    lw = layer_on(cuda, L)
    x = synthetic.make_tokens(cfg).to(cuda)
    ids = torch.tensor([[3, 3, 5, 9], [1, 2, 3, 4], [15, 0, 7, 7], [8, 6, 4, 2]], dtype=torch.int32)
    w = torch.full((4, 4), 0.25)
    bufs = ops.moe_workspace(cfg.M, cfg.H, cfg.I, cfg.topk, 0, cuda)
    out = run_moe(x, ids.to(cuda), w.to(cuda), lw, bufs)
    torch.cuda.synchronize()
    ref = moe_ref.moe_rounded(x.cpu(), ids, w, L["w13"], L["s13"], L["w2"], L["s2"])
    assert_close_to_oracle(out, ref)
    assert ops.moe_error_word(bufs["ctrl"]) == 0
    bad = ids.clone()
    bad[1, 2] = 99
    out2 = run_moe(x, bad.to(cuda), w.to(cuda), lw, bufs)
    torch.cuda.synchronize()
    assert ops.moe_error_word(bufs["ctrl"]) & 0x2
    assert int(bufs["err_host"][0]) & 0x2          # the host mirror saw it without another synchronisation
    assert torch.isfinite(out2.float()).all()
    ok_rows = [0, 2, 3]
    assert torch.equal(out2[ok_rows].cpu(), out[ok_rows].cpu())
    # the next call on this workspace raises (and resets the workspace) instead of launching
    with pytest.raises(RuntimeError, match="out of range"):
        run_moe(x, ids.to(cuda), w.to(cuda), lw, bufs)
    out3 = run_moe(x, ids.to(cuda), w.to(cuda), lw, bufs)
    torch.cuda.synchronize()
    assert ops.moe_error_word(bufs["ctrl"]) == 0 and torch.equal(out3.cpu(), out.cpu())


def test_repack_kernels_match_host_layout(cuda):
    g = torch.Generator(device="cpu").manual_seed(5)
    for (N, K, gated) in [(1024, 2048, True), (2048, 512, False), (768, 384, True)]:
        q = synthetic.random_int4_words((3, N, K // 8), g, "cpu")
        s = synthetic.group_scales((3, N, K // 128), g, "cpu")
        wk, sk = formats.repack_w4(q.to(cuda), s.to(cuda), gated)
        wt, st = formats.repack_w4_torch(q, s, gated)
        assert torch.equal(wk.cpu(), wt) and torch.equal(sk.cpu(), st)
        q2, s2 = formats.unpack_w4(wk, sk, N, K, gated)
        assert torch.equal(q2.cpu(), q) and torch.equal(s2.cpu(), s)
    for (N, K, gated) in [(1024, 2048, True), (2048, 512, False)]:
        w = torch.randn(N, K, generator=g).to(BF)
        wk = formats.repack_bf16(w.to(cuda), gated)
        assert torch.equal(wk.cpu(), formats.repack_bf16_torch(w, gated))
        assert torch.equal(formats.unpack_bf16(wk, N, K, gated).cpu(), w)


def test_checkpoint_on_device(cuda, tmp_path):
    """The repack exactness check with the CUDA unpack kernels, and a saved layer loaded onto the GPU that runs the
    same layer-step bits as the layer it was saved from."""
    from qwenfast_b200 import checkpoint
    cfg = synthetic.MoEConfig("ckpt-gpu", 2048, 32, 512, 4, 6, 512, 77)
    L = synthetic.make_moe_layer(cfg)
    lw = layer_on(cuda, L)
    checkpoint.verify_layer(lw, L, experts_per_block=8)
    path = os.path.join(tmp_path, "layer.safetensors")
    checkpoint.save_layer(path, lw)
    lw2 = checkpoint.load_layer(path, device=cuda)
    x = synthetic.make_tokens(cfg, device=cuda)
    outs = []
    for w in (lw, lw2):
        bufs = ops.moe_workspace(cfg.M, cfg.H, cfg.I, cfg.topk, cfg.Is, cuda)
        outs.append(ops.moe_layer_step(x, w, cfg.topk, bufs, ops.router_bufs(cuda), torch.empty_like(x))[0])
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])


def test_int8_shared_expert_as_the_reference_passes_it(cfg1, cuda):
    """The shared expert given as INT8 weights with bf16 group scales (the reference's in-kernel shared expert,
    serve/overlays/sglang/srt/qwenfast.py:1092-1113, passed as shq1, shs1, shq2, shs2): against the oracle of that
    w8g arithmetic (test_a16moe.py:68-73) within the layer tolerance; converted once per weight tensor."""
    from oracle import w8_ref
    cfg, L, lw, C = cfg1
    sq1, ss1 = w8_ref.w8_quant(C["sh_gu"])
    sq2, ss2 = w8_ref.w8_quant(C["sh_d"])
    dq = [t.to(cuda) for t in (sq1, ss1, sq2, ss2)]
    x = synthetic.make_tokens(cfg, device=cuda, seed=21)
    w, ids, _ = ops.router_topk(x, lw.router, cfg.topk, True, *ops.router_bufs(cuda))
    bufs = ops.moe_workspace(cfg.M, cfg.H, cfg.I, cfg.topk, cfg.Is, cuda)
    outs = []
    for _ in range(2):
        out = torch.empty_like(x)
        ops.a16_moe_decode(x, ids, w, lw.w13, lw.s13, None, lw.w2, lw.s2, None, lw.w_gate, None, bufs["hbuf"],
                           bufs["ybuf"], bufs["gl"], bufs["ctrl"], out, 4, None, bufs["pbuf"], *dq, bufs["shbuf"])
        outs.append(out)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1]) and ops.moe_error_word(bufs["ctrl"]) == 0
    key_hits = [v for k, v in ops._W8_SHARED.items() if k[0][0] == dq[0].data_ptr()]
    assert len(key_hits) == 1                              # converted once
    shared = w8_ref.shared_expert_w8g(x.cpu(), sq1, ss1, sq2, ss2)
    ref = moe_ref.moe_rounded(x.cpu(), ids.cpu(), w.cpu(), C["w13"], C["s13"], C["w2"], C["s2"], shared=shared,
                              w_gate=C["w_gate"])
    assert_close_to_oracle(outs[0], ref)
    with pytest.raises(RuntimeError, match="INT8 shared-expert"):
        ops.a16_moe_decode(x, ids, w, lw.w13, lw.s13, None, lw.w2, lw.s2, None, lw.w_gate, None, bufs["hbuf"],
                           bufs["ybuf"], bufs["gl"], bufs["ctrl"], torch.empty_like(x), 4, None, bufs["pbuf"],
                           dq[0], dq[1][:, :8].contiguous(), dq[2], dq[3], bufs["shbuf"])


def test_bounded_wait_runs_out_and_is_reported(cfg1, cuda):
    """Failure detection without a GPU fault: diagnostic mode 2 makes one producer wait for a dependency that never
    arrives. The wait gives up at its bound (about one second), the launch drains and returns, the sticky error word
    holds QF_MOE_ERR_TIMEOUT, and once the caller has zeroed the control block and pbuf again the next launch on the
    same context is correct."""
    import time
    from qwenfast_b200 import _lib
    cfg, L, lw, C = cfg1
    x = synthetic.make_tokens(cfg, device=cuda, seed=31)
    w, ids, _ = ops.router_topk(x, lw.router, cfg.topk, True, *ops.router_bufs(cuda))
    bufs = ops.moe_workspace(cfg.M, cfg.H, cfg.I, cfg.topk, cfg.Is, cuda)
    torch.cuda.synchronize()
    t0 = time.time()
    ops.a16_moe_decode(x, ids, w, lw.w13, lw.s13, None, lw.w2, lw.s2, None, lw.w_gate, None, bufs["hbuf"],
                       bufs["ybuf"], bufs["gl"], bufs["ctrl"], torch.empty_like(x), 4, None, bufs["pbuf"], lw.sh_w13,
                       None, lw.sh_w2, None, bufs["shbuf"], mode=2)
    torch.cuda.synchronize()
    elapsed = time.time() - t0
    assert ops.moe_error_word(bufs["ctrl"]) & _lib.QF_MOE_ERR_TIMEOUT
    assert 0.2 < elapsed < 30, elapsed
    assert int(bufs["err_host"][0]) & _lib.QF_MOE_ERR_TIMEOUT
    # the op reports the earlier launch's error before its next launch and resets the control block and pbuf
    with pytest.raises(RuntimeError, match="bounded wait ran out"):
        run_moe(x, ids, w, lw, bufs)
    out = run_moe(x, ids, w, lw, bufs)
    torch.cuda.synchronize()
    assert ops.moe_error_word(bufs["ctrl"]) == 0
    ref = moe_ref.moe_rounded(x.cpu(), ids.cpu(), w.cpu(), C["w13"], C["s13"], C["w2"], C["s2"], w_gate=C["w_gate"],
                              shared_w=(C["sh_gu"], C["sh_d"]))
    assert_close_to_oracle(out, ref)


@pytest.mark.parametrize("M", [1, 10, 64])
def test_split_phases_equal_whole_layer(cfg1, cuda, M):
    """The reference's split phases (qf_a16moe.cu:889, 915): phase 1 (gate logits into gl, gate_up + SwiGLU into
    hbuf) then phase 2 (down, weighting, combine with the precomputed shared term) over one workspace give the same
    bits as the one-launch layer (phase 4), queued without a sync; phase 1 alone leaves the control block re-armed.
    In-kernel shared-expert weights are refused in the split phases, as in the reference."""
    cfg, L, lw, C = cfg1
    x = synthetic.make_tokens(cfg, M=M, device=cuda, seed=70 + M)
    g = torch.Generator(device="cpu").manual_seed(M)
    shared = (torch.randn(M, cfg.H, generator=g) * 0.05).to(BF).to(cuda)
    w, ids, _ = ops.router_topk(x, lw.router, cfg.topk, True, *ops.router_bufs(cuda))
    whole_bufs = ops.moe_workspace(M, cfg.H, cfg.I, cfg.topk, 0, cuda)
    whole = run_moe(x, ids, w, lw, whole_bufs, shared=shared, use_shw=False)
    bufs = ops.moe_workspace(M, cfg.H, cfg.I, cfg.topk, 0, cuda)
    outs = []
    for rep in range(2):
        out = torch.empty_like(x)
        for phase in (1, 2):
            ops.a16_moe_decode(x, ids, w, lw.w13, lw.s13, None, lw.w2, lw.s2, None, lw.w_gate, shared, bufs["hbuf"],
                               bufs["ybuf"], bufs["gl"], bufs["ctrl"], out, phase, None, bufs["pbuf"], None, None,
                               None, None, bufs["shbuf"])
        outs.append(out)
    torch.cuda.synchronize()
    assert ops.moe_error_word(bufs["ctrl"]) == 0
    assert int(bufs["ctrl"][:QF_MOE_CTRL_MIRROR].abs().sum().item()) == 0
    for out in outs:
        assert torch.equal(out, whole)
    with pytest.raises(RuntimeError, match="whole layer"):
        ops.a16_moe_decode(x, ids, w, lw.w13, lw.s13, None, lw.w2, lw.s2, None, lw.w_gate, None, bufs["hbuf"],
                           bufs["ybuf"], bufs["gl"], bufs["ctrl"], torch.empty_like(x), 1, None, bufs["pbuf"],
                           lw.sh_w13, None, lw.sh_w2, None, bufs["shbuf"])
