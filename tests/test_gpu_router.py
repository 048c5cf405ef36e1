"""router_topk on the GPU vs the CPU oracle (protocol of serve/qwenfast/test_router.py:41-43 and test_router3.py):
bf16 logits within one bf16 ulp of the oracle's, top-k ids bit-exact given the kernel's own logits, weights within
fp32 tolerance; on integer-valued inputs (exact logits, heavy ties, exact zeros) ids equal the oracle's outright."""
import pytest
import torch

from oracle import router_ref
from qwenfast_b200 import ops

pytestmark = pytest.mark.gpu


def run(x, w, topk, renorm):
    scratch, counter = ops.router_bufs(x.device, rows=x.shape[0], experts=w.shape[0])
    wts, ids, lg = ops.router_topk(x, w, topk, renorm, scratch, counter)
    torch.cuda.synchronize()
    assert int(counter.item()) == 0, "ticket counter must be re-armed"
    return wts.cpu(), ids.cpu(), lg.cpu()


def check(x, w, topk, renorm, exact_logits=False):
    wts, ids, lg = run(x, w, topk, renorm)
    ref = router_ref.router_logits(x.cpu(), w.cpu()).float()
    got = lg.float()
    if exact_logits:
        assert torch.equal(got, ref)
    else:
        tol = torch.maximum(ref.abs(), got.abs()) * 2.0 ** -7 + 1e-30
        assert bool(((got - ref).abs() <= tol).all()), "logits differ by more than one bf16 ulp"
    ow, oids = router_ref.topk_from_logits(lg, topk, renorm)
    assert torch.equal(ids, oids), "top-k ids must be bit-exact given the kernel logits"
    torch.testing.assert_close(wts, ow, rtol=3e-5, atol=1e-6)
    return wts, ids, lg


@pytest.mark.parametrize("H,E,topk,M", [(256, 16, 4, 4), (2048, 512, 10, 10), (2560, 512, 10, 8), (4096, 256, 8, 3),
                                        (2048, 1024, 16, 5)])
@pytest.mark.parametrize("renorm", [True, False])
def test_router_matches_oracle(cuda, H, E, topk, M, renorm):
    g = torch.Generator(device="cpu").manual_seed(H + E + M)
    x = torch.randn(M, H, generator=g).to(torch.bfloat16).to(cuda)
    w = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16).to(cuda)
    check(x, w, topk, renorm)


@pytest.mark.parametrize("M", [1, 2, 4, 8, 16, 32, 64])
def test_router_token_sweep(cuda, M):
    g = torch.Generator(device="cpu").manual_seed(M)
    x = (torch.randn(M, 2048, generator=g) * 0.7).to(torch.bfloat16).to(cuda)
    w = (torch.randn(512, 2048, generator=g) * 0.02).to(torch.bfloat16).to(cuda)
    check(x, w, 10, True)


def test_router_ties_and_zeros_kat(cuda):
    """Coarse +-1 tokens at 0.2% density and integer router weights in [-2, 2]: exact integer logits, many ties and
    exact zeros (the case generator of serve/qwenfast/test_router3.py:25-28)."""
    g = torch.Generator(device="cpu").manual_seed(1234)
    for M in (1, 3, 8, 16):
        x = (torch.randint(-1, 2, (M, 2048), generator=g).float() * (torch.rand(M, 2048, generator=g) < 0.002))
        w = torch.randint(-2, 3, (512, 2048), generator=g).float()
        x, w = x.to(torch.bfloat16).to(cuda), w.to(torch.bfloat16).to(cuda)
        for renorm in (True, False):
            _, ids, _ = check(x, w, 10, renorm, exact_logits=True)
            _, oids, _ = router_ref.router_topk(x.cpu(), w.cpu(), 10, renorm)
            assert torch.equal(ids, oids)


def test_router_one_hot_kat(cuda):
    g = torch.Generator(device="cpu").manual_seed(7)
    w = (torch.randn(512, 2048, generator=g) * 0.02).to(torch.bfloat16).to(cuda)
    x = torch.zeros(8, 2048, dtype=torch.bfloat16, device=cuda)
    for t in range(8):
        x[t, 37 * t + 5] = 1.0
    _, ids, _ = check(x, w, 10, True, exact_logits=True)
    _, oids, _ = router_ref.router_topk(x.cpu(), w.cpu(), 10, True)
    assert torch.equal(ids, oids)


def test_router_nan_row_ranks_last(cuda):
    g = torch.Generator(device="cpu").manual_seed(9)
    w = (torch.randn(16, 256, generator=g) * 0.02)
    w[3] = float("nan")
    w = w.to(torch.bfloat16).to(cuda)
    x = torch.randn(4, 256, generator=g).to(torch.bfloat16).to(cuda)
    _, ids, lg = run(x, w, 16, False)
    assert torch.isnan(lg[:, 3].float()).all()
    _, oids = router_ref.topk_from_logits(lg, 16, False)
    assert torch.equal(ids, oids) and (ids[:, -1] == 3).all()


def test_router_batch_invariant_and_back_to_back(cuda):
    g = torch.Generator(device="cpu").manual_seed(11)
    x = torch.randn(10, 2048, generator=g).to(torch.bfloat16).to(cuda)
    w = (torch.randn(512, 2048, generator=g) * 0.02).to(torch.bfloat16).to(cuda)
    scratch, counter = ops.router_bufs(cuda)
    outs = [ops.router_topk(x, w, 10, True, scratch, counter) for _ in range(4)]   # no sync between launches
    single = [ops.router_topk(x[r:r + 1].contiguous(), w, 10, True, scratch, counter) for r in range(10)]
    torch.cuda.synchronize()
    for o in outs[1:]:
        assert all(torch.equal(a, b) for a, b in zip(o, outs[0]))
    assert torch.equal(torch.cat([s[1] for s in single]), outs[0][1])
    assert torch.equal(torch.cat([s[2] for s in single]), outs[0][2])
    assert int(counter.item()) == 0
