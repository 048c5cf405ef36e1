"""The router entry point for callers that cannot allocate device memory (qf_router_topk_noalloc).

Plugin-style hosts (an inference engine that fixes its device memory at start-up, or code running while a CUDA graph
is captured) cannot pass scratch tensors; this entry point keeps the router's scratch in a static device array of the
library. Checked here through the C ABI: two calls in a row give the same ids and logits as qf_router_topk and weights
within the router tests' tolerance. This file is named to be collected last."""
import ctypes

import pytest
import torch

from qwenfast_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def _noalloc(lib, x, w, topk, renorm):
    rows, H = x.shape
    E = w.shape[0]
    wts = torch.empty(rows, topk, dtype=torch.float32, device=x.device)
    ids = torch.empty(rows, topk, dtype=torch.int32, device=x.device)
    logits = torch.empty(rows, E, dtype=torch.bfloat16, device=x.device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
    _lib.check(lib.qf_router_topk_noalloc(x.data_ptr(), w.data_ptr(), rows, H, E, topk, int(renorm), wts.data_ptr(),
                                          ids.data_ptr(), logits.data_ptr(), 1, stream), "router_topk_noalloc")
    return wts, ids, logits


def test_noalloc_router_matches_allocating_entry_point(cuda, lib):
    g = torch.Generator(device="cpu").manual_seed(77)
    cases = [(10, 2048, 512, 10, True), (64, 2048, 1024, 16, False)]
    for rows, H, E, topk, renorm in cases:
        x = [torch.randn(rows, H, generator=g).to(torch.bfloat16).to(cuda) for _ in range(2)]
        w = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16).to(cuda)
        got = [_noalloc(lib, xi, w, topk, renorm) for xi in x]           # two calls in a row, no sync between
        scratch, counter = ops.router_bufs(cuda, rows=rows, experts=E)
        ref = [ops.router_topk(xi, w, topk, renorm, scratch, counter) for xi in x]
        torch.cuda.synchronize()
        for (gw, gi, gl), (rw, ri, rl) in zip(got, ref):
            assert torch.equal(gi, ri) and torch.equal(gl, rl)
            torch.testing.assert_close(gw, rw, rtol=3e-5, atol=1e-6)


def test_noalloc_router_rejects_oversize(lib):
    p = ctypes.c_void_p(256)
    assert lib.qf_router_topk_noalloc(p, p, 65, 2048, 1024, 10, 1, p, p, p, 1, None) == -1
    assert b"static scratch" in lib.qf_last_error()
