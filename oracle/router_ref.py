"""CPU restatement of the reference router (test infrastructure only; see ``oracle/__init__.py``).

Reference: ``serve/qwenfast/qf_router.cu``
  * logits[t, e] = bf16(fp32 dot(x[t], w[e]))                              (:3, :84-86)
  * p = softmax over the bf16 logits, in fp32, max-subtracted             (:103-121)
  * ranking on the logits themselves through order-preserving uint32 keys: NaN ranks as -1e30 (:116), -0 folds
    onto +0 (:128), strictly greater wins so the lowest expert id wins ties (:134-141)
  * routed = sum of the selected p in selection order; weights = p / routed when renormalising, with a
    guard that keeps the weights unnormalised when the sum is not positive (:152-155)
The selection given the logits is integer work and must match bit-for-bit; the softmax weights depend on the
exp implementation and are compared with a tolerance.
"""
import numpy as np
import torch


def router_logits(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """bf16 [M, H] x bf16 [E, H] -> bf16 [M, E]: fp32 products and sums, one rounding to bf16 (qf_router.cu:84-86)."""
    return (x.float() @ w.float().T).to(torch.bfloat16)


def order_keys(v: np.ndarray) -> np.ndarray:
    """fp32 values -> uint32 keys whose unsigned order is the float order (qf_router.cu:116, 123-130)."""
    r = np.where(np.isnan(v), np.float32(-1e30), v).astype(np.float32)
    u = r.view(np.uint32).copy()
    u[u == np.uint32(0x80000000)] = 0
    neg = (u & np.uint32(0x80000000)) != 0
    return np.where(neg, ~u, u | np.uint32(0x80000000)).astype(np.uint32)


def topk_from_logits(logits: torch.Tensor, topk: int, renormalize: bool):
    """bf16 logits [M, E] -> (weights fp32 [M, k], ids int32 [M, k]) with the reference's selection rules."""
    lg = logits.float().numpy().astype(np.float32)
    M, E = lg.shape
    ids = np.zeros((M, topk), np.int32)
    wts = np.zeros((M, topk), np.float32)
    for t in range(M):
        v = lg[t]
        finite = v[~np.isnan(v)]
        mx = np.float32(finite.max()) if finite.size else np.float32(-np.inf)
        ex = np.exp((v - mx).astype(np.float32)).astype(np.float32)
        total = np.float32(ex.sum(dtype=np.float32))
        keys = order_keys(v).astype(np.int64)
        order = np.lexsort((np.arange(E), -keys))          # key descending, expert id ascending
        sel = order[:topk]
        p = (ex[sel] / total).astype(np.float32)
        routed = np.float32(0.0)
        for pi in p:
            routed = np.float32(routed + pi)
        norm = routed if routed > 0 else np.float32(1.0)
        ids[t] = sel
        wts[t] = (p / norm).astype(np.float32) if renormalize else p
    return torch.from_numpy(wts), torch.from_numpy(ids)


def router_topk(x: torch.Tensor, w: torch.Tensor, topk: int, renormalize: bool):
    """Full oracle router: (weights fp32 [M, k], ids int32 [M, k], logits bf16 [M, E])."""
    lg = router_logits(x, w)
    wts, ids = topk_from_logits(lg, topk, renormalize)
    return wts, ids, lg
