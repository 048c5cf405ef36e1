"""Selection semantics of the router oracle (qf_router.cu:116-151): ties to the lower id, NaN ranks as -1e30,
-0 equals +0, renormalisation guard. These are the rules the GPU kernel is checked against bit-for-bit."""
import numpy as np
import torch

from oracle import router_ref


def _lg(rows):
    return torch.tensor(rows, dtype=torch.float32).to(torch.bfloat16)


def test_ties_go_to_lower_expert_id():
    w, ids = router_ref.topk_from_logits(_lg([[1.0] * 16]), 4, True)
    assert ids.tolist() == [[0, 1, 2, 3]]
    torch.testing.assert_close(w, torch.full((1, 4), 0.25))


def test_ranking_is_by_value_then_id():
    row = [0.0] * 16
    row[5], row[9], row[2], row[12] = 2.0, 2.0, 3.0, -1.0
    _, ids = router_ref.topk_from_logits(_lg([row]), 5, False)
    assert ids.tolist() == [[2, 5, 9, 0, 1]]


def test_nan_ranks_below_finite_and_negative_zero_equals_zero():
    row = [-2.0] * 16
    row[3] = float("nan")
    row[7] = -0.0
    row[8] = 0.0
    row[1] = float("-inf")
    _, ids = router_ref.topk_from_logits(_lg([row]), 16, False)
    order = ids[0].tolist()
    assert order[:2] == [7, 8]                    # -0 and +0 tie -> lower id first
    assert order.index(3) == 14 and order[-1] == 1   # NaN (as -1e30) below every finite value, -inf last


def test_renormalisation_sums_to_one_and_plain_weights_are_softmax():
    g = torch.Generator().manual_seed(0)
    lg = torch.randn(6, 64, generator=g).to(torch.bfloat16)
    w, ids = router_ref.topk_from_logits(lg, 10, True)
    torch.testing.assert_close(w.sum(1), torch.ones(6), rtol=1e-6, atol=1e-6)
    p, ids2 = router_ref.topk_from_logits(lg, 10, False)
    assert torch.equal(ids, ids2)
    sm = torch.softmax(lg.float(), -1).gather(1, ids.long())
    torch.testing.assert_close(p, sm, rtol=1e-5, atol=1e-7)


def test_order_keys_are_monotone():
    v = np.array([-np.inf, -3.5, -1e-30, -0.0, 0.0, 1e-30, 2.0, np.inf], np.float32)
    k = router_ref.order_keys(v)
    assert all(k[i] <= k[i + 1] for i in range(len(k) - 1)) and k[3] == k[4]
