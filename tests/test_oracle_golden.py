"""The CPU oracle against outputs of the reference's own Python functions (tests/golden/make_golden.py)."""
import os

import torch

from conftest import GOLDEN
from oracle import moe_ref, router_ref, w8_ref

REF = torch.load(os.path.join(GOLDEN, "reference_fns.pt"))


def test_w8_quant_matches_reference_bit_exact():
    for tag in ("w8_g128", "w8_g64"):
        r = REF[tag]
        q, s = w8_ref.w8_quant(r["w"])
        assert torch.equal(q, r["q"]) and torch.equal(s, r["s"]), tag
        assert r["w"].shape[1] // s.shape[1] == r["G"]
    assert REF["w8q_equals_w8_quant"]


def test_router_selection_matches_reference_route():
    r = REF["route"]
    # the reference test's route(): fp32 logits, softmax, torch.topk, renormalise (no ties in this fixture)
    wts, ids = router_ref.topk_from_logits(r["logits"], r["ids"].shape[1], True)
    assert torch.equal(ids, r["ids"].int())
    torch.testing.assert_close(wts, r["w"].float(), rtol=1e-5, atol=1e-7)
    # and our logits restate the same fp32 product
    torch.testing.assert_close((r["x"].float() @ r["router"].float().T), r["logits"], rtol=0, atol=0)


def test_shared_expert_matches_reference_bit_exact():
    r = REF["shared_ref"]
    out = w8_ref.shared_expert_w8g(r["x"], r["sq1"], r["ss1"], r["sq2"], r["ss2"])
    assert torch.equal(out, r["out"])


def test_moe_truth_matches_reference_truth():
    r = REF["truth"]
    out = moe_ref.moe_truth(r["x"], r["ids"], r["w"], r["w13"], r["s13"], r["w2"], r["s2"], shared=r["shared"],
                            w_gate=r["wg"])
    torch.testing.assert_close(out, r["out"], rtol=1e-6, atol=1e-6)


def test_rounded_oracle_close_to_reference_truth():
    r = REF["truth"]
    out = moe_ref.moe_rounded(r["x"], r["ids"], r["w"], r["w13"], r["s13"], r["w2"], r["s2"], shared=r["shared"],
                              w_gate=r["wg"])
    d = out.float() - r["out"]
    assert d.norm() / r["out"].norm() < 1e-2
    assert d.abs().max() < 2e-2


def test_nvfp4_dequant_matches_reference_deq():
    """The NVFP4 restatement (oracle/nvfp4_ref.py) against the reference's own E2M1 table and deq
    (serve/qwenfast/test_a16moe.py:134-137), bit for bit."""
    from oracle import nvfp4_ref
    r = REF["nvfp4_deq"]
    assert torch.equal(nvfp4_ref.dequant_nvfp4(r["wp"], r["sf"], r["g"]), r["out"])


def test_nvfp4_truth_matches_reference_truth():
    """The fp32 layer truth on NVFP4 experts against the reference's truth run with its own deq."""
    from oracle import nvfp4_ref
    r = REF["nvfp4_truth"]
    out = nvfp4_ref.truth(r["x"], r["ids"], r["w"], r["w13"], r["s13"], r["g13"], r["w2"], r["s2"], r["g2"],
                          w_gate=r["wg"], shared=r["shared"])
    torch.testing.assert_close(out, r["out"], rtol=1e-6, atol=1e-6)


def test_nvfp4_group_products_are_exact_in_bf16():
    """Every e2m1 value times every finite E4M3 scale is a bf16 value: a group dequantises exactly with one bf16
    multiply, and the global 1 / g can wait for the epilogue."""
    from oracle import nvfp4_ref
    sf = torch.arange(256, dtype=torch.int32).to(torch.uint8).view(torch.float8_e4m3fn).float()
    sf = sf[torch.isfinite(sf)]
    prod = nvfp4_ref.e2m1_values()[:, None] * sf[None, :]
    assert torch.equal(prod.to(torch.bfloat16).float(), prod)
