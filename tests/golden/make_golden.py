"""Generate the golden fixtures under tests/golden/ (run in the build container, where the reference is mounted).

1. ``reference_fns.pt`` -- outputs of the reference's OWN Python functions, run on seeded CPU inputs:
   * ``w8_quant``  from serve/overlays/sglang/srt/qwenfast.py:301-315 (INT8 group quantisation),
   * ``w8q``, ``route``, ``shared_ref``, ``truth`` from serve/qwenfast/test_a16moe.py:61-86, 139-148,
   * the NVFP4 format: the module-level ``E2M1`` table and ``deq`` (test_a16moe.py:134-137), and ``truth`` once more
     with that real ``deq`` on NVFP4 experts (``nvfp4_deq``, ``nvfp4_truth``).
   The functions are extracted from the reference sources with ``ast`` (their modules import sglang and load a
   CUDA extension at import time, neither of which exists here) and executed in a namespace that supplies the
   globals they read (top-k ``K``, sizes ``I``/``Hd``, device ``dev`` = cpu). ``truth`` dequantises through a global
   ``deq``; it is given the int4 zero-point-8 / group-128 dequantisation of the synthetic format with unit global
   scales, so the reference's combine structure (per token and top-k position, SwiGLU, weighted sum, sigmoid-gated
   shared term) runs unchanged on that format.
2. ``config0.pt`` -- the toy configuration's oracle outputs (router + MoE) with input checksums, used by the GPU
   parity tests without recomputing the oracle.

Usage: python tests/golden/make_golden.py --reference <checkout of the reference repository>
(or set QWENFAST_REFERENCE to that directory)
"""
import argparse
import ast
import hashlib
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "qwen-3.8-flash-next-pro6000_b200"))


def extract(path, names):
    """Source of the top-level functions (or single-name assignments) called ``names`` in a Python file."""
    src = open(path).read()
    tree = ast.parse(src)
    out = {}
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name in names:
            out[node.name] = ast.get_source_segment(src, node)
        elif (isinstance(node, ast.Assign) and len(node.targets) == 1 and isinstance(node.targets[0], ast.Name)
              and node.targets[0].id in names):
            out[node.targets[0].id] = ast.get_source_segment(src, node)
    missing = set(names) - set(out)
    if missing:
        raise SystemExit(f"{path}: functions {sorted(missing)} not found")
    return out


def checksum(*ts):
    h = hashlib.sha256()
    for t in ts:
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes() if t.dtype != torch.bfloat16
                 else t.contiguous().view(torch.int16).numpy().tobytes())
    return h.hexdigest()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("QWENFAST_REFERENCE"),
                    help="root of the reference repository (required; or QWENFAST_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or QWENFAST_REFERENCE) must name the reference repository")
    ref = args.reference
    qf_src = extract(os.path.join(ref, "serve/overlays/sglang/srt/qwenfast.py"), ["w8_quant"])
    t_src = extract(os.path.join(ref, "serve/qwenfast/test_a16moe.py"), ["w8q", "route", "shared_ref", "truth"])

    from oracle import moe_ref

    E, Hd, I, K = 16, 256, 128, 4
    ns = dict(torch=torch, dev="cpu", E=E, Hd=Hd, I=I, K=K,
              deq=lambda wp, sf, g: moe_ref.dequant_int4(wp, sf) / float(g))
    for s in list(qf_src.values()) + list(t_src.values()):
        exec(compile(s, "<reference>", "exec"), ns)

    g = torch.Generator().manual_seed(20261201)
    res = {}
    # (1) INT8 group quantisation, G = 128 and the K % 128 != 0 case (G = 64)
    for tag, (N, Kk) in {"w8_g128": (64, 256), "w8_g64": (32, 192)}.items():
        w = (torch.randn(N, Kk, generator=g) * 0.02).to(torch.bfloat16)
        p = ns["w8_quant"](w)
        res[tag] = dict(w=w, q=p["q"], s=p["s"], G=p["G"])
    w = res["w8_g128"]["w"]
    q2, s2 = ns["w8q"](w)
    res["w8q_equals_w8_quant"] = bool(torch.equal(q2, res["w8_g128"]["q"]) and torch.equal(s2, res["w8_g128"]["s"]))

    # (2) routing of the reference test (fp32 logits, softmax, torch.topk, renormalise)
    x = torch.randn(4, Hd, generator=g).to(torch.bfloat16)
    router = (torch.randn(E, Hd, generator=g) * 0.02).to(torch.bfloat16)
    logits, tw, ids = ns["route"](dict(router=router), x)
    res["route"] = dict(x=x, router=router, logits=logits, w=tw, ids=ids)

    # (3) the reference's w8g shared expert with bf16 rounding points
    gu = (torch.randn(2 * I, Hd, generator=g) * 0.02).to(torch.bfloat16)
    dn = (torch.randn(Hd, I, generator=g) * 0.02).to(torch.bfloat16)
    sq1, ss1 = ns["w8q"](gu)
    sq2, ss2 = ns["w8q"](dn)
    d = dict(sq1=sq1, ss1=ss1, sq2=sq2, ss2=ss2)
    res["shared_ref"] = dict(x=x, **d, out=ns["shared_ref"](d, x))

    # (4) fp32 truth of the MoE layer on int4 zero-point-8 experts
    from qwenfast_b200 import synthetic
    w13 = synthetic.random_int4_words((E, 2 * I, Hd // 8), g, "cpu")
    s13 = synthetic.group_scales((E, 2 * I, Hd // 128), g, "cpu")
    w2 = synthetic.random_int4_words((E, Hd, I // 8), g, "cpu")
    s2_ = synthetic.group_scales((E, Hd, I // 128), g, "cpu")
    wg = (torch.randn(Hd, generator=g) * 0.02).to(torch.bfloat16)
    shared = (torch.randn(4, Hd, generator=g) * 0.05).to(torch.bfloat16)
    canon = dict(w13=w13, s13=s13, w2=w2, s2=s2_, g13=torch.ones(E, 2), g2=torch.ones(E))
    out = ns["truth"](dict(canon=canon, wg=wg), x, tw, ids, shared)
    res["truth"] = dict(x=x, ids=ids, w=tw, w13=w13, s13=s13, w2=w2, s2=s2_, wg=wg, shared=shared, out=out)

    # (5) NVFP4: the reference's own E2M1 table and deq, and its truth on NVFP4 experts
    from oracle import nvfp4_ref
    n_src = extract(os.path.join(ref, "serve/qwenfast/test_a16moe.py"), ["E2M1", "deq", "truth"])
    ns4 = dict(torch=torch, dev="cpu", E=E, Hd=Hd, I=I, K=K)
    for name in ("E2M1", "deq", "truth"):
        exec(compile(n_src[name], "<reference>", "exec"), ns4)
    wp, sf = nvfp4_ref.random_nvfp4((48, 256), g)
    res["nvfp4_deq"] = dict(wp=wp, sf=sf, g=0.25, out=ns4["deq"](wp, sf, 0.25))
    w13f, s13f = nvfp4_ref.random_nvfp4((E, 2 * I, Hd), g)
    w2f, s2f = nvfp4_ref.random_nvfp4((E, Hd, I), g)
    g13f = torch.rand(E, 2, generator=g) * 2 + 0.5
    g2f = torch.rand(E, generator=g) * 2 + 0.5
    canon4 = dict(w13=w13f, s13=s13f, w2=w2f, s2=s2f, g13=g13f, g2=g2f)
    out4 = ns4["truth"](dict(canon=canon4, wg=wg), x, tw, ids, shared)
    res["nvfp4_truth"] = dict(x=x, ids=ids, w=tw, **canon4, wg=wg, shared=shared, out=out4)
    torch.save(res, os.path.join(HERE, "reference_fns.pt"))

    # config 0 oracle outputs (inputs are regenerated from the seed; checksums guard the generator)
    from oracle import router_ref
    cfg = synthetic.CONFIGS[0]
    L = synthetic.make_moe_layer(cfg)
    xt = synthetic.make_tokens(cfg)
    rw, rids, rlg = router_ref.router_topk(xt, L["router"], cfg.topk, True)
    out_r = moe_ref.moe_rounded(xt, rids, rw, L["w13"], L["s13"], L["w2"], L["s2"])
    out_t = moe_ref.moe_truth(xt, rids, rw, L["w13"], L["s13"], L["w2"], L["s2"])
    torch.save(dict(checksum=checksum(xt, L["router"], L["w13"], L["s13"], L["w2"], L["s2"]),
                    logits=rlg, ids=rids, weights=rw, out_rounded=out_r, out_truth=out_t),
               os.path.join(HERE, "config0.pt"))
    print("wrote", os.listdir(HERE))


if __name__ == "__main__":
    main()
