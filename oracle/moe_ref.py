"""CPU restatement of the W4A16 decode MoE layer (test infrastructure only; see ``oracle/__init__.py``).

Weight format (the synthetic configurations' canonical form): int4 codes 0..15 with zero point 8, packed eight
per int32 along K with the lowest k in the low nibble, layout ``[E, N, K/8]``; one bf16 scale per 128 k,
layout ``[E, N, K/128]``; the dequantised weight is ``(q - 8) * s``.

Two references are provided:

``moe_rounded``  the layer with the bf16 rounding points of the reference kernel
                 (``serve/qwenfast/qf_a16moe.cu:2-4``): gemm1 ``bf16(bf16(acc) * gs13)`` and SwiGLU to bf16
                 (:733-735); gemm2 ``bf16(bf16(acc) * bf16(gs2 * bf16(w_topk)))`` (:804-805); fp32 sum over the
                 top-k positions in top-k order, rounded to bf16, then ``bf16(sigmoid(gl) * shared + routed)``
                 (:449-461).  Products are fp32.  The per-expert global scales default to 1.
``moe_truth``    the fp32 reference of ``serve/qwenfast/test_a16moe.py:139-148`` (dequantise, fp32 matmuls,
                 weighted sum, plus ``sigmoid(x . w_gate) * shared``).

The shared expert with bf16 weights follows ``serve/qwenfast/test_a16moe.py:68-73`` (gate_up to bf16, SwiGLU to
bf16, down to bf16).
"""
import torch
import torch.nn.functional as F

GROUP = 128


def bf16r(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).float()


def unpack_int4(packed: torch.Tensor) -> torch.Tensor:
    """int32 [..., N, K/8] -> int64 codes [..., N, K] in 0..15 (low nibble = lowest k)."""
    shifts = torch.arange(0, 32, 4, dtype=torch.int32)
    q = (packed.unsqueeze(-1) >> shifts) & 0xF
    return q.reshape(*packed.shape[:-1], packed.shape[-1] * 8).long()


def dequant_int4(packed: torch.Tensor, scales: torch.Tensor, group: int = GROUP) -> torch.Tensor:
    """(q - 8) * s in fp32, [N, K]."""
    q = unpack_int4(packed).float() - 8.0
    return q * scales.float().repeat_interleave(group, dim=-1)


def shared_expert_bf16(x: torch.Tensor, w_gu: torch.Tensor, w_d: torch.Tensor) -> torch.Tensor:
    """Shared expert on bf16 weights: gate_up [2Is, H], down [H, Is] -> bf16 [M, H] (test_a16moe.py:68-73)."""
    i_s = w_d.shape[1]
    gu = bf16r(x.float() @ w_gu.float().T)
    h = bf16r(F.silu(gu[:, :i_s]) * gu[:, i_s:])
    return (h @ w_d.float().T).to(torch.bfloat16)


def shared_gate_logits(x: torch.Tensor, w_gate: torch.Tensor) -> torch.Tensor:
    """gl[t] = x[t] . w_gate in fp32 (qf_a16moe.cu:470-478)."""
    return x.float() @ w_gate.float()


def moe_rounded(x, topk_ids, topk_w, w13, s13, w2, s2, gs13=None, gs2=None,
                shared=None, w_gate=None, shared_w=None, expert_range=None, return_slots=False, dequant=None):
    """The routed-expert layer with the kernel's rounding points.

    x bf16 [M, H]; topk_ids int [M, k]; topk_w fp32 [M, k]; w13 int32 [E, 2I, H/8]; s13 bf16 [E, 2I, H/128];
    w2 int32 [E, H, I/8]; s2 bf16 [E, H, I/128]; gs13/gs2 bf16 [E] or None (= 1).
    Shared term: ``shared`` bf16 [M, H] precomputed, or ``shared_w = (w_gu, w_d)`` bf16 weights computed here;
    either needs ``w_gate`` bf16 [H].  ``expert_range=(lo, hi)`` keeps only the slots whose expert is in range
    (the expert-parallel shard of one rank; the other slots are zero).
    Returns out bf16 [M, H] (and the per-slot y bf16 [M, k, H] when ``return_slots``).
    ``dequant(w, s)`` -> fp32 [N, K] replaces the int4 dequantisation for another expert format (NVFP4: the codes and
    E4M3 scales, with the per-expert global multiplier passed as gs13 / gs2, as the reference's kernel applies it).
    """
    M, H = x.shape
    k = topk_ids.shape[1]
    deq = dequant_int4 if dequant is None else dequant
    xf = x.float()
    ids = topk_ids.long()
    y = torch.zeros(M, k, H)
    for e in torch.unique(ids).tolist():
        if expert_range is not None and not (expert_range[0] <= e < expert_range[1]):
            continue
        toks, kps = torch.nonzero(ids == e, as_tuple=True)
        g13 = 1.0 if gs13 is None else float(gs13[e].float())
        g2 = torch.tensor(1.0) if gs2 is None else gs2[e].float()
        w_gu = deq(w13[e], s13[e])
        I = w_gu.shape[0] // 2
        acc = xf[toks] @ w_gu.T
        g = bf16r(bf16r(acc[:, :I]) * g13)
        u = bf16r(bf16r(acc[:, I:]) * g13)
        h = bf16r(g / (1.0 + torch.exp(-g)) * u)
        acc2 = h @ deq(w2[e], s2[e]).T
        tw = bf16r(g2 * bf16r(topk_w[toks, kps].float()))
        y[toks, kps] = bf16r(bf16r(acc2) * tw[:, None])
    if shared_w is not None:
        shared = shared_expert_bf16(x, *shared_w)
    out = combine_slots(x, y, shared, w_gate)
    return (out, y.to(torch.bfloat16)) if return_slots else out


def combine_slots(x, y, shared=None, w_gate=None):
    """The combine (qf_a16moe.cu:449-461): fp32 sum of the slot outputs y [M, k, H] in top-k order, rounded to bf16,
    then ``bf16(sigmoid(x . w_gate) * shared + routed)`` when a shared term is given."""
    y = y.float()
    acc = y[:, 0].clone()
    for kp in range(1, y.shape[1]):
        acc = acc + y[:, kp]
    routed = bf16r(acc)
    if shared is None:
        return routed.to(torch.bfloat16)
    gate = torch.sigmoid(shared_gate_logits(x, w_gate))
    return (gate[:, None] * shared.float() + routed).to(torch.bfloat16)


def moe_truth(x, topk_ids, topk_w, w13, s13, w2, s2, gs13=None, gs2=None,
              shared=None, w_gate=None, shared_w=None):
    """fp32 reference (test_a16moe.py:139-148): no intermediate rounding at all.

    With ``shared_w`` the shared expert is evaluated in fp32 as well."""
    M, H = x.shape
    k = topk_ids.shape[1]
    I = w2.shape[2] * 8
    xf = x.float()
    out = torch.zeros(M, H)
    cache = {}
    for t in range(M):
        for kp in range(k):
            e = int(topk_ids[t, kp])
            if e not in cache:
                a = dequant_int4(w13[e], s13[e]) * (1.0 if gs13 is None else float(gs13[e].float()))
                b = dequant_int4(w2[e], s2[e]) * (1.0 if gs2 is None else float(gs2[e].float()))
                cache[e] = (a, b)
            a, b = cache[e]
            gu = a @ xf[t]
            h = F.silu(gu[:I]) * gu[I:]
            out[t] += float(topk_w[t, kp]) * (b @ h)
    if shared_w is not None:
        w_gu, w_d = shared_w
        i_s = w_d.shape[1]
        gu = xf @ w_gu.float().T
        shared_f = (F.silu(gu[:, :i_s]) * gu[:, i_s:]) @ w_d.float().T
    elif shared is not None:
        shared_f = shared.float()
    else:
        return out
    gate = torch.sigmoid(xf @ w_gate.float())
    return out + gate[:, None] * shared_f


def layer_bytes(topk_ids, H, I, E, I_s=0, M=None, group=GROUP):
    """Algorithmic HBM bytes of one layer-step: distinct experts' int4 weights + bf16 scales, the bf16 router
    weight, the bf16 shared expert (gate_up, down, gate vector), and the activations in and out."""
    U = int(torch.unique(topk_ids).numel())
    per_expert = (2 * I * H + H * I) // 2 + 2 * (2 * I * H + H * I) // group
    M = topk_ids.shape[0] if M is None else M
    shared = (3 * H * I_s + H) * 2 if I_s else 0
    return U * per_expert + E * H * 2 + shared + 2 * M * H * 2
