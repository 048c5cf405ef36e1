"""CPU restatement of the reference's NVFP4 expert format (test infrastructure only; see ``oracle/__init__.py``).

The reference's routed experts are NVFP4 (``serve/qwenfast/test_a16moe.py:134-137``, ``qf_a16moe.cu:43-57``): per
expert matrix [N, K], codes packed two per byte ``wp uint8 [N, K/2]`` (even k in the low nibble), one E4M3 scale per
16 k ``sf float8_e4m3fn [N, K/16]`` and a per-expert global value ``g`` stored as the reciprocal of the multiplier:

    w[n, k] = e2m1(code[n, k]) * sf[n, k / 16] / g

where e2m1 is the 4-bit float of the OCP microscaling formats (1 sign bit, 2 exponent bits with bias 1, 1 mantissa
bit; values 0, 0.5, 1, 1.5, 2, 3, 4, 6 and their negatives). ``truth`` restates the reference's fp32 layer truth on
that format (``test_a16moe.py:138-148``).

A fact the sm_100a front end for this format relies on (tested): e2m1 * sf, the product of a 2-significant-bit and
a 4-significant-bit value, is exact in bf16, so one bf16 multiply per weight pair dequantises a group exactly and
1 / g can be applied once, in the epilogue, like the int4 path's per-expert global scale.
"""
import torch
import torch.nn.functional as F


def e2m1_values() -> torch.Tensor:
    """fp32 [16]: the value of each 4-bit e2m1 code (bit 3 sign, bits 1-2 exponent, bit 0 mantissa)."""
    out = torch.empty(16)
    for c in range(16):
        e, m = (c >> 1) & 3, c & 1
        mag = (m * 0.5) if e == 0 else (2.0 ** (e - 1)) * (1.0 + 0.5 * m)
        out[c] = -mag if c & 8 else mag
    return out


def unpack_e2m1(wp: torch.Tensor) -> torch.Tensor:
    """uint8 [..., N, K/2] -> int64 codes [..., N, K] (even k from the low nibble)."""
    lo, hi = (wp & 15).long(), (wp >> 4).long()
    return torch.stack([lo, hi], -1).reshape(*wp.shape[:-1], wp.shape[-1] * 2)


def dequant_nvfp4(wp: torch.Tensor, sf: torch.Tensor, g) -> torch.Tensor:
    """fp32 [N, K] = e2m1(code) * sf (per 16 k) / g."""
    v = e2m1_values()[unpack_e2m1(wp)]
    return v * sf.float().repeat_interleave(16, dim=-1) / float(g)


def truth(x, topk_ids, topk_w, w13, s13, g13, w2, s2, g2, w_gate=None, shared=None):
    """fp32 layer on NVFP4 experts: w13 uint8 [E, 2I, H/2], s13 e4m3 [E, 2I, H/16], g13 fp32 [E, 2] (column 0 used,
    as the reference does), w2 uint8 [E, H, I/2], s2 e4m3 [E, H, I/16], g2 fp32 [E]; plus
    sigmoid(x . w_gate) * shared when a shared output is given."""
    M, H = x.shape
    I = w2.shape[2] * 2
    xf = x.float()
    out = torch.zeros(M, H)
    for t in range(M):
        for kp in range(topk_ids.shape[1]):
            e = int(topk_ids[t, kp])
            a = dequant_nvfp4(w13[e], s13[e], g13[e, 0])
            b = dequant_nvfp4(w2[e], s2[e], g2[e])
            gu = a @ xf[t]
            h = F.silu(gu[:I]) * gu[I:]
            out[t] += float(topk_w[t, kp]) * (b @ h)
    if shared is None:
        return out
    gate = torch.sigmoid(xf @ w_gate.float())
    return out + gate[:, None] * shared.float()


def random_nvfp4(shape_nk, g: torch.Generator):
    """Seeded NVFP4 weights of one matrix family [..., N, K]: uniform codes, E4M3 scales |N(0, 1)| * 2 + 1/64
    (normal E4M3 values), for tests."""
    *lead, N, K = shape_nk
    wp = torch.randint(0, 256, (*lead, N, K // 2), generator=g, dtype=torch.int32).to(torch.uint8)
    sf = (torch.randn(*lead, N, K // 16, generator=g).abs() * 2 + 1.0 / 64).to(torch.float8_e4m3fn)
    return wp, sf
