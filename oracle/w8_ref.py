"""CPU restatement of the INT8 dense projections (test infrastructure only; see ``oracle/__init__.py``).

* ``w8_quant``: symmetric INT8 with one bf16 scale per group of 128 k (64 when K % 128 != 0); the scale is
  rounded to bf16 *before* quantising, so ``q * s`` is the exact dequantised weight
  (``serve/overlays/sglang/srt/qwenfast.py:301-315``).
* ``w8g_ref``: W8A16 product ``x @ (q * s)^T`` in fp32, one rounding to bf16 (``serve/qwenfast/qf_w8g.cu:7-8``;
  truth as in ``serve/qwenfast/test_w8m.py:39`` and ``test_w8k.py:86``).
* ``w8a8_*``: the W8A8 definition of the benchmark configuration (no reference code exists):
  ``sx[t] = absmax_t / 127`` (fp32; 1 for an all-zero row), ``xq = rint(x / sx)`` clamped to [-127, 127],
  ``acc = sum xq * q`` exact (int64 here, int32 on the GPU), ``y = bf16((float(acc) * sx[t]) * sw[n])`` with
  round-to-nearest fp32 multiplies in that order.
"""
import torch


def w8_quant(w: torch.Tensor):
    """bf16 [N, K] -> (q int8 [N, K], s bf16 [N, K/G])."""
    N, K = w.shape
    G = 128 if K % 128 == 0 else 64
    xg = w.float().view(N, K // G, G)
    s16 = (xg.abs().amax(2) / 127).clamp_(min=1e-30).to(torch.bfloat16)
    q = (xg / s16.float().unsqueeze(-1)).round_().clamp_(-127, 127).to(torch.int8).view(N, K)
    return q.contiguous(), s16.contiguous()


def w8g_dequant(q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    N, K = q.shape
    G = K // s.shape[1]
    return (q.float().view(N, K // G, G) * s.float().unsqueeze(-1)).view(N, K)


def w8g_ref(x: torch.Tensor, q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """fp32 truth of the W8A16 group-scaled product, rounded once to bf16."""
    return (x.float() @ w8g_dequant(q, s).T).to(torch.bfloat16)


def w8a8_quant_act(x: torch.Tensor):
    """bf16 [M, K] -> (xq int8 [M, K], sx fp32 [M])."""
    xf = x.float()
    amax = xf.abs().amax(dim=1)
    sx = torch.where(amax > 0, amax / torch.tensor(127.0), torch.ones_like(amax))
    xq = torch.round(xf / sx[:, None]).clamp_(-127, 127).to(torch.int8)
    return xq, sx


def w8a8_acc(xq: torch.Tensor, q: torch.Tensor) -> torch.Tensor:
    """Exact accumulators, int64 [M, N] (they fit int32 for K <= 133144)."""
    return xq.long() @ q.long().T


def w8a8_ref(x: torch.Tensor, q: torch.Tensor, sw: torch.Tensor):
    """Returns (y bf16 [M, N], acc int64 [M, N], xq int8 [M, K], sx fp32 [M])."""
    xq, sx = w8a8_quant_act(x)
    acc = w8a8_acc(xq, q)
    y = ((acc.to(torch.float32) * sx[:, None]) * sw.float()[None, :]).to(torch.bfloat16)
    return y, acc, xq, sx


def shared_expert_w8g(x: torch.Tensor, sq1, ss1, sq2, ss2) -> torch.Tensor:
    """Shared expert on group-scaled INT8 weights (gate_up [2I, H], down [H, I]) with the bf16 rounding points of
    the reference's in-kernel shared expert (``serve/qwenfast/test_a16moe.py:68-73``)."""
    i_s = sq2.shape[1]
    gu = (x.float() @ w8g_dequant(sq1, ss1).T).to(torch.bfloat16).float()
    h = (torch.nn.functional.silu(gu[:, :i_s]) * gu[:, i_s:]).to(torch.bfloat16).float()
    return (h @ w8g_dequant(sq2, ss2).T).to(torch.bfloat16)
