"""Host side of the reference's SGLang overlay for this path (serve/overlays/sglang/srt/qwenfast.py): the gates that
decide, per call, whether a decode MoE block or an INT8 linear goes to the sm_100a kernels, the per-(device, stream)
scratch caches, and the calls themselves. Same function names, argument meaning and decline behaviour as the
reference; the shape gates follow this build's limits and weight formats instead of the reference's fixed model
(H = 2560, M <= 8, NVFP4 / Marlin experts):

* ``w8_quant`` / ``w8_linear`` -- the INT8 (W8A16, group-scaled) dense projections
  (qwenfast.py:301-315, 337-360). A call the kernel does not take (bias, more than 64 rows, unsupported
  K, N or layout) declines to the reference's own fallback: the weight rows are unpacked on the device into bf16
  (``w8g_unpack``) and multiplied with ``torch.nn.functional.linear``.
* ``w8a8_linear`` -- the per-token W8A8 projection (no reference code); more than 16 rows run as 16-row calls of
  the same kernel (per-token quantisation makes rows independent, so the result is the same bits).
* ``why_not`` / ``_a16_ok`` / ``_a16_shared`` / ``dual`` -- the decode MoE block (qwenfast.py:1076-1201): the
  router-first fast path, the routed experts in the W4A16 kernel with the shared expert inside it when its weights
  qualify, otherwise passed in precomputed. ``dual`` returns ``(out, None)`` like the reference (the gated shared
  term is already added). SGLang's own routing post-processing (``_post_process_topk_ids``, the expert
  distribution recorder) is the caller's, as it is not part of this library.

Blocks and layers are read by attribute, so SGLang's module objects (``Qwen2MoeSparseMoeBlock``, ``FusedMoE``,
``LinearBase``) and any object with the same attribute names work. Nothing here imports sglang. The kernels are
called through the registered operators ``torch.ops.qwenfast_b200.*`` (``torch_ops``), so the fast paths also run
inside ``torch.compile``d forwards; the host mirror of the MoE error word is checked on eager calls only.
"""
import os
from collections import namedtuple
from typing import Optional

import torch

from . import _lib, formats, ops, torch_ops

BF16 = torch.bfloat16
TopKOutput = namedtuple("TopKOutput", ["topk_weights", "topk_ids", "router_logits"])   # SGLang StandardTopKOutput


# ------------------------------------------------------------------------------------------------ INT8 linear
@torch.no_grad()
def w8_quant(w: torch.Tensor, rows_per_chunk: int = 8192) -> dict:
    """bf16 [N, K] -> dict(kind="w8", q int8 [N, K], s bf16 [N, K/G], shape, G): symmetric INT8 with one bf16 scale
    per group of G = 128 k (64 when K % 128 != 0), the scale rounded to bf16 before quantising, so ``q * s`` is the
    exact dequantised weight (qwenfast.py:301-315). Load-time preparation, run where ``w`` lives."""
    N, K = w.shape
    G = 128 if K % 128 == 0 else 64
    q = torch.empty((N, K), dtype=torch.int8, device=w.device)
    sc = torch.empty((N, K // G), dtype=BF16, device=w.device)
    for r0 in range(0, N, rows_per_chunk):
        r1 = min(N, r0 + rows_per_chunk)
        xg = w[r0:r1].float().view(r1 - r0, K // G, G)
        s16 = (xg.abs().amax(2) / 127).clamp_(min=1e-30).to(BF16)
        q[r0:r1] = (xg / s16.float().unsqueeze(-1)).round_().clamp_(-127, 127).to(torch.int8).view(r1 - r0, K)
        sc[r0:r1] = s16
    return dict(kind="w8", q=q, s=sc, shape=(N, K), G=G)


def w8_route(entry, x: torch.Tensor, bias=None) -> Optional[str]:
    """None when ``w8_linear`` runs the kernel for this call, else the first failing condition (the decline path's
    reason): the gate of qwenfast.py:346-349 with this build's limits (M <= 64 rows, output rows a multiple of 8,
    K % 64 == 0, G 128 or 64)."""
    p, r0, r1 = entry
    N, K = p["shape"]
    x2 = x.reshape(-1, K)
    M = x2.shape[0]
    checks = (
        ("bias", bias is None),
        ("rows", 1 <= M <= _lib.QF_MAX_TOKENS),
        ("shape", r1 - r0 >= 8 and (r1 - r0) % 8 == 0),
        ("group", p["G"] in (64, 128) and K % 64 == 0 and K % p["G"] == 0),
        ("dtype", x2.dtype == BF16),
        ("layout", x2.stride(1) == 1 and x2.stride(0) % 8 == 0 and x2.data_ptr() % 16 == 0),
        ("device", x2.is_cuda),
    )
    return next((name for name, good in checks if not good), None)


_pk_scratch = {}


def _w8_unpack_rows(p: dict, r0: int, r1: int) -> torch.Tensor:
    """bf16 [r1 - r0, K] = q * s of weight rows r0 .. r1, unpacked on the device into a reused per-device buffer
    (qwenfast.py:318-328)."""
    N, K = p["shape"]
    dev = p["q"].device
    need = (r1 - r0) * K
    buf = _pk_scratch.get(dev)
    if buf is None or buf.numel() < need:
        buf = _pk_scratch[dev] = torch.empty(need, dtype=BF16, device=dev)
    w = buf[:need].view(r1 - r0, K)
    torch_ops.load().w8g_unpack(p["q"][r0:r1], p["s"][r0:r1], w)
    return w


def w8_linear(entry, x: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = x @ (q * s)[r0:r1]^T (+ bias) for ``entry = (p, r0, r1)``, p from ``w8_quant`` (qwenfast.py:337-360):
    the W8A16 kernel when ``w8_route`` accepts the call, else the unpack + ``F.linear`` decline path."""
    p, r0, r1 = entry
    N, K = p["shape"]
    shp = x.shape
    x2 = x.reshape(-1, K)
    n_out = r1 - r0
    if x2.shape[0] == 0:
        return x.new_empty((*shp[:-1], n_out))
    if w8_route(entry, x, bias) is None:
        q, s = (p["q"], p["s"]) if (r0 == 0 and r1 == N) else (p["q"][r0:r1], p["s"][r0:r1])
        y = torch_ops.load().w8g_gemm(x2, q, s, 0)
        return y.view(*shp[:-1], n_out)
    w = _w8_unpack_rows(p, r0, r1)
    return torch.nn.functional.linear(x2, w, bias).view(*shp[:-1], n_out)


def w8a8_prepare(q: torch.Tensor, sw: torch.Tensor) -> dict:
    """Load time: int8 [N, K] weight + fp32 per-channel scales -> the W8A8 entry (weight in the kernel layout)."""
    return dict(kind="w8a8", qk=formats.repack_w8(q), sw=sw.float().contiguous(), shape=tuple(q.shape))


def w8a8_linear(p: dict, x: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Per-token W8A8 projection (``w8a8_gemm``): rows quantised one by one, so more than 16 rows run as 16-row
    calls with identical results. A bias is added in fp32 after the kernel's bf16 rounding, then rounded again."""
    N, K = p["shape"]
    shp = x.shape
    x2 = x.reshape(-1, K)
    M = x2.shape[0]
    if M == 0:
        return x.new_empty((*shp[:-1], N))
    if x2.stride(1) != 1 or x2.stride(0) % 8 != 0 or x2.data_ptr() % 16 != 0:
        x2 = x2.contiguous()
    y = torch.empty(M, N, dtype=BF16, device=x2.device)
    for m0 in range(0, M, 16):
        y[m0:m0 + 16] = torch_ops.load().w8a8_gemm(x2[m0:m0 + 16], p["qk"], p["sw"])
    if bias is not None:
        y = (y.float() + bias.float()).to(BF16)
    return y.view(*shp[:-1], N)


# ------------------------------------------------------------------------------------------------ MoE block
_router_scratch = {}
_a16_scratch = {}


def _stream_key(device):
    dev = torch.device(device)
    return dev, torch.cuda.current_stream(dev).cuda_stream


def _router_bufs(device):
    """Router scratch per (device, stream) (qwenfast.py:1032-1038), sized for the kernel's limits."""
    key = _stream_key(device)
    b = _router_scratch.get(key)
    if b is None:
        b = _router_scratch[key] = ops.router_bufs(key[0], _lib.QF_MAX_TOKENS, _lib.QF_MAX_EXPERTS)
    return b


def _a16_bufs(device, H: int, I: int, topk: int, Is: int) -> dict:
    """MoE scratch per (device, stream, layer shape) (qwenfast.py:1044-1059), sized for the largest token count:
    one workspace serves every M <= 64 (its zero-kept counters sit at the same place for any M)."""
    key = _stream_key(device) + (H, I, topk, Is)
    b = _a16_scratch.get(key)
    if b is None:
        b = _a16_scratch[key] = ops.moe_workspace(_lib.QF_MAX_TOKENS, H, I, topk, Is, key[0])
    return b


def _a16_weights(block):
    """(w13, s13, g13, w2, s2, g2) of a block's routed experts in this build's kernel layout (``formats.repack_w4``):
    a decode copy attached as ``experts._qf_a16``, else the experts' own parameters (qwenfast.py:1062-1071)."""
    ex = block.experts
    o = getattr(ex, "_qf_a16", None)
    if o is not None:
        return o
    return tuple(getattr(ex, n, None) for n in ("w13_weight", "w13_weight_scale", "w13_weight_scale_2",
                                                "w2_weight", "w2_weight_scale", "w2_weight_scale_2"))


def _a16_format(block) -> str:
    """"nvfp4" when the routed experts carry E4M3 group-16 scales (uint8, ``formats.repack_nvfp4``), else "int4"."""
    s13 = _a16_weights(block)[1]
    return "nvfp4" if s13 is not None and s13.dtype == torch.uint8 else "int4"


def _a16_ok(block, x: torch.Tensor) -> bool:
    """The routed experts qualify for the W4A16 kernel (qwenfast.py:1074-1089): int32 kernel-layout codes of E
    experts with either bf16 group-128 scales (int4) or E4M3 group-16 scales (NVFP4, the reference's format, as uint8
    from ``formats.repack_nvfp4``), optional bf16 [E] global multipliers, and the shared-expert gate (bf16 [H], no
    bias)."""
    w13, s13, g13, w2, s2, g2 = _a16_weights(block)
    sg = getattr(block, "shared_expert_gate", None)
    gw = getattr(block.gate, "weight", None)
    if not (x.dim() == 2 and x.dtype == BF16 and x.is_contiguous() and gw is not None):
        return False
    M, H = x.shape
    E = gw.shape[0]

    def shaped(t, dtype, shape):
        return t is not None and t.dtype == dtype and tuple(t.shape) == shape and t.is_contiguous()

    if w2 is None or w2.dim() != 2 or w2.shape[0] != E:
        return False
    I = w2.shape[1] * 8 // H
    sdt, grp = (torch.uint8, 16) if _a16_format(block) == "nvfp4" else (BF16, 128)
    return (
        1 <= M <= _lib.QF_MAX_TOKENS and I >= 128 and I % 128 == 0 and w2.shape[1] * 8 == H * I
        and shaped(w13, torch.int32, (E, 2 * I * H // 8)) and shaped(s13, sdt, (E, 2 * I * H // grp))
        and shaped(w2, torch.int32, (E, H * I // 8)) and shaped(s2, sdt, (E, H * I // grp))
        and (g13 is None or (g13.dtype == BF16 and g13.numel() == E))
        and (g2 is None or (g2.dtype == BF16 and g2.numel() == E))
        and sg is not None and getattr(sg, "weight", None) is not None and sg.weight.numel() == H
        and sg.weight.dtype == BF16 and getattr(sg, "bias", None) is None
    )


def _a16_shared(block):
    """Kernel-layout bf16 weights (gate_up, down, Is) of the shared expert when the MoE kernel can compute it itself
    (bf16 gate_up [2 Is, H] and down [H, Is], SiluAndMul, no biases, Is % 64 == 0 and <= 1024), else None: the
    caller's shared expert runs separately and its output is passed in (qwenfast.py:1092-1113). Cached on the block
    (``_qf_a16sh``); the repack runs once, on the weights' device."""
    hit = getattr(block, "_qf_a16sh", 0)
    if hit != 0:
        return hit
    hit = None
    se = getattr(block, "shared_expert", None)
    act = type(getattr(se, "act_fn", None)).__name__
    if os.environ.get("QWENFAST_A16SHARED", "1") == "1" and se is not None and act == "SiluAndMul":
        gu = getattr(getattr(se, "gate_up_proj", None), "weight", None)
        dn = getattr(getattr(se, "down_proj", None), "weight", None)
        if (gu is not None and dn is not None and gu.dtype == BF16 and dn.dtype == BF16 and gu.is_cuda
                and gu.dim() == 2 and dn.dim() == 2 and gu.shape[0] == 2 * dn.shape[1] and gu.shape[1] == dn.shape[0]
                and dn.shape[1] % 64 == 0 and 64 <= dn.shape[1] <= 1024
                and getattr(se.gate_up_proj, "bias", None) is None and getattr(se.down_proj, "bias", None) is None):
            hit = (formats.repack_bf16(gu.contiguous(), gated=True), formats.repack_bf16(dn.contiguous(), gated=False),
                   dn.shape[1])
    block._qf_a16sh = hit
    return hit


def why_not(block, x: torch.Tensor, lora_active: bool = False) -> Optional[str]:
    """None when the router-first fast path applies to ``block`` for input ``x``, else the first failing condition
    (qwenfast.py:1127-1161). ``lora_active`` stands for SGLang's experimental-LoRA module flag."""
    topk = getattr(block, "topk", None)
    cfg = getattr(topk, "topk_config", None)
    gate = getattr(block, "gate", None)
    gw = getattr(gate, "weight", None)
    H = x.shape[-1] if x.dim() >= 1 else 0
    checks = (
        ("shape", x.dim() == 2 and 1 <= x.shape[0] <= _lib.QF_MAX_TOKENS and H % 256 == 0 and 256 <= H <= 4096),
        ("dtype", x.dtype == BF16 and x.is_contiguous()),
        ("shared", getattr(block, "shared_expert", None) is not None
         and not getattr(block, "enable_shared_expert_fusion", False)),
        ("lora", not lora_active),
        ("inplace", getattr(getattr(getattr(block, "experts", None), "moe_runner_config", None), "inplace", True)
         is False),
        ("gate", gw is not None and gw.dtype == BF16 and gw.dim() == 2 and gw.shape[1] == H and gw.is_contiguous()
         and gw.shape[0] % 16 == 0 and gw.shape[0] <= _lib.QF_MAX_EXPERTS and getattr(gate, "bias", None) is None
         and type(getattr(gate, "quant_method", None)).__name__ in ("UnquantizedLinearMethod", "NoneType")),
        ("topk", cfg is not None and 1 <= cfg.top_k <= _lib.QF_MAX_TOPK and cfg.top_k <= gw.shape[0]
         and not getattr(cfg, "use_grouped_topk", False) and getattr(cfg, "num_fused_shared_experts", 0) == 0
         and getattr(cfg, "custom_routing_function", None) is None and getattr(cfg, "correction_bias", None) is None
         and not getattr(cfg, "apply_routed_scaling_factor_on_output", False)
         and getattr(cfg, "scoring_func", "softmax") == "softmax" and getattr(cfg, "output_format", None) is None),
        ("waterfill", not getattr(topk, "enable_waterfill", False) and getattr(topk, "waterfill_balancer", None) is None),
        ("simulate", os.environ.get("SGLANG_SIMULATE_UNIFORM_EXPERTS", "") in ("", "0", "false")
         and os.environ.get("SGLANG_SIMULATE_ROUND_ROBIN_EXPERTS", "") in ("", "0", "false")),
        ("device", x.is_cuda and gw.device == x.device),
    )
    return next((name for name, good in checks if not good), None)


def dual(block, hidden_states: torch.Tensor, orig=None, lora_active: bool = False, shared_output=None):
    """The decode MoE block's forward (qwenfast.py:1163-1201). Declined calls go to ``orig(block, hidden_states)``
    (the stock forward), or raise ``RuntimeError`` naming the reason when no ``orig`` is given.

    Routed experts in the W4A16 kernel (``_a16_ok``): one launch runs router, experts, shared expert (its weights
    in the kernel, or ``shared_output`` / the block's ``_forward_shared_experts(x, apply_gate=False)`` passed in,
    ungated) and the gated combine; returns ``(out, None)``. Otherwise the router kernel runs and the block's own ``experts`` module gets a
    ``TopKOutput``; returns ``(routed, shared_output)`` as the reference does. Either way the step's routing
    (``TopKOutput``: weights, ids, bf16 logits) is left in ``block._qf_topk`` for the caller's routing
    post-processing and expert-distribution recording (qwenfast.py:1181-1183)."""
    reason = why_not(block, hidden_states, lora_active)
    if reason is not None:
        if orig is not None:
            return orig(block, hidden_states)
        raise RuntimeError(f"qwenfast_b200 dual: fast path declined ({reason})")
    cfg = block.topk.topk_config
    x = hidden_states
    M, H = x.shape
    qops = torch_ops.load()
    none = torch.empty(0, dtype=BF16, device=x.device)
    opt = lambda t: none if t is None else t   # noqa: E731 -- empty tensors mean "absent" to the operators
    if _a16_ok(block, x):
        w13, s13, g13, w2, s2, g2 = _a16_weights(block)
        sh = _a16_shared(block)
        shared = None
        if sh is None:
            shared = (shared_output if shared_output is not None
                      else block._forward_shared_experts(x.clone(), apply_gate=False))   # the kernel gates it
            shared = shared.contiguous()
        I = w2.shape[1] * 8 // H
        b = _a16_bufs(x.device, H, I, cfg.top_k, sh[2] if sh is not None else 0)
        if not torch.compiler.is_compiling():
            ops.check_moe_error(b["ctrl"])
        out = torch.empty_like(x)
        wg = block.shared_expert_gate.weight.view(-1)
        if _a16_format(block) == "nvfp4":   # the reference's order: the router op, then the MoE op
            scratch, counter = _router_bufs(x.device)
            tw, ids, logits = qops.router_topk(x, block.gate.weight, cfg.top_k, bool(cfg.renormalize), scratch,
                                               counter, True)
            qops.a16_moe_decode_nvfp4(x, ids, tw, w13, s13, opt(g13), w2, s2, opt(g2), wg, opt(shared), b["hbuf"],
                                      b["ybuf"], b["gl"], b["ctrl"], out, 4, b["none_i64"], b["pbuf"],
                                      sh[0] if sh is not None else none, none, sh[1] if sh is not None else none,
                                      none, b["shbuf"])
            block._qf_topk = TopKOutput(tw, ids, logits)
            return out, None
        tw, ids, logits = qops.moe_layer_decode(x, block.gate.weight, bool(cfg.renormalize), w13, s13, opt(g13), w2,
                                                s2, opt(g2), wg, opt(shared), sh[0] if sh is not None else none,
                                                sh[1] if sh is not None else none, cfg.top_k, b["hbuf"], b["ybuf"],
                                                b["gl"], b["ctrl"], b["pbuf"], b["shbuf"], out)
        block._qf_topk = TopKOutput(tw, ids, logits)
        return out, None
    scratch, counter = _router_bufs(x.device)
    tw, ids, logits = qops.router_topk(x, block.gate.weight, cfg.top_k, bool(cfg.renormalize), scratch, counter, True)
    if shared_output is None:
        shared_output = block._forward_shared_experts(x.clone(), apply_gate=True)
    block._qf_topk = TopKOutput(tw, ids, logits)
    return block.experts(x, block._qf_topk), shared_output
