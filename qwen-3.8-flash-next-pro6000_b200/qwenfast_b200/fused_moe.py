"""A quant method for SGLang's ``FusedMoE`` layer that runs the routed experts on this library's W4A16 kernel.

It fills the slot that ``CompressedTensorsW4A4Nvfp4MoE`` fills for the reference's NVFP4 checkpoint
(serve/overlays/sglang/srt/layers/quantization/compressed_tensors/schemes/compressed_tensors_w4a4_nvfp4_moe.py:62-95
``create_weights``, :173-190 ``process_weights_after_loading``, :388-410 ``apply_weights``), for experts in this
build's format: int4 codes with zero point 8, eight per int32 along K (lowest k in the low nibble), one bf16 scale per
128 k. Where the reference hands the routed experts to a Marlin MoE runner, ``apply_weights`` calls
``torch.ops.qwenfast_b200.a16_moe_decode``: the persistent decode MoE kernel, routed experts only (the block adds the
shared expert itself), out = bf16(sum over the top-k positions of bf16(bf16(expert_out) * bf16(topk_w))).

Token counts up to 64 are one launch; larger batches (prefill) run as 64-token launches of the same kernel (each
streams its routed experts again: correct, not a prefill-speed path). Nothing here imports sglang; the result is
returned as SGLang's ``StandardCombineInput`` when sglang is importable, else as ``CombineInput`` below (the same
``hidden_states`` attribute).
"""
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib, formats, ops, torch_ops

BF16 = torch.bfloat16


@dataclass
class CombineInput:
    """The routed experts' output, under the attribute name of SGLang's ``StandardCombineInput``."""
    hidden_states: torch.Tensor


def _combine_input(out: torch.Tensor):
    try:   # SGLang's own type when it is present (the runner's callers expect it)
        from sglang.srt.layers.moe.token_dispatcher.standard import StandardCombineInput  # type: ignore
        return StandardCombineInput(hidden_states=out)
    except Exception:   # noqa: BLE001 -- no sglang here: the stand-in with the same attribute
        return CombineInput(hidden_states=out)


class QwenFastW4A16MoEMethod:
    """``create_weights`` / ``process_weights_after_loading`` / ``apply_weights`` (and the older ``apply``) of a
    FusedMoE quant method. ``process_weights_after_loading`` repacks the canonical int4 experts once into the kernel
    layout (``formats.repack_w4``) and drops the canonical copies, so the layer holds one copy of its experts."""

    def __init__(self, group_size: int = 128, max_tokens_per_launch: int = _lib.QF_MAX_TOKENS):
        if group_size != 128:
            raise RuntimeError("QwenFastW4A16MoEMethod: the kernel takes group-128 scales")
        self.group_size = group_size
        self.max_tokens = max(1, min(int(max_tokens_per_launch), _lib.QF_MAX_TOKENS))

    # ---------------------------------------------------------------------------------------------- weights
    def create_weights(self, layer: torch.nn.Module, num_experts: int, hidden_size: int,
                       intermediate_size_per_partition: int, params_dtype: torch.dtype = BF16, **extra_weight_attrs):
        """Canonical checkpoint parameters: w13_qweight int32 [E, 2I, H/8] (gate rows, then up rows),
        w13_scales bf16 [E, 2I, H/128], w2_qweight int32 [E, H, I/8], w2_scales bf16 [E, H, I/128]. Extra attributes
        (SGLang's ``weight_loader`` and friends) are set on every parameter."""
        E, H, I = num_experts, hidden_size, intermediate_size_per_partition
        if H % 256 or I % 128:
            raise RuntimeError(f"QwenFastW4A16MoEMethod: H must be a multiple of 256 and I of 128 (H={H}, I={I})")
        layer.params_dtype = params_dtype
        shapes = dict(w13_qweight=((E, 2 * I, H // 8), torch.int32), w13_scales=((E, 2 * I, H // 128), BF16),
                      w2_qweight=((E, H, I // 8), torch.int32), w2_scales=((E, H, I // 128), BF16))
        for name, (shape, dt) in shapes.items():
            prm = torch.nn.Parameter(torch.empty(shape, dtype=dt), requires_grad=False)
            for k, v in extra_weight_attrs.items():
                setattr(prm, k, v)
            layer.register_parameter(name, prm)
        layer._qf_shape = (E, H, I)

    def process_weights_after_loading(self, layer: torch.nn.Module) -> None:
        """Repack once into the kernel layout (exact; ``formats.unpack_w4`` restores the canonical tensors)."""
        E, H, I = layer._qf_shape
        wk13, sk13 = formats.repack_w4(layer.w13_qweight.data, layer.w13_scales.data, gated=True)
        wk2, sk2 = formats.repack_w4(layer.w2_qweight.data, layer.w2_scales.data, gated=False)
        for name in ("w13_qweight", "w13_scales", "w2_qweight", "w2_scales"):
            delattr(layer, name)
        layer.w13_weight = torch.nn.Parameter(wk13, requires_grad=False)
        layer.w13_weight_scale = torch.nn.Parameter(sk13, requires_grad=False)
        layer.w2_weight = torch.nn.Parameter(wk2, requires_grad=False)
        layer.w2_weight_scale = torch.nn.Parameter(sk2, requires_grad=False)

    # ---------------------------------------------------------------------------------------------- forward
    def routed_experts(self, layer: torch.nn.Module, x: torch.Tensor, topk_ids: torch.Tensor,
                       topk_weights: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """bf16 [M, H]: the top-k weighted sum of the routed experts for every token (no shared expert)."""
        E, H, I = layer._qf_shape
        if x.dim() != 2 or x.shape[1] != H or x.dtype != BF16:
            raise RuntimeError(f"QwenFastW4A16MoEMethod: hidden states must be bf16 [M, {H}]")
        if not x.is_cuda:
            raise RuntimeError("QwenFastW4A16MoEMethod: the routed experts run on CUDA tensors only (no CPU path)")
        ids = topk_ids.to(torch.int32).contiguous()
        w = topk_weights.to(torch.float32).contiguous()
        topk = ids.shape[1]
        x = x.contiguous()
        out = torch.empty_like(x) if out is None else out
        if x.shape[0] == 0:
            return out
        qops = torch_ops.load()
        from .overlay import _a16_bufs   # the per-(device, stream, shape) workspace of the decode kernel
        b = _a16_bufs(x.device, H, I, topk, 0)
        if not torch.compiler.is_compiling():
            ops.check_moe_error(b["ctrl"])
        none = b["none"]
        for m0 in range(0, x.shape[0], self.max_tokens):
            m1 = min(x.shape[0], m0 + self.max_tokens)
            qops.a16_moe_decode(x[m0:m1], ids[m0:m1], w[m0:m1], layer.w13_weight, layer.w13_weight_scale, none,
                                layer.w2_weight, layer.w2_weight_scale, none, none, none, b["hbuf"], b["ybuf"], b["gl"],
                                b["ctrl"], out[m0:m1], 4, b["none_i64"], b["pbuf"], none, none, none, none,
                                b["shbuf"])
        return out

    def apply_weights(self, layer: torch.nn.Module, dispatch_output):
        """SGLang's quant-method entry (compressed_tensors_w4a4_nvfp4_moe.py:388-410): ``dispatch_output`` carries
        ``hidden_states`` and ``topk_output`` (``topk_weights``, ``topk_ids``); returns the combine input."""
        topk = dispatch_output.topk_output
        out = self.routed_experts(layer, dispatch_output.hidden_states, topk.topk_ids, topk.topk_weights)
        return _combine_input(out)

    def apply(self, layer: torch.nn.Module, x: torch.Tensor, topk_output, **kwargs) -> torch.Tensor:
        """The older FusedMoE entry (``apply(layer, x, topk_output)``): the routed output tensor."""
        return self.routed_experts(layer, x, topk_output.topk_ids, topk_output.topk_weights)
