"""qwenfast_b200 -- B200 (sm_100a) kernels for the Qwen3-Next-style decode MoE path, behind the reference's op API.

Ops (reference names, serve/qwenfast/qf_bind.cpp): ``router_topk``, ``a16_moe_decode``, ``w8g_gemm``,
``w8g_unpack``; plus ``w8a8_gemm`` (per-token / per-channel INT8) and the weight repackers in ``formats``.
The kernels live in ``libqwenfast_b200.so`` (C ABI: include/qwenfast_b200.h), built in-tree by ``build.build()``.
"""
from . import _lib, formats, synthetic  # noqa: F401
from .ops import (LayerStep, MoELayerWeights, W8A8Linear, W8Linear, a16_moe_decode,  # noqa: F401
                  moe_error_word, moe_layer_step, moe_workspace, router_bufs, router_topk, w8a8_gemm, w8g_gemm, w8g_unpack)

__all__ = ["router_topk", "a16_moe_decode", "w8g_gemm", "w8g_unpack", "w8a8_gemm", "moe_workspace", "router_bufs",
           "moe_layer_step", "LayerStep", "MoELayerWeights", "W8Linear", "W8A8Linear", "moe_error_word", "formats",
           "synthetic"]
