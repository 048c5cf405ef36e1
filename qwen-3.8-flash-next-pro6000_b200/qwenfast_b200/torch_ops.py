"""``torch.ops.qwenfast_b200``: the decode-path kernels as torch custom operators.

``load()`` loads ``libqwenfast_b200_torch.so`` (built by ``build.build``), whose ``TORCH_LIBRARY(qwenfast_b200, m)``
registers ``router_topk``, ``a16_moe_decode``, ``a16_moe_decode_nvfp4``, ``moe_layer_decode``, ``w8g_gemm``,
``w8g_unpack`` and ``w8a8_gemm`` with CUDA and Meta (shape) kernels -- the reference extension's op names and argument
roles (serve/qwenfast/qf_bind.cpp), callable from eager code, CUDA graphs and ``torch.compile``. Loading it needs no
GPU.
"""
import os

import torch

from . import _lib

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libqwenfast_b200_torch.so")
_loaded = False


def load(path: str = LIB_PATH):
    """Register the operators (once); raises RuntimeError when the library is not built."""
    global _loaded
    if _loaded:
        return torch.ops.qwenfast_b200
    if not os.path.exists(path):
        raise RuntimeError(f"qwenfast_b200: {path} is missing; build it with qwenfast_b200.build.build()")
    _lib.load()   # the C-ABI library it links against (also resolvable through its $ORIGIN rpath)
    torch.ops.load_library(path)
    _loaded = True
    return torch.ops.qwenfast_b200


OP_NAMES = ("router_topk", "a16_moe_decode", "a16_moe_decode_nvfp4", "moe_layer_decode", "w8g_gemm", "w8g_unpack",
            "w8a8_gemm")
