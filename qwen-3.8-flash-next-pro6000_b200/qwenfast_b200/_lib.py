"""ctypes binding of ``libqwenfast_b200.so`` (the C ABI declared in ``include/qwenfast_b200.h``).

The library is loaded from this directory. There is no fallback: when it is missing, every op raises.
"""
import ctypes
import os

LIB_NAME = "libqwenfast_b200.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

QF_OK = 0
QF_ERR_UNSUPPORTED = -3
QF_MAX_TOKENS = 64
QF_MAX_TOPK = 16
QF_MAX_EXPERTS = 1024
QF_MOE_CTRL_WORDS = 2048
QF_MOE_CTRL_ERR = 3
QF_MOE_CTRL_MIRROR = 2046
QF_MOE_ERR_TIMEOUT = 0x1
QF_MOE_ERR_BAD_EXPERT = 0x2
QF_MOE_ERR_PIPELINE = 0x4

_p = ctypes.c_void_p
_i = ctypes.c_int
_l = ctypes.c_int64

# name -> argument types (every function returns int)
SIGNATURES = {
    "qf_version": [],
    "qf_router_topk": [_p, _p, _i, _i, _i, _i, _i, _p, _p, _p, _p, _l, _p, _i, _p],
    "qf_router_topk_noalloc": [_p, _p, _i, _i, _i, _i, _i, _p, _p, _p, _i, _p],
    "qf_a16_moe_workspace": [_i, _i, _i, _i, _i, _p, _p, _p, _p, _p, _p],
    "qf_a16_moe_decode": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p,
                          _p, _l, _p, _l, _p, _l, _p, _l, _p, _l, _p, _l,
                          _p, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _p, _i, _p],
    "qf_a16_moe_decode_nvfp4": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p,
                                _p, _l, _p, _l, _p, _l, _p, _l, _p, _l, _p, _l,
                                _p, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _p, _i, _p],
    "qf_moe_layer_decode": [_p, _p, _p, _i, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p,
                            _p, _l, _p, _l, _p, _l, _p, _l, _p, _l, _p, _l,
                            _p, _i, _i, _i, _i, _i, _i, _i, _i, _i, _p, _i, _p],
    "qf_moe_layer_decode_nvfp4": [_p, _p, _p, _i, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p,
                                  _p, _l, _p, _l, _p, _l, _p, _l, _p, _l, _p, _l,
                                  _p, _i, _i, _i, _i, _i, _i, _i, _i, _i, _p, _i, _p],
    "qf_moe_combine": [_p, _p, _p, _i, _p, _i, _i, _i, _i, _p],
    "qf_w4_repack": [_p, _p, _p, _p, _i, _i, _i, _i, _p],
    "qf_w4_unpack": [_p, _p, _p, _p, _i, _i, _i, _i, _p],
    "qf_bf16_repack": [_p, _p, _i, _i, _i, _p],
    "qf_bf16_unpack": [_p, _p, _i, _i, _i, _p],
    "qf_w8g_gemm": [_p, _l, _p, _p, _p, _l, _i, _i, _i, _i, _i, _p, _l, _i, _p],
    "qf_w8g_fixup_elems": [_i, _p],
    "qf_w8g_take_status": [_p],
    "qf_w8g_unpack": [_p, _p, _p, _l, _i, _i, _p],
    "qf_w8a8_gemm": [_p, _l, _p, _p, _p, _l, _i, _i, _i, _p, _p, _p, _p, _i, _p],
    "qf_w8_repack": [_p, _p, _i, _i, _p],
    "qf_w8a8_take_status": [_p],
    "qf_w8a8_fixup_elems": [_i, _p],
    "qf_w8_unpack": [_p, _p, _i, _i, _p],
}

_lib = None


def load(path: str = LIB_PATH):
    """Load (once) and return the native library; raises RuntimeError when it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(f"qwenfast_b200: native library {path} is missing; build it with qwenfast_b200.build.build()")
    lib = ctypes.CDLL(path)
    lib.qf_last_error.restype = ctypes.c_char_p
    lib.qf_last_error.argtypes = []
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = ctypes.c_int
        fn.argtypes = args
    _lib = lib
    return lib


def exported_symbols():
    return ["qf_last_error"] + list(SIGNATURES)


class Unsupported(RuntimeError):
    """A valid request this build declines (QF_ERR_UNSUPPORTED), e.g. a fused layer-step whose grid cannot be
    co-resident; callers that have another path take it."""


def check(status: int, what: str = ""):
    """Raise RuntimeError (the reference's TORCH_CHECK failure type) for a non-zero status (``Unsupported`` for
    QF_ERR_UNSUPPORTED)."""
    if status != QF_OK:
        msg = load().qf_last_error().decode(errors="replace")
        text = f"{what}: {msg}" if what and not msg.startswith(what) else msg
        raise Unsupported(text) if status == QF_ERR_UNSUPPORTED else RuntimeError(text)
