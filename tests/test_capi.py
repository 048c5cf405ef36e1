"""The C ABI library: it loads, exports every entry point include/qwenfast_b200.h declares, and its host-side
argument checks reject bad requests before anything is enqueued (so these calls need no GPU)."""
import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "qwenfast_b200.h")


def declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^(?:const char\*|int)\s+(qf_\w+)\(", src, flags=re.M)))


def test_exports_every_declared_symbol(lib):
    names = declared()
    assert len(names) >= 13
    for n in names:
        assert hasattr(lib, n), n
    from qwenfast_b200 import _lib
    assert set(names) == set(_lib.exported_symbols())


def test_version_and_error_text(lib):
    assert lib.qf_version() >= 1
    assert isinstance(lib.qf_last_error(), bytes)


def test_router_rejects_bad_arguments(lib):
    from qwenfast_b200 import _lib
    p = ctypes.c_void_p(16)
    st = lib.qf_router_topk(p, p, 0, 2048, 512, 10, 1, p, p, p, p, 512 * 64, p, 1, None)
    assert st == -1 and b"rows" in lib.qf_last_error()
    st = lib.qf_router_topk(p, p, 4, 2048, 512, 17, 1, p, p, p, p, 512 * 64, p, 1, None)
    assert st == -1 and b"topk" in lib.qf_last_error()
    st = lib.qf_router_topk(p, p, 4, 2048, 512, 10, 1, p, p, p, p, 100, p, 1, None)
    assert st == -1 and b"scratch" in lib.qf_last_error()
    st = lib.qf_router_topk(None, p, 4, 2048, 512, 10, 1, p, p, p, p, 512 * 64, p, 1, None)
    assert st == -1
    with pytest.raises(RuntimeError, match="rows"):
        _lib.check(lib.qf_router_topk(p, p, 65, 2048, 512, 10, 1, p, p, p, p, 1 << 20, p, 1, None), "router_topk")


def test_moe_rejects_bad_arguments(lib):
    p = ctypes.c_void_p(256)
    # x, ids, w, w13, s13, gs13, w2, s2, gs2, w_gate, shared (absent), sh_w13, sh_w2 + scratch + out
    head = [p] * 10 + [None, p, p]
    args = head + [p, 1 << 30, p, 1 << 30, p, 64, p, 2048, p, 1 << 26, p, 1 << 30, p]
    ok_dims = [10, 2048, 512, 512, 10, 512]
    st = lib.qf_a16_moe_decode(*args, 10, 2048, 512, 512, 10, 512, 1, 0, 0, 512, None, 1, None)
    assert st == -1 and b"phase" in lib.qf_last_error()
    st = lib.qf_a16_moe_decode(*args, 65, 2048, 512, 512, 10, 512, 4, 0, 0, 512, None, 1, None)
    assert st == -1 and b"M must" in lib.qf_last_error()
    st = lib.qf_a16_moe_decode(*args, *ok_dims, 4, 0, 0, 513, None, 1, None)
    assert st == -1 and b"expert range" in lib.qf_last_error()
    small = head + [p, 16, p, 1 << 30, p, 64, p, 2048, p, 1 << 26, p, 1 << 30, p]
    st = lib.qf_a16_moe_decode(*small, *ok_dims, 4, 0, 0, 512, None, 1, None)
    assert st == -1 and b"scratch" in lib.qf_last_error()
    unaligned = [ctypes.c_void_p(258)] + head[1:] + args[13:]
    st = lib.qf_a16_moe_decode(*unaligned, *ok_dims, 4, 0, 0, 512, None, 1, None)
    assert st == -1 and b"aligned" in lib.qf_last_error()


def test_gemms_reject_bad_arguments(lib):
    p = ctypes.c_void_p(256)
    assert lib.qf_w8g_gemm(p, 2048, p, p, p, 2048, 0, 2048, 2048, 128, 0, p, 1 << 30, 0, None) == -1
    assert lib.qf_w8g_gemm(p, 2048, p, p, p, 2048, 4, 2048, 2048, 96, 0, p, 1 << 30, 0, None) == -1
    assert lib.qf_w8g_gemm(p, 2048, p, p, p, 2048, 4, 2004, 2048, 128, 0, p, 1 << 30, 0, None) == -1   # N % 8
    assert lib.qf_w8a8_gemm(p, 2048, p, p, p, 2048, 4, 2048, 2000, p, p, None, None, 1, None) == -1
    assert lib.qf_w4_repack(p, p, p, p, 1, 100, 256, 1, None) == -1


def test_workspace_sizes(lib):
    v = [ctypes.c_int64() for _ in range(6)]
    assert lib.qf_a16_moe_workspace(10, 2048, 512, 10, 512, *[ctypes.byref(a) for a in v]) == 0
    hb, yb, gl, ctrl, pb, sh = (a.value for a in v)
    assert hb == 10 * 10 * 512 * 2 and yb == 10 * 11 * 2048 * 2 and gl == 10 and ctrl == 2048
    units = 10 * 10 * (2 * 512 // 128)   # gate_up k-half partials: M * topk token groups x 2I / 128 tiles
    cnt = 64 * 10 * (2 * 512 // 128)     # their zero-kept counters, sized for 64 tokens (the same place for any M)
    s1 = (2 * 512 // 128) * 1 * 4 * 2048  # shared gate_up: 4 k splits of 2Is / 128 tiles x token groups x 128 x 16
    assert pb == cnt + s1 + units * 2 * 2048 and sh == 10 * (512 + 2048) * 2
    assert lib.qf_a16_moe_workspace(32, 2048, 512, 10, 512, *[ctypes.byref(a) for a in v]) == 0
    units = 32 * 10 * (2 * 512 // 128)   # two token groups
    assert v[4].value == cnt + (2 * 512 // 128) * 2 * 4 * 2048 + units * 2 * 2048
