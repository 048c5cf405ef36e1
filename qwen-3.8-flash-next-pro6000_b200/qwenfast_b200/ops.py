"""Torch-facing ops with the reference extension's names and argument roles (serve/qwenfast/qf_bind.cpp).

Each op validates like the reference's TORCH_CHECKs (raising RuntimeError), allocates its outputs like the
reference (``at::empty``), and enqueues the sm_100a kernel on the current CUDA stream through the C ABI. There is no
CPU path: CPU tensors are rejected.
"""
import ctypes
import weakref
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib
from .formats import repack_bf16, repack_w4

BF16 = torch.bfloat16
DBG_NUMEL = 32 * 512          # QF_MOE_DBG_NUMEL: entries of the optional MoE timeline buffer


def _req(cond: bool, msg: str):
    if not cond:
        raise RuntimeError(msg)


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None or t.numel() == 0 else t.data_ptr()


def _present(t: Optional[torch.Tensor]) -> bool:
    return t is not None and t.numel() > 0


def _stream(dev: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _cuda(t: torch.Tensor, name: str, op: str):
    _req(t.is_cuda, f"{op}: {name} must be a CUDA tensor")


# ------------------------------------------------------------------------------------------------- router
def router_topk(x: torch.Tensor, w: torch.Tensor, topk: int, renormalize: bool, scratch: torch.Tensor,
                counter: torch.Tensor, pdl: bool = True):
    """(topk_weights fp32 [rows, k], topk_ids int32 [rows, k], router_logits bf16 [rows, E]).

    Mirrors ``router_topk`` (serve/qwenfast/qf_router.cu:164-193): scratch fp32 >= rows * E, counter int32 [1]
    zeroed once and re-armed by the kernel. rows 1..64."""
    op = "router_topk"
    _cuda(x, "x", op)
    _req(x.dtype == BF16 and x.dim() == 2 and x.is_contiguous(), f"{op}: x must be contiguous bf16 [rows, H]")
    _req(w.dtype == BF16 and w.dim() == 2 and w.size(1) == x.size(1) and w.is_contiguous() and w.device == x.device,
         f"{op}: w must be contiguous bf16 [E, H] on x's device")
    _req(scratch.dtype == torch.float32 and scratch.device == x.device, f"{op}: scratch must be fp32 on x's device")
    _req(counter.dtype == torch.int32 and counter.numel() >= 1 and counter.device == x.device,
         f"{op}: counter must be int32 [>=1] on x's device")
    rows, H = x.shape
    E = w.shape[0]
    weights = torch.empty(rows, topk, dtype=torch.float32, device=x.device)
    ids = torch.empty(rows, topk, dtype=torch.int32, device=x.device)
    logits = torch.empty(rows, E, dtype=BF16, device=x.device)
    with torch.cuda.device(x.device):
        _lib.check(_lib.load().qf_router_topk(
            x.data_ptr(), w.data_ptr(), rows, H, E, int(topk), int(bool(renormalize)), weights.data_ptr(),
            ids.data_ptr(), logits.data_ptr(), scratch.data_ptr(), scratch.numel(), counter.data_ptr(), int(bool(pdl)),
            _stream(x.device)), op)
    return weights, ids, logits


def router_bufs(device, rows: int = 64, experts: int = 1024):
    """Caller-owned router scratch (reference qwenfast.py:1032-1038): fp32 [rows * experts], counter int32 [1]."""
    return (torch.empty(rows * experts, dtype=torch.float32, device=device),
            torch.zeros(1, dtype=torch.int32, device=device))


# ------------------------------------------------------------------------------------------------- MoE
_W8_SHARED = {}


def tensor_cache(cache: dict, tensors, build):
    """``build()`` once per set of live tensors: the entry is found again while every tensor of the set is alive (the
    same objects, not just the same addresses) and is dropped when the first of them is freed, so a cache of
    converted weights does not outlive the weights it was made from."""
    key = tuple((t.data_ptr(), tuple(t.shape), t.dtype) for t in tensors)
    hit = cache.get(key)
    if hit is not None and all(r() is t for r, t in zip(hit[0], tensors)):
        return hit[1]
    val = build()
    cache[key] = (tuple(weakref.ref(t) for t in tensors), val)
    weakref.finalize(tensors[0], cache.pop, key, None)
    return val


def shared_w8_as_bf16(sq1, ss1, sq2, ss2, H: int, op: str = "a16_moe_decode"):
    """The shared expert given as the reference passes it to its MoE op (qwenfast.py:1092-1113, 1196-1200): INT8
    gate_up sq1 [2Is, H] and down sq2 [H, Is] with bf16 group scales ss1 / ss2 (``w8_quant`` format, group 128 or
    64) -> the kernel-layout bf16 weights the MoE kernel streams, ``bf16(q * s)`` dequantised on the device
    (``w8g_unpack``) and repacked. Done once per weight tensor: the result is cached for as long as ``sq1`` lives, so
    only the first call allocates (make it before any graph capture). The weights are then rounded to bf16 (relative
    2^-9 per weight) where the reference's w8g arithmetic applies the scale to fp32 group sums -- within the layer's
    tolerance (tested against that arithmetic). The converted copy is dropped when ``sq1`` is freed."""
    for name, q, sc in (("shq1 / shs1", sq1, ss1), ("shq2 / shs2", sq2, ss2)):
        _req(q is not None and sc is not None and q.dtype == torch.int8 and q.dim() == 2 and q.is_contiguous()
             and sc.dtype == BF16 and sc.dim() == 2 and sc.is_contiguous() and sc.size(0) == q.size(0)
             and q.size(1) % sc.size(1) == 0 and q.size(1) // sc.size(1) in (64, 128) and q.is_cuda and sc.is_cuda,
             f"{op}: INT8 shared-expert weights {name} must be int8 [N, K] with bf16 group scales [N, K/128]")
    Is = sq2.size(1)
    _req(tuple(sq1.shape) == (2 * Is, H) and tuple(sq2.shape) == (H, Is),
         f"{op}: INT8 shared-expert weights must be gate_up [2Is, H] and down [H, Is]")

    def build():
        w1 = torch.empty(2 * Is, H, dtype=BF16, device=sq1.device)
        w2 = torch.empty(H, Is, dtype=BF16, device=sq1.device)
        w8g_unpack(sq1, ss1, w1)
        w8g_unpack(sq2, ss2, w2)
        return repack_bf16(w1, gated=True), repack_bf16(w2, gated=False)

    return tensor_cache(_W8_SHARED, (sq1, ss1, sq2, ss2), build)


# control block -> (its pinned host mirror of the sticky error word, the pbuf it is used with): see moe_workspace
_MOE_MIRRORS = {}


def moe_workspace(M: int, H: int, I: int, topk: int, Is: int, device) -> dict:
    """Caller-owned scratch for ``a16_moe_decode`` (the reference's ``_a16_bufs``, qwenfast.py:1044-1059).

    The control block gets a host mirror of its sticky error word (``err_host``, pinned host memory whose address
    sits in ctrl words QF_MOE_CTRL_MIRROR..+1): every launch that ends with an error copies the word there, and the
    ops read it before their next launch on this workspace without synchronising (``check_moe_error``)."""
    lib = _lib.load()
    v = [ctypes.c_int64() for _ in range(6)]
    _lib.check(lib.qf_a16_moe_workspace(M, H, I, topk, Is, *[ctypes.byref(a) for a in v]), "moe_workspace")
    hb, yb, gl, ctrl, pb, sh = (a.value for a in v)
    bufs = dict(
        hbuf=torch.empty(hb // 2, dtype=BF16, device=device),
        ybuf=torch.empty(yb // 2, dtype=BF16, device=device),
        gl=torch.empty(gl, dtype=torch.float32, device=device),
        ctrl=torch.zeros(ctrl, dtype=torch.int32, device=device),
        pbuf=torch.zeros(max(pb, 1), dtype=torch.float32, device=device),   # holds counters: zeroed once
        shbuf=torch.empty(max(sh // 2, 1), dtype=BF16, device=device),
        none=torch.empty(0, dtype=BF16, device=device),
        none_i64=torch.empty(0, dtype=torch.int64, device=device),   # an absent timeline buffer (operators' dbg)
        err_host=torch.zeros(1, dtype=torch.int32, pin_memory=True),
    )
    attach_error_mirror(bufs["ctrl"], bufs["err_host"], bufs["pbuf"])
    return bufs


def attach_error_mirror(ctrl: torch.Tensor, err_host: torch.Tensor, pbuf: torch.Tensor):
    """Point the control block's mirror words at ``err_host`` (pinned int32 [1]; under unified addressing its host
    address is also its device address) and remember the pair, so that the ops check it before each launch."""
    _req(err_host.dtype == torch.int32 and err_host.is_pinned() and err_host.numel() >= 1,
         "attach_error_mirror: err_host must be a pinned int32 host tensor")
    _req(ctrl.dtype == torch.int32 and ctrl.numel() >= _lib.QF_MOE_CTRL_WORDS and ctrl.is_contiguous(),
         "attach_error_mirror: ctrl must be a contiguous int32 control block")
    ctrl.view(torch.int64)[_lib.QF_MOE_CTRL_MIRROR // 2] = err_host.data_ptr()
    key = ctrl.data_ptr()
    _MOE_MIRRORS[key] = (weakref.ref(ctrl), err_host, pbuf)
    weakref.finalize(ctrl, _MOE_MIRRORS.pop, key, None)


def check_moe_error(ctrl: torch.Tensor):
    """Raise RuntimeError when an earlier launch on this control block reported an error through its host mirror (a
    plain read of pinned host memory: no synchronisation). Before raising, the workspace is made usable again on the
    current stream: the control block (except its mirror words) and pbuf are zeroed, as a hard error requires."""
    ent = _MOE_MIRRORS.get(ctrl.data_ptr())
    if ent is None or ent[0]() is not ctrl:
        return
    err = int(ent[1][0])
    if err == 0:
        return
    ctrl[: _lib.QF_MOE_CTRL_MIRROR].zero_()
    ent[2].zero_()
    ent[1].zero_()
    names = [n for b, n in ((_lib.QF_MOE_ERR_TIMEOUT, "a bounded wait ran out"),
                            (_lib.QF_MOE_ERR_BAD_EXPERT, "a routed expert id was out of range"),
                            (_lib.QF_MOE_ERR_PIPELINE, "a pipeline wait ran out")) if err & b]
    raise RuntimeError(f"a16_moe_decode: an earlier launch on this workspace reported error {err:#x} "
                       f"({'; '.join(names)}); its outputs were undefined, the workspace has been reset")


def a16_moe_decode(x, topk_ids, topk_w, w13, s13, gs13, w2, s2, gs2, w_gate, shared, hbuf, ybuf, gl, ctrl, out,
                   phase: int = 4, dbg=None, pbuf=None, shq1=None, shs1=None, shq2=None, shs2=None, shbuf=None,
                   pdl: bool = True, mode: int = 0, expert_range=None, num_experts: Optional[int] = None,
                   router_w: Optional[torch.Tensor] = None, renormalize: bool = True,
                   logits: Optional[torch.Tensor] = None, x_stage: Optional[torch.Tensor] = None,
                   fmt: str = "int4"):
    """Routed experts + shared expert + combine; writes ``out`` in place and returns it.

    Argument roles follow ``a16_moe_decode`` (serve/qwenfast/qf_a16moe.cu:852-863). Weight format: the kernel
    layout of ``repack_w4`` -- w13 int32 [E, 2I*H/8], s13 bf16 [E, 2I*H/128], w2 int32 [E, H*I/8],
    s2 bf16 [E, H*I/128]; gs13 / gs2 bf16 [E] or empty (= 1). The in-kernel shared expert takes bf16 weights in the
    kernel layout of ``repack_bf16``: shq1 = gate_up [2Is*H], shq2 = down [H*Is], shs1 / shs2 empty -- or, as the
    reference passes it, INT8 weights shq1 [2Is, H] / shq2 [H, Is] with bf16 group scales shs1 / shs2 (converted
    once, see ``shared_w8_as_bf16``). ``shared`` is a precomputed bf16 [M, H] shared output instead (or empty).
    Empty tensors mean "absent", as in the reference.

    ``mode=1`` is one expert-parallel shard: the weights hold only experts ``expert_range = (lo, hi)`` of
    ``num_experts`` (the router's expert count), and instead of ``out`` the kernel leaves the shard's exact slot
    contribution in ``ybuf`` (``[M*topk + M, H]``: routed slots, then the shared rows); the shards' ``ybuf`` summed
    and passed to ``moe_combine`` give the mode-0 output bit for bit.

    With ``router_w`` (bf16 [E, H]) the router runs inside the same launch (C ABI ``qf_moe_layer_decode``):
    ``topk_ids`` / ``topk_w`` and ``logits`` (bf16 [M, E]) are then outputs, written by the kernel. With it,
    ``x_stage`` (CUDA bf16 [M, H]) means ``x`` is a pinned host tensor that the kernel copies into ``x_stage`` itself,
    and ``out`` may be a pinned host tensor as well (written by the kernel).

    ``fmt="nvfp4"``: the experts are NVFP4 (the reference's own format) in the layout of ``formats.repack_nvfp4`` --
    w13 / w2 the e2m1 codes (int32, int4 kernel layout), s13 / s2 the E4M3 group-16 scales (uint8 [E, N*K/16]),
    gs13 / gs2 the per-expert multipliers 1 / g (C ABI ``qf_a16_moe_decode_nvfp4``, with ``router_w``
    ``qf_moe_layer_decode_nvfp4``)."""
    op = "a16_moe_decode" if router_w is None else "moe_layer_decode"
    check_moe_error(ctrl)
    if x_stage is None:
        _cuda(x, "x", op)
        dev = x.device
    else:
        _req(router_w is not None, f"{op}: x_stage needs the fused router (router_w)")
        _req(not x.is_cuda and x.is_pinned(), f"{op}: with x_stage, x must be a pinned host tensor")
        _cuda(x_stage, "x_stage", op)
        _req(x_stage.dtype == BF16 and x_stage.is_contiguous() and x_stage.shape == x.shape,
             f"{op}: x_stage must be contiguous bf16 shaped like x")
        dev = x_stage.device
    host_out = not out.is_cuda
    _req(not host_out or (x_stage is not None and out.is_pinned()),
         f"{op}: out must be a CUDA tensor (or a pinned host tensor, with x_stage)")
    M, H = x.shape
    _req(x.dtype == BF16 and x.dim() == 2 and x.is_contiguous(), f"{op}: x must be contiguous bf16 [M, H]")
    _req(topk_ids.dtype == torch.int32 and topk_ids.dim() == 2 and topk_ids.size(0) == M and topk_ids.is_contiguous(),
         f"{op}: topk_ids must be contiguous int32 [M, topk]")
    _req(topk_w.dtype == torch.float32 and tuple(topk_w.shape) == tuple(topk_ids.shape) and topk_w.is_contiguous(),
         f"{op}: topk_w must be contiguous fp32 [M, topk]")
    _req(w13.dtype == torch.int32 and w2.dtype == torch.int32 and w13.dim() == 2 and w2.dim() == 2,
         f"{op}: w13 / w2 must be int32 kernel-layout [E, *] tensors (see repack_w4)")
    E = w13.shape[0]          # experts held in w13 / w2 (the shard's, in mode 1)
    I = (w2.shape[1] * 8) // H
    _req(w2.shape[0] == E and w13.shape[1] == 2 * I * H // 8 and w2.shape[1] * 8 == H * I,
         f"{op}: w13 / w2 shapes do not match H={H}")
    _req(fmt in ("int4", "nvfp4"), f"{op}: fmt must be 'int4' or 'nvfp4'")
    if fmt == "nvfp4":
        _req(s13.dtype == torch.uint8 and tuple(s13.shape) == (E, 2 * I * H // 16) and s13.is_contiguous(),
             f"{op}: NVFP4 s13 must be the E4M3 scales uint8 [E, 2I*H/16] (formats.repack_nvfp4)")
        _req(s2.dtype == torch.uint8 and tuple(s2.shape) == (E, H * I // 16) and s2.is_contiguous(),
             f"{op}: NVFP4 s2 must be the E4M3 scales uint8 [E, H*I/16] (formats.repack_nvfp4)")
    else:
        _req(s13.dtype == BF16 and tuple(s13.shape) == (E, 2 * I * H // 128), f"{op}: s13 must be bf16 [E, 2I*H/128]")
        _req(s2.dtype == BF16 and tuple(s2.shape) == (E, H * I // 128), f"{op}: s2 must be bf16 [E, H*I/128]")
    for name, g in (("gs13", gs13), ("gs2", gs2)):
        _req(not _present(g) or (g.dtype == BF16 and g.numel() == E), f"{op}: {name} must be bf16 [E] or empty")
    if _present(shs1) or _present(shs2):
        # the reference's in-kernel shared expert: group-scaled INT8 weights (w8_quant format)
        shq1, shq2 = shared_w8_as_bf16(shq1, shs1, shq2, shs2, H, op)
        shs1 = shs2 = None
    has_shw = _present(shq1)
    Is = 0
    if has_shw:
        _req(_present(shq2) and shq1.dtype == BF16 and shq2.dtype == BF16, f"{op}: shq1 / shq2 must be bf16")
        Is = shq2.numel() // H
        _req(shq1.numel() == 2 * Is * H and shq2.numel() == H * Is, f"{op}: shared-expert weight sizes do not match")
    if _present(shared):
        _req(shared.dtype == BF16 and shared.is_contiguous() and tuple(shared.shape) == (M, H),
             f"{op}: shared must be contiguous bf16 [M, H]")
    _req(out.dtype == BF16 and tuple(out.shape) == (M, H) and out.is_contiguous(), f"{op}: out must be bf16 [M, H]")
    _req(dbg is None or (dbg.is_cuda and dbg.dtype == torch.int64 and dbg.is_contiguous() and dbg.numel() >= DBG_NUMEL),
         f"{op}: dbg must be a contiguous int64 CUDA tensor of at least {DBG_NUMEL} entries")
    E_all = E if num_experts is None else int(num_experts)
    lo, hi = (0, E_all) if expert_range is None else (int(expert_range[0]), int(expert_range[1]))
    _req(mode in (0, 1, 2), f"{op}: mode must be 0, 1 or 2")
    _req(mode == 0 or hi - lo == E, f"{op}: mode 1 takes the weights of experts [lo, hi) only ({hi - lo} != {E})")
    _req(mode == 1 or E == E_all, f"{op}: mode 0 takes every expert's weights")
    tensors = [topk_ids, topk_w, w13, s13, w2, s2, hbuf, ybuf, gl, ctrl] + ([] if host_out else [out])
    _req(all(t.device == dev for t in tensors), f"{op}: every tensor must be on x's device")
    if router_w is not None:
        _req(router_w.dtype == BF16 and router_w.is_contiguous() and tuple(router_w.shape) == (E_all, H)
             and router_w.device == dev, f"{op}: router_w must be contiguous bf16 [E, H] on x's device")
        _req(logits is not None and logits.dtype == BF16 and logits.is_contiguous()
             and tuple(logits.shape) == (M, E_all) and logits.device == dev,
             f"{op}: logits must be a contiguous bf16 [M, E] tensor on x's device")
        _req(int(phase) in (3, 4), f"{op}: phase must be 3 or 4")
        with torch.cuda.device(dev):
            layer_entry = _lib.load().qf_moe_layer_decode_nvfp4 if fmt == "nvfp4" else _lib.load().qf_moe_layer_decode
            _lib.check(layer_entry(
                x.data_ptr(), _ptr(x_stage), router_w.data_ptr(), int(bool(renormalize)), topk_w.data_ptr(),
                topk_ids.data_ptr(),
                logits.data_ptr(), w13.data_ptr(), s13.data_ptr(), _ptr(gs13), w2.data_ptr(), s2.data_ptr(),
                _ptr(gs2), _ptr(w_gate), _ptr(shared), _ptr(shq1) if has_shw else None,
                _ptr(shq2) if has_shw else None,
                hbuf.data_ptr(), hbuf.numel() * hbuf.element_size(), ybuf.data_ptr(),
                ybuf.numel() * ybuf.element_size(), gl.data_ptr(), gl.numel(), ctrl.data_ptr(), ctrl.numel(),
                _ptr(pbuf), 0 if pbuf is None else pbuf.numel(),
                _ptr(shbuf), 0 if shbuf is None else shbuf.numel() * shbuf.element_size(),
                out.data_ptr(), M, H, I, E_all, topk_ids.shape[1], Is, int(mode), int(lo), int(hi),
                _ptr(dbg), int(bool(pdl)), _stream(dev)), op)
        return out
    entry = _lib.load().qf_a16_moe_decode_nvfp4 if fmt == "nvfp4" else _lib.load().qf_a16_moe_decode
    with torch.cuda.device(x.device):
        _lib.check(entry(
            x.data_ptr(), topk_ids.data_ptr(), topk_w.data_ptr(), w13.data_ptr(), s13.data_ptr(), _ptr(gs13),
            w2.data_ptr(), s2.data_ptr(), _ptr(gs2), _ptr(w_gate), _ptr(shared), _ptr(shq1) if has_shw else None,
            _ptr(shq2) if has_shw else None,
            hbuf.data_ptr(), hbuf.numel() * hbuf.element_size(), ybuf.data_ptr(), ybuf.numel() * ybuf.element_size(),
            gl.data_ptr(), gl.numel(), ctrl.data_ptr(), ctrl.numel(),
            _ptr(pbuf), 0 if pbuf is None else pbuf.numel(),
            _ptr(shbuf), 0 if shbuf is None else shbuf.numel() * shbuf.element_size(),
            out.data_ptr(), M, H, I, E_all, topk_ids.shape[1], Is, int(phase), int(mode), int(lo), int(hi),
            _ptr(dbg), int(bool(pdl)), _stream(x.device)), op)
    return out


def moe_combine(ybuf: torch.Tensor, x: torch.Tensor, w_gate: Optional[torch.Tensor], has_shared: bool,
                out: torch.Tensor, topk: int, pdl: bool = True) -> torch.Tensor:
    """Expert-parallel finish: ``out`` = the layer output from the shards' summed slot buffers (``ybuf`` as left by
    mode-1 ``a16_moe_decode``, summed over the shards). The gate logit is recomputed from ``x`` and ``w_gate``."""
    op = "moe_combine"
    _cuda(x, "x", op)
    M, H = x.shape
    _req(x.dtype == BF16 and x.is_contiguous() and ybuf.dtype == BF16 and ybuf.is_contiguous(), f"{op}: bf16 tensors")
    _req(ybuf.numel() >= M * (topk + 1) * H, f"{op}: ybuf must hold [M*topk + M, H]")
    _req(out.dtype == BF16 and tuple(out.shape) == (M, H) and out.is_contiguous(), f"{op}: out must be bf16 [M, H]")
    _req(not has_shared or (w_gate is not None and w_gate.numel() == H), f"{op}: a shared term needs w_gate [H]")
    with torch.cuda.device(x.device):
        _lib.check(_lib.load().qf_moe_combine(ybuf.data_ptr(), x.data_ptr(), _ptr(w_gate) if has_shared else None,
                                              int(bool(has_shared)), out.data_ptr(), M, H, int(topk), int(bool(pdl)),
                                              _stream(x.device)), op)
    return out


def moe_error_word(ctrl: torch.Tensor) -> int:
    """The sticky error word of a MoE control block (reads the device; synchronises)."""
    return int(ctrl[_lib.QF_MOE_CTRL_ERR].item())


def clear_moe_error(ctrl: torch.Tensor, pbuf: Optional[torch.Tensor] = None):
    """Zero the sticky error word (and, after a hard error, pbuf) and the host mirror of this control block."""
    ctrl[_lib.QF_MOE_CTRL_ERR] = 0
    if pbuf is not None:
        pbuf.zero_()
    ent = _MOE_MIRRORS.get(ctrl.data_ptr())
    if ent is not None and ent[0]() is ctrl:
        torch.cuda.synchronize(ctrl.device)
        ent[1].zero_()


@dataclass
class MoELayerWeights:
    """One MoE layer in kernel layout (routed experts + optional bf16 shared expert + router)."""
    router: torch.Tensor            # bf16 [E, H]
    w13: torch.Tensor               # int32 [E, 2I*H/8]
    s13: torch.Tensor               # bf16 [E, 2I*H/128]
    w2: torch.Tensor                # int32 [E, H*I/8]
    s2: torch.Tensor                # bf16 [E, H*I/128]
    w_gate: Optional[torch.Tensor]  # bf16 [H]
    sh_w13: Optional[torch.Tensor]  # bf16 [2Is*H] kernel layout
    sh_w2: Optional[torch.Tensor]   # bf16 [H*Is] kernel layout
    H: int
    I: int
    E: int
    Is: int

    @staticmethod
    def from_canonical(router, w13, s13, w2, s2, w_gate=None, sh_gu=None, sh_d=None) -> "MoELayerWeights":
        """Repack canonical tensors (see formats.py) on their CUDA device."""
        E, N13, _ = w13.shape
        H = router.shape[1]
        I = N13 // 2
        wk13, sk13 = repack_w4(w13, s13, gated=True)
        wk2, sk2 = repack_w4(w2, s2, gated=False)
        shw13 = repack_bf16(sh_gu, gated=True) if sh_gu is not None else None
        shw2 = repack_bf16(sh_d, gated=False) if sh_d is not None else None
        Is = sh_d.shape[1] if sh_d is not None else 0
        return MoELayerWeights(router.contiguous(), wk13, sk13, wk2, sk2,
                               None if w_gate is None else w_gate.contiguous(), shw13, shw2, H, I, E, Is)


def moe_layer_step(x: torch.Tensor, lw: MoELayerWeights, topk: int, bufs: dict, rbufs, out: torch.Tensor,
                   renormalize: bool = True, pdl: bool = True, fused: bool = True,
                   x_stage: Optional[torch.Tensor] = None):
    """One decode MoE layer-step: the reference's ``dual`` fast path (qwenfast.py:1177-1201: router_topk, then
    a16_moe_decode with the shared expert computed in-kernel). ``fused`` (default) runs the router inside the MoE
    launch (``qf_moe_layer_decode``, a cooperative launch); if that grid cannot be co-resident on this device the
    launch is declined and the step takes the two launches of ``fused=False``: ``router_topk`` (scratch ``rbufs``),
    then ``a16_moe_decode``. Host I/O: ``x`` and ``out`` pinned host tensors and ``x_stage`` a CUDA bf16 [M, H]
    buffer -- the fused kernel reads x from host memory and writes out there (the two-launch path copies through
    ``x_stage`` and a device buffer instead). Returns (out, topk_w, topk_ids, logits)."""
    M = x.shape[0]
    dev = x.device if x_stage is None else x_stage.device
    if fused:
        tw = torch.empty(M, topk, dtype=torch.float32, device=dev)
        ids = torch.empty(M, topk, dtype=torch.int32, device=dev)
        logits = torch.empty(M, lw.E, dtype=BF16, device=dev)
        try:
            a16_moe_decode(x, ids, tw, lw.w13, lw.s13, None, lw.w2, lw.s2, None, lw.w_gate, None, bufs["hbuf"],
                           bufs["ybuf"], bufs["gl"], bufs["ctrl"], out, 4, None, bufs["pbuf"], lw.sh_w13, None,
                           lw.sh_w2, None, bufs["shbuf"], pdl=pdl, router_w=lw.router, renormalize=renormalize,
                           logits=logits, x_stage=x_stage)
            return out, tw, ids, logits
        except _lib.Unsupported:
            pass   # the fused grid cannot be co-resident here: the reference's two launches instead
    xd = x
    if not x.is_cuda:
        _req(x_stage is not None, "moe_layer_step: a host x needs x_stage")
        x_stage.copy_(x, non_blocking=True)
        xd = x_stage
    od = out if out.is_cuda else torch.empty(M, x.shape[1], dtype=BF16, device=dev)
    tw, ids, logits = router_topk(xd, lw.router, topk, renormalize, rbufs[0], rbufs[1], pdl)
    a16_moe_decode(xd, ids, tw, lw.w13, lw.s13, None, lw.w2, lw.s2, None, lw.w_gate, None, bufs["hbuf"],
                   bufs["ybuf"], bufs["gl"], bufs["ctrl"], od, 4, None, bufs["pbuf"], lw.sh_w13, None, lw.sh_w2,
                   None, bufs["shbuf"], pdl=pdl)
    if od is not out:
        out.copy_(od, non_blocking=True)
    return out, tw, ids, logits


class LayerStep:
    """``moe_layer_step`` (fused router, int4 experts) prepared for one layer's weights and one workspace.

    Every check of the weights and the workspace (types, shapes, devices) runs once, here, and the C-ABI argument list
    is built once; a call checks x and out only, reads the workspace's host error mirror and makes one
    ``qf_moe_layer_decode`` call (the C ABI still checks sizes, alignment and M on every call). The routing outputs
    (topk_w fp32 [M, topk], topk_ids int32 [M, topk], logits bf16 [M, E]) are views of buffers this object holds, so
    they are valid until its next call. Where the fused grid cannot be co-resident (``_lib.Unsupported``), a call
    takes ``moe_layer_step``'s two launches instead, with router scratch made on first use."""

    def __init__(self, lw: MoELayerWeights, topk: int, bufs: dict, renormalize: bool = True, pdl: bool = True):
        op = "LayerStep"
        dev = lw.w13.device
        _req(dev.type == "cuda", f"{op}: the weights must be CUDA tensors")
        H, I, E, Is = lw.H, lw.I, lw.E, lw.Is
        _req(1 <= topk <= _lib.QF_MAX_TOPK and topk <= E, f"{op}: topk must be in [1, min(E, {_lib.QF_MAX_TOPK})]")

        def tensor(t, name, dtype, numel):
            _req(t is not None and t.dtype == dtype and t.is_contiguous() and t.numel() == numel and t.device == dev,
                 f"{op}: {name} must be a contiguous {dtype} tensor of {numel} elements on the weights' device")

        tensor(lw.router, "router", BF16, E * H)
        tensor(lw.w13, "w13", torch.int32, E * 2 * I * H // 8)
        tensor(lw.s13, "s13", BF16, E * 2 * I * H // 128)
        tensor(lw.w2, "w2", torch.int32, E * H * I // 8)
        tensor(lw.s2, "s2", BF16, E * H * I // 128)
        has_shw = lw.sh_w13 is not None
        _req(has_shw == (lw.sh_w2 is not None) and has_shw == (Is > 0), f"{op}: give both shared-expert weights, or none")
        if has_shw:
            tensor(lw.sh_w13, "sh_w13", BF16, 2 * Is * H)
            tensor(lw.sh_w2, "sh_w2", BF16, H * Is)
        if lw.w_gate is not None:
            tensor(lw.w_gate, "w_gate", BF16, H)
        for name in ("hbuf", "ybuf", "gl", "ctrl", "pbuf", "shbuf"):
            t = bufs.get(name)
            _req(t is not None and t.device == dev and t.is_contiguous(), f"{op}: workspace {name} missing or misplaced")
        self.lw, self.topk, self.bufs, self.renormalize, self.pdl, self.dev = lw, topk, bufs, renormalize, pdl, dev
        cap = _lib.QF_MAX_TOKENS
        self._tw = torch.empty(cap, topk, dtype=torch.float32, device=dev)
        self._ids = torch.empty(cap, topk, dtype=torch.int32, device=dev)
        self._logits = torch.empty(cap, E, dtype=BF16, device=dev)
        self._err = bufs["err_host"].numpy() if "err_host" in bufs else None
        self._rbufs = None
        b = bufs
        nbytes = lambda t: t.numel() * t.element_size()   # noqa: E731
        # qf_moe_layer_decode's arguments: (x, x_stage) + head + (out, M) + tail + (stream,)
        self._head = (lw.router.data_ptr(), int(bool(renormalize)), self._tw.data_ptr(), self._ids.data_ptr(),
                      self._logits.data_ptr(), lw.w13.data_ptr(), lw.s13.data_ptr(), None, lw.w2.data_ptr(),
                      lw.s2.data_ptr(), None, _ptr(lw.w_gate), None, _ptr(lw.sh_w13) if has_shw else None,
                      _ptr(lw.sh_w2) if has_shw else None, b["hbuf"].data_ptr(), nbytes(b["hbuf"]),
                      b["ybuf"].data_ptr(), nbytes(b["ybuf"]), b["gl"].data_ptr(), b["gl"].numel(),
                      b["ctrl"].data_ptr(), b["ctrl"].numel(), b["pbuf"].data_ptr(), b["pbuf"].numel(),
                      b["shbuf"].data_ptr(), nbytes(b["shbuf"]))
        self._tail = (H, I, E, topk, Is, 0, 0, E, None, int(bool(pdl)))
        self._fn = _lib.load().qf_moe_layer_decode
        self._fused = True
        self._views = {}   # M -> the routing outputs' views

    def __call__(self, x: torch.Tensor, out: torch.Tensor, x_stage: Optional[torch.Tensor] = None):
        """One layer-step on x (bf16 [M, H]: a CUDA tensor, or a pinned host tensor with ``x_stage`` a CUDA bf16
        [M, H] buffer) into out (bf16 [M, H]: CUDA, or pinned host memory with ``x_stage``). Returns
        (out, topk_w, topk_ids, logits)."""
        op = "LayerStep"
        if self._err is not None and self._err[0] != 0:
            check_moe_error(self.bufs["ctrl"])          # raises, after resetting the workspace
        M = x.shape[0]
        _req(x.dtype == BF16 and x.dim() == 2 and x.shape[1] == self.lw.H and x.is_contiguous(),
             f"{op}: x must be contiguous bf16 [M, H]")
        _req(out.dtype == BF16 and out.shape == x.shape and out.is_contiguous(), f"{op}: out must be bf16 [M, H]")
        if x_stage is None:
            _req(x.device == self.dev and out.device == self.dev, f"{op}: x and out must be on the weights' device")
            xs = None
        else:
            _req(not x.is_cuda and x.is_pinned(), f"{op}: with x_stage, x must be a pinned host tensor")
            _req(x_stage.device == self.dev and x_stage.dtype == BF16 and x_stage.shape == x.shape
                 and x_stage.is_contiguous(), f"{op}: x_stage must be contiguous bf16 [M, H] on the weights' device")
            _req(out.device == self.dev or (not out.is_cuda and out.is_pinned()),
                 f"{op}: out must be on the weights' device or in pinned host memory")
            xs = x_stage.data_ptr()
        if self._fused:
            try:
                if torch.cuda.current_device() == self.dev.index:
                    st = self._fn(x.data_ptr(), xs, *self._head, out.data_ptr(), M, *self._tail,
                                  torch.cuda.current_stream().cuda_stream)
                else:
                    with torch.cuda.device(self.dev):
                        st = self._fn(x.data_ptr(), xs, *self._head, out.data_ptr(), M, *self._tail,
                                      torch.cuda.current_stream().cuda_stream)
                _lib.check(st, "moe_layer_decode")
                v = self._views.get(M)
                if v is None:
                    v = self._views[M] = (self._tw[:M], self._ids[:M], self._logits[:M])
                return (out,) + v
            except _lib.Unsupported:
                self._fused = False
        if self._rbufs is None:
            self._rbufs = router_bufs(self.dev, _lib.QF_MAX_TOKENS, self.lw.E)
        return moe_layer_step(x, self.lw, self.topk, self.bufs, self._rbufs, out, self.renormalize, self.pdl,
                              fused=False, x_stage=x_stage)


# ------------------------------------------------------------------------------------------------- INT8
_W8G_FIXUP = {}


def w8g_fixup(N: int, device, stream=None) -> torch.Tensor:
    """The W8A16 GEMM's fixup buffer (split-tile partial sums and zero-kept counters) for an N-row weight, one per
    (device, stream, N); the first call allocates (make it before any CUDA-graph capture)."""
    dev = torch.device(device)
    st = (stream or torch.cuda.current_stream(dev)).cuda_stream
    key = (dev.index, st, N)
    buf = _W8G_FIXUP.get(key)
    if buf is None:
        n = ctypes.c_int64(0)
        with torch.cuda.device(dev):
            _lib.check(_lib.load().qf_w8g_fixup_elems(N, ctypes.byref(n)), "w8g_fixup_elems")
        buf = _W8G_FIXUP[key] = torch.zeros(n.value, dtype=torch.float32, device=dev)
    return buf


def w8g_gemm(x: torch.Tensor, q: torch.Tensor, s: torch.Tensor, rpw: int = 0, pdl: bool = False,
             fixup: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = x @ (q * s)^T (W8A16, group-scaled int8) on the tensor cores. Mirrors ``w8g_gemm``
    (serve/qwenfast/qf_w8g.cu:303-336): x bf16 [M, K] (unit column stride, row stride % 8 == 0), q int8 [N, K] as
    stored (canonical), s bf16 [N, K/group], group 128 or 64; returns y bf16 [M, N]. ``rpw``: the reference's path bits
    (qf_w8g.cu:315-318): 0x100 forces the tensor-memory kernel, 0x200 forbids it (RuntimeError when the
    register-fragment kernel does not take the shape); the low byte (rows per warp) is ignored. ``fixup``: the split-tile buffer (``w8g_fixup``; the
    current stream's by default)."""
    op = "w8g_gemm"
    _cuda(x, "x", op)
    _req(q.is_cuda and s.is_cuda and x.dtype == BF16, f"{op}: x bf16, q, s on CUDA")
    _req(q.dtype == torch.int8 and s.dtype == BF16, f"{op}: q int8, s bf16")
    _req(x.dim() == 2 and q.dim() == 2 and x.size(1) == q.size(1) and q.is_contiguous() and s.is_contiguous(),
         f"{op}: shapes")
    _req(s.dim() == 2 and s.size(0) == q.size(0) and q.size(1) % s.size(1) == 0, f"{op}: scale shape")
    _req(x.stride(1) == 1 and x.stride(0) % 8 == 0 and x.data_ptr() % 16 == 0, f"{op}: x layout")
    M, K = x.shape
    N = q.shape[0]
    group = K // s.shape[1]
    if fixup is None:
        fixup = w8g_fixup(N, x.device)
    y = torch.empty(M, N, dtype=BF16, device=x.device)
    with torch.cuda.device(x.device):
        _lib.check(_lib.load().qf_w8g_gemm(x.data_ptr(), x.stride(0), q.data_ptr(), s.data_ptr(), y.data_ptr(), N, M,
                                           N, K, group, int(rpw), fixup.data_ptr(), fixup.numel(), int(bool(pdl)),
                                           _stream(x.device)), op)
    return y


def w8g_take_status() -> int:
    """Sticky wait-timeout bits of the W8A16 kernel since the last call (0 = clean); clears them. After a non-zero
    status the fixup buffers may hold partial counts, so the cached ones are zeroed again."""
    v = ctypes.c_uint32(0)
    _lib.check(_lib.load().qf_w8g_take_status(ctypes.byref(v)), "w8g_take_status")
    if v.value:
        for buf in _W8G_FIXUP.values():
            buf.zero_()
    return v.value


class W8Linear:
    """``w8g_gemm`` prepared for one weight (q int8 [N, K], s bf16 [N, K/group]): the weight's checks, its group size
    and its C-ABI arguments are made once; a call checks x, allocates y (or writes ``out``) and makes one
    ``qf_w8g_gemm`` call with the current stream's fixup buffer (``w8g_fixup``, looked up once per stream). Same
    launch and bits as ``w8g_gemm(x, q, s, rpw, pdl)``; the C ABI still checks sizes and alignment on every call."""

    def __init__(self, q: torch.Tensor, s: torch.Tensor, rpw: int = 0, pdl: bool = False):
        op = "W8Linear"
        _req(q.is_cuda and s.is_cuda and q.device == s.device, f"{op}: q and s must be CUDA tensors on one device")
        _req(q.dtype == torch.int8 and s.dtype == BF16 and q.dim() == 2 and s.dim() == 2 and q.is_contiguous()
             and s.is_contiguous(), f"{op}: q must be contiguous int8 [N, K] and s contiguous bf16 [N, K/group]")
        _req(s.size(0) == q.size(0) and q.size(1) % s.size(1) == 0, f"{op}: scale shape")
        self.q, self.s, self.dev = q, s, q.device
        self.N, self.K = q.shape
        self.group = self.K // s.shape[1]
        self._args = (q.data_ptr(), s.data_ptr())
        self._rpw, self._pdl = int(rpw), int(bool(pdl))
        self._fix = {}   # stream handle -> (fixup pointer, elements, the buffer)
        self._fn = _lib.load().qf_w8g_gemm

    def __call__(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        op = "W8Linear"
        _req(x.dtype == BF16 and x.dim() == 2 and x.shape[1] == self.K and x.stride(1) == 1 and x.device == self.dev,
             f"{op}: x must be bf16 [M, K] with unit column stride on the weight's device")
        M, N = x.shape[0], self.N
        if out is None:
            out = torch.empty(M, N, dtype=BF16, device=self.dev)
        else:
            _req(out.dtype == BF16 and out.dim() == 2 and out.shape[0] == M and out.shape[1] == N
                 and out.is_contiguous() and out.device == self.dev, f"{op}: out must be contiguous bf16 [M, N]")
        if torch.cuda.current_device() != self.dev.index:
            with torch.cuda.device(self.dev):
                return self(x, out)
        stream = torch.cuda.current_stream()
        st = stream.cuda_stream
        fx = self._fix.get(st)
        if fx is None:
            buf = w8g_fixup(N, self.dev, stream)
            fx = self._fix[st] = (buf.data_ptr(), buf.numel(), buf)
        _lib.check(self._fn(x.data_ptr(), x.stride(0), *self._args, out.data_ptr(), N, M, N, self.K, self.group,
                            self._rpw, fx[0], fx[1], self._pdl, st), "w8g_gemm")
        return out


def w8g_unpack(q: torch.Tensor, s: torch.Tensor, w: torch.Tensor):
    """w bf16 [rows, K] <- bf16(q * s). Mirrors ``w8g_unpack`` (serve/qwenfast/qf_w8g.cu:338-351)."""
    op = "w8g_unpack"
    _req(q.dtype == torch.int8 and s.dtype == BF16 and w.dtype == BF16, f"{op}: dtypes")
    _req(q.dim() == 2 and q.is_contiguous() and s.is_contiguous() and w.is_contiguous() and w.shape == q.shape,
         f"{op}: shapes")
    K = q.shape[1]
    group = K // s.shape[1]
    _req(group * s.shape[1] == K, f"{op}: scale shape")
    with torch.cuda.device(q.device):
        _lib.check(_lib.load().qf_w8g_unpack(q.data_ptr(), s.data_ptr(), w.data_ptr(), q.shape[0], K, group,
                                             _stream(q.device)), op)


_W8A8_FIXUP = {}


def w8a8_fixup(N: int, device, stream=None) -> torch.Tensor:
    """The zero-kept int32 split-K fixup buffer of the W8A8 GEMM for an N-row weight, one per (device, stream, N)."""
    dev = torch.device(device)
    st = (stream or torch.cuda.current_stream(dev)).cuda_stream
    key = (dev.index, st, N)
    buf = _W8A8_FIXUP.get(key)
    if buf is None:
        n = ctypes.c_int64(0)
        _lib.check(_lib.load().qf_w8a8_fixup_elems(N, ctypes.byref(n)), "w8a8_fixup_elems")
        buf = _W8A8_FIXUP[key] = torch.zeros(n.value, dtype=torch.int32, device=dev)
    return buf


def w8a8_gemm(x: torch.Tensor, q: torch.Tensor, sw: torch.Tensor, xq: Optional[torch.Tensor] = None,
              sx: Optional[torch.Tensor] = None, acc_out: Optional[torch.Tensor] = None,
              pdl: bool = True, fixup: Optional[torch.Tensor] = None) -> torch.Tensor:
    """W8A8: per-token int8 activations (absmax/127), per-channel fp32 weight scales, int32 accumulation on the
    tensor cores. ``q`` is the int8 [N, K] weight in the kernel layout of ``formats.repack_w8`` (repacked once at
    load time). Returns y bf16 [M, N], M <= 16. ``xq`` (int8 [16*K], the packed quantised activations) / ``sx``
    (fp32 [M]) scratch are allocated when not given; ``acc_out`` (int32 [M, N]) receives the exact accumulators
    when given; ``fixup`` is the zero-kept split-K buffer (``w8a8_fixup``; the current stream's by default)."""
    op = "w8a8_gemm"
    _cuda(x, "x", op)
    _req(x.dtype == BF16 and x.dim() == 2 and x.stride(1) == 1, f"{op}: x must be bf16 [M, K] with unit column stride")
    _req(q.dtype == torch.int8 and q.dim() == 2 and q.is_contiguous() and q.size(1) == x.size(1), f"{op}: q int8 [N, K]")
    _req(sw.dtype == torch.float32 and sw.numel() == q.size(0), f"{op}: sw fp32 [N]")
    M, K = x.shape
    N = q.shape[0]
    if xq is None:
        xq = torch.empty(16 * K, dtype=torch.int8, device=x.device)
    _req(xq.dtype == torch.int8 and xq.numel() >= 16 * K, f"{op}: xq int8 [16*K]")
    if sx is None:
        sx = torch.empty(max(M, 1), dtype=torch.float32, device=x.device)
    if acc_out is not None:
        _req(acc_out.dtype == torch.int32 and acc_out.numel() >= M * N, f"{op}: acc_out int32 [M, N]")
    if fixup is None and N % 128 == 0:
        fixup = w8a8_fixup(N, x.device)
    y = torch.empty(M, N, dtype=BF16, device=x.device)
    with torch.cuda.device(x.device):
        _lib.check(_lib.load().qf_w8a8_gemm(x.data_ptr(), x.stride(0), q.data_ptr(), sw.data_ptr(), y.data_ptr(), N,
                                            M, N, K, xq.data_ptr(), sx.data_ptr(), _ptr(fixup), _ptr(acc_out),
                                            int(bool(pdl)), _stream(x.device)), op)
    return y


def w8a8_take_status() -> int:
    """Sticky wait-timeout bits of the W8A8 kernel since the last call (0 = clean); clears them. After a non-zero
    status the fixup buffers may hold partial sums, so the cached ones are zeroed again."""
    v = ctypes.c_uint32(0)
    _lib.check(_lib.load().qf_w8a8_take_status(ctypes.byref(v)), "w8a8_take_status")
    if v.value:
        for buf in _W8A8_FIXUP.values():
            buf.zero_()
    return v.value


class W8A8Linear:
    """``w8a8_gemm`` prepared for one weight (q int8 [N, K] in the ``formats.repack_w8`` layout, sw fp32 [N]): the
    weight's checks and C-ABI arguments are made once, and per stream the fixup buffer (``w8a8_fixup``) and the
    quantised-activation scratch (xq int8 [16*K], sx fp32 [16]) are made on first use and reused, stream-ordered. A
    call checks x, allocates y (or writes ``out``) and makes one ``qf_w8a8_gemm`` call: the same launch and bits as
    ``w8a8_gemm(x, q, sw, pdl=pdl)``."""

    def __init__(self, q: torch.Tensor, sw: torch.Tensor, pdl: bool = True):
        op = "W8A8Linear"
        _req(q.is_cuda and sw.device == q.device, f"{op}: q and sw must be CUDA tensors on one device")
        _req(q.dtype == torch.int8 and q.dim() == 2 and q.is_contiguous(), f"{op}: q must be contiguous int8 [N, K]")
        _req(sw.dtype == torch.float32 and sw.numel() == q.size(0) and sw.is_contiguous(), f"{op}: sw fp32 [N]")
        self.q, self.sw, self.dev = q, sw, q.device
        self.N, self.K = q.shape
        self._args = (q.data_ptr(), sw.data_ptr())
        self._pdl = int(bool(pdl))
        self._per_stream = {}   # stream handle -> (xq, sx, fixup pointer or None, the tensors)
        self._fn = _lib.load().qf_w8a8_gemm

    def __call__(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        op = "W8A8Linear"
        _req(x.dtype == BF16 and x.dim() == 2 and x.shape[1] == self.K and x.stride(1) == 1 and x.device == self.dev,
             f"{op}: x must be bf16 [M, K] with unit column stride on the weight's device")
        M, N = x.shape[0], self.N
        if out is None:
            out = torch.empty(M, N, dtype=BF16, device=self.dev)
        else:
            _req(out.dtype == BF16 and out.dim() == 2 and out.shape[0] == M and out.shape[1] == N
                 and out.is_contiguous() and out.device == self.dev, f"{op}: out must be contiguous bf16 [M, N]")
        if torch.cuda.current_device() != self.dev.index:
            with torch.cuda.device(self.dev):
                return self(x, out)
        stream = torch.cuda.current_stream()
        st = stream.cuda_stream
        ps = self._per_stream.get(st)
        if ps is None:
            xq = torch.empty(16 * self.K, dtype=torch.int8, device=self.dev)
            sx = torch.empty(16, dtype=torch.float32, device=self.dev)
            fix = w8a8_fixup(N, self.dev, stream) if N % 128 == 0 else None
            ps = self._per_stream[st] = (xq.data_ptr(), sx.data_ptr(), _ptr(fix), (xq, sx, fix))
        _lib.check(self._fn(x.data_ptr(), x.stride(0), *self._args, out.data_ptr(), N, M, N, self.K, ps[0], ps[1],
                            ps[2], None, self._pdl, st), "w8a8_gemm")
        return out
