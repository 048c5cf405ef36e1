"""On-disk format of repacked MoE layers, and the exactness check of a repack.

The reference repacks its experts once at load time (``process_weights_after_loading``,
compressed_tensors_w4a4_nvfp4_moe.py:302-364) and checks that its own packed formats reproduce the original bit for
bit (``pk_pack``, serve/overlays/sglang/srt/qwenfast.py:195-202: one unpack per row block, compared with
``torch.equal``, ``RuntimeError`` otherwise). Here:

* ``verify_layer(lw, canonical)`` -- the kernel-layout tensors of a ``MoELayerWeights`` unpacked again (on their own
  device: the CUDA unpack kernels for CUDA tensors, the torch index maps otherwise) and compared with the canonical
  tensors, expert by expert; ``RuntimeError`` on the first difference.
* ``save_layer(path, lw)`` / ``load_layer(path, device)`` -- one layer in a safetensors file: the kernel-layout
  tensors as they are streamed by the kernels (no repack at load), plus metadata naming this format and its
  version, the layer's sizes, and a SHA-256 digest of every tensor's bytes. ``load_layer`` refuses another format
  or version, sizes that do not match the tensors, and (``verify=True``, the default) any tensor whose bytes do not
  match its digest.
"""
import hashlib
import json

import torch
from safetensors.torch import load_file, save_file

from . import formats
from .ops import MoELayerWeights

FORMAT = "qwenfast_b200.moe_layer"
VERSION = 2   # 2: int4 / bf16 / NVFP4 stages in mma fragment order
_TENSORS = ("router", "w13", "s13", "w2", "s2", "w_gate", "sh_w13", "sh_w2")


def _digest(t: torch.Tensor) -> str:
    b = t.detach().contiguous().cpu()
    return hashlib.sha256(b.view(torch.uint8).numpy().tobytes() if b.numel() else b"").hexdigest()


def _expected_shapes(H, I, E, Is):
    shapes = dict(router=(E, H), w13=(E, 2 * I * H // 8), s13=(E, 2 * I * H // 128), w2=(E, H * I // 8),
                  s2=(E, H * I // 128))
    if Is:
        shapes.update(w_gate=(H,), sh_w13=(2 * Is * H,), sh_w2=(H * Is,))
    return shapes


def save_layer(path: str, lw: MoELayerWeights) -> None:
    """Write one kernel-layout layer (any device) to ``path`` (safetensors)."""
    tensors = {n: getattr(lw, n).detach().contiguous().cpu() for n in _TENSORS if getattr(lw, n) is not None}
    meta = dict(format=FORMAT, version=str(VERSION), H=str(lw.H), I=str(lw.I), E=str(lw.E), Is=str(lw.Is),
                digests=json.dumps({n: _digest(t) for n, t in tensors.items()}, sort_keys=True))
    save_file(tensors, path, metadata=meta)


def load_layer(path: str, device="cuda", verify: bool = True) -> MoELayerWeights:
    """Read a layer written by ``save_layer`` onto ``device``; see the module docstring for the checks."""
    from safetensors import safe_open
    with safe_open(path, framework="pt") as f:
        meta = f.metadata() or {}
    if meta.get("format") != FORMAT or meta.get("version") != str(VERSION):
        raise RuntimeError(f"{path}: not a {FORMAT} v{VERSION} file (format {meta.get('format')!r}, "
                           f"version {meta.get('version')!r})")
    H, I, E, Is = (int(meta[k]) for k in ("H", "I", "E", "Is"))
    tensors = load_file(path)
    want = _expected_shapes(H, I, E, Is)
    for n, shape in want.items():
        if n not in tensors or tuple(tensors[n].shape) != shape:
            got = None if n not in tensors else tuple(tensors[n].shape)
            raise RuntimeError(f"{path}: tensor {n} has shape {got}, the metadata's sizes need {shape}")
    if verify:
        digests = json.loads(meta["digests"])
        for n, t in tensors.items():
            if digests.get(n) != _digest(t):
                raise RuntimeError(f"{path}: tensor {n} does not match its recorded digest")
    t = {n: v.to(device) for n, v in tensors.items()}
    return MoELayerWeights(t["router"], t["w13"], t["s13"], t["w2"], t["s2"], t.get("w_gate"), t.get("sh_w13"),
                           t.get("sh_w2"), H, I, E, Is)


def _unpack_w4(wk, sk, N, K, gated):
    if wk.is_cuda:
        return formats.unpack_w4(wk, sk, N, K, gated)
    return formats.unpack_w4_torch(wk, sk, N, K, gated)


def _unpack_bf16(wk, N, K, gated):
    if wk.is_cuda:
        return formats.unpack_bf16(wk, N, K, gated)
    return formats.unpack_bf16_torch(wk, N, K, gated)


def verify_layer(lw: MoELayerWeights, canonical: dict, experts_per_block: int = 64) -> None:
    """Raise ``RuntimeError`` unless the kernel-layout layer reproduces ``canonical`` exactly (keys ``w13``, ``s13``,
    ``w2``, ``s2`` and, when the layer has a shared expert, ``sh_gu``, ``sh_d``), unpacking a block of experts at a
    time."""
    H, I, E = lw.H, lw.I, lw.E
    for e0 in range(0, E, experts_per_block):
        e1 = min(E, e0 + experts_per_block)
        for name, wk, sk, N, K, gated in (("w13", lw.w13, lw.s13, 2 * I, H, True), ("w2", lw.w2, lw.s2, H, I, False)):
            q, s = _unpack_w4(wk[e0:e1].contiguous(), sk[e0:e1].contiguous(), N, K, gated)
            sname = "s13" if name == "w13" else "s2"
            if not (torch.equal(q.cpu(), canonical[name][e0:e1].cpu())
                    and torch.equal(s.view(torch.int16).cpu(), canonical[sname][e0:e1].view(torch.int16).cpu())):
                raise RuntimeError(f"repacked {name} experts {e0}..{e1 - 1} do not reproduce the original")
    if lw.Is:
        for name, wk, N, K, gated in (("sh_gu", lw.sh_w13, 2 * lw.Is, H, True), ("sh_d", lw.sh_w2, H, lw.Is, False)):
            w = _unpack_bf16(wk, N, K, gated)
            if not torch.equal(w.view(torch.int16).cpu(), canonical[name].view(torch.int16).cpu()):
                raise RuntimeError(f"repacked shared expert {name} does not reproduce the original")
