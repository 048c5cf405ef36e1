"""Weight formats: the canonical int4 expert format and the kernel-native layouts the sm_100a kernels stream.

Canonical (what a checkpoint loader holds, and the synthetic configurations' definition)
    int4 codes 0..15, zero point 8, eight codes per int32 along K with the lowest k in the low nibble:
    ``qweight int32 [E, N, K/8]``; one bf16 scale per 128 k: ``scales bf16 [E, N, K/128]``;
    dequantised weight ``(code - 8) * scale``.

Kernel layout (one expert matrix [N, K]; ``gated`` for gate_up, where N = 2I rows are gate then up)
    128-row tiles of eight m16 tiles (the tensor cores' m16n8k16 register fragments). Plain: m16 tile m of tile r
    holds rows 128r + 16m .. +15. gate_up: its fragment rows g = 0..7 are gate rows 64r + 8m + g and rows 8 + g the
    matching up rows N/2 + 64r + 8m + g, so one lane's fragment holds a whole SwiGLU pair.
    int4: each tile is a run of stages of 128 k (one scale group, 8 KB); a stage is [m16 tile m][64-k half h]
    [lane (32)][step s (4)] words. The word of lane (g, t4) holds rows A = 16m + g and B = A + 8 at the four k
    128st + 64h + 16t4 + 4s + (0..3): nibbles 0, 4, 2, 6 are A's codes, 1, 5, 3, 7 B's, so nibble pair (j, j + 4)
    is the mma's A register j after one lop3, and the lane's k run matches one 32-byte run of each token row.
    Scales per stage: [consumer warp w (4)][g (8)][c (4)] bf16 = row 16(2w + c/2) + g + 8(c % 2).
bf16 (the shared expert): stages of 32 k laid out [m16 tile m][step s (2)][lane][8 elements]: element 2w + h of lane
    (g, t4) is row 16m + g + 8(w % 2) at k = 32st + 8t4 + 4s + 2(w // 2) + h -- the A registers of each k16 step.
NVFP4: the e2m1 codes in the int4 layout; the E4M3 scales (one per 16 k) per stage [w][lane][8 bytes], byte
    (mm * 2 + h) * 2 + ro = row 16(2w + mm) + g + 8 ro, group 8st + 4h + t4 (the lane's 16 k of that half).

W8A8 weights (int8 [N, K]): contiguous 16 KB tiles [N/128][K/128][128 rows][128 B], each row's 16-byte k chunk c
    stored at position c ^ (row % 8) -- the K-major 128-byte-swizzle operand layout of the tensor cores.

The CUDA entry points ``qf_w4_repack``/``qf_bf16_repack``/``qf_w8_repack`` produce these layouts on the device; the
``*_torch`` functions here compute the same index maps with tensor ops (any device) and are used by the CPU tests.
"""
import ctypes

import torch

from . import _lib

# kernel-word nibble i holds row B (i odd) or A (i even) at k offset KPOS[i] of the word's four k
KPOS = (0, 0, 2, 2, 1, 1, 3, 3)


# ------------------------------------------------------------------------------------------ canonical helpers
def pack_int4(codes: torch.Tensor) -> torch.Tensor:
    """int codes [..., N, K] in 0..15 -> int32 [..., N, K/8] (lowest k in the low nibble)."""
    c = codes.to(torch.int64).reshape(*codes.shape[:-1], codes.shape[-1] // 8, 8)
    shifts = torch.arange(0, 32, 4, device=codes.device, dtype=torch.int64)
    w = (c << shifts).sum(-1)
    w = torch.where(w >= 2 ** 31, w - 2 ** 32, w)
    return w.to(torch.int32)


def unpack_int4(words: torch.Tensor) -> torch.Tensor:
    shifts = torch.arange(0, 32, 4, device=words.device, dtype=torch.int32)
    q = (words.unsqueeze(-1) >> shifts) & 0xF
    return q.reshape(*words.shape[:-1], words.shape[-1] * 8)


# ----------------------------------------------------------------------------------------------- index maps
def kernel_row_source(N: int, gated: bool, device=None) -> torch.Tensor:
    """Kernel row position -> source row."""
    p = torch.arange(N, device=device, dtype=torch.int64)
    if not gated:
        return p
    r, rho = p // 128, p % 128
    j = 64 * r + 8 * (rho // 16) + rho % 8
    return torch.where((rho & 8) == 0, j, N // 2 + j)


def w4_code_map(N: int, K: int, gated: bool, device=None) -> torch.Tensor:
    """Kernel-layout code (word o, nibble i), flattened o * 8 + i -> canonical code index row * K + k."""
    o = torch.arange(N * K // 8, device=device, dtype=torch.int64)
    per_tile = 128 * K // 8
    r, ot = o // per_tile, o % per_tile
    st, os_ = ot // 2048, ot % 2048
    s, lane, h, m = os_ & 3, (os_ >> 2) & 31, (os_ >> 7) & 1, os_ >> 8
    k0 = 128 * st + 64 * h + 16 * (lane & 3) + 4 * s
    src = kernel_row_source(N, gated, device)
    ra = src[128 * r + 16 * m + (lane >> 2)]
    rb = src[128 * r + 16 * m + (lane >> 2) + 8]
    i = torch.arange(8, device=device, dtype=torch.int64)
    kpos = torch.tensor(KPOS, device=device, dtype=torch.int64)
    row = torch.where((i & 1) == 0, ra[:, None], rb[:, None])
    return (row * K + k0[:, None] + kpos[None, :]).reshape(-1)


def w4_scale_map(N: int, K: int, gated: bool, device=None) -> torch.Tensor:
    """Kernel-layout scale entry o -> canonical index row * (K/128) + group."""
    o = torch.arange(N * K // 128, device=device, dtype=torch.int64)
    r, ot = o // K, o % K
    st, e = ot // 128, ot % 128
    w, g, c = e >> 5, (e >> 2) & 7, e & 3
    row = kernel_row_source(N, gated, device)[128 * r + 16 * (2 * w + (c >> 1)) + g + 8 * (c & 1)]
    return row * (K // 128) + st


def nvfp4_scale_map(N: int, K: int, gated: bool, device=None) -> torch.Tensor:
    """NVFP4 kernel-layout scale byte o -> canonical index row * (K/16) + group, for one [N, K] matrix: per 128-row
    tile r and 128-k stage st, [consumer warp w (4)][lane (32)][8 bytes], byte (mm * 2 + h) * 2 + ro = row
    16(2w + mm) + g + 8 ro at 16-k group 8st + 4h + t4 -- one 8-byte load gives a lane every scale of its stage."""
    o = torch.arange(N * K // 16, device=device, dtype=torch.int64)
    per_tile = 128 * K // 16
    r, ot = o // per_tile, o % per_tile
    st, os_ = ot // 1024, ot % 1024
    w, lane, b = os_ >> 8, (os_ >> 3) & 31, os_ & 7
    mm, h, ro = b >> 2, (b >> 1) & 1, b & 1
    row = kernel_row_source(N, gated, device)[128 * r + 16 * (2 * w + mm) + (lane >> 2) + 8 * ro]
    return row * (K // 16) + 8 * st + 4 * h + (lane & 3)


def bf16_elem_map(N: int, K: int, gated: bool, device=None) -> torch.Tensor:
    """bf16 kernel-layout element o -> canonical index row * K + k."""
    o = torch.arange(N * K, device=device, dtype=torch.int64)
    per_tile = 128 * K
    r, ot = o // per_tile, o % per_tile
    st, os_ = ot >> 12, ot & 4095
    el, lane, s, m = os_ & 7, (os_ >> 3) & 31, (os_ >> 8) & 1, os_ >> 9
    w, h = el >> 1, el & 1
    k = 32 * st + 8 * (lane & 3) + 4 * s + 2 * (w >> 1) + h
    row = kernel_row_source(N, gated, device)[128 * r + 16 * m + (lane >> 2) + 8 * (w & 1)]
    return row * K + k


def w8_byte_map(N: int, K: int, device=None) -> torch.Tensor:
    """W8A8 kernel layout byte o -> canonical index n * K + k: contiguous 16 KB tiles [N/128][K/128][128 rows]
    [128 bytes], the row's 16-byte k chunk c stored at position c ^ (row % 8) (K-major 128-byte swizzle)."""
    o = torch.arange(N * K, device=device, dtype=torch.int64)
    tile, within = o // 16384, o % 16384
    r, ks = tile // (K // 128), tile % (K // 128)
    rr, pos, b = within // 128, (within // 16) % 8, within % 16
    c = pos ^ (rr % 8)
    return (r * 128 + rr) * K + ks * 128 + c * 16 + b


def _check_w4(qweight, scales):
    if qweight.dtype != torch.int32 or qweight.dim() != 3:
        raise RuntimeError("qweight must be int32 [E, N, K/8]")
    E, N, KW = qweight.shape
    K = KW * 8
    if scales.dtype != torch.bfloat16 or tuple(scales.shape) != (E, N, K // 128):
        raise RuntimeError(f"scales must be bf16 [E, N, K/128] = {(E, N, K // 128)}, got {tuple(scales.shape)}")
    if N % 128 or K % 128:
        raise RuntimeError(f"N and K must be multiples of 128, got N={N}, K={K}")
    return E, N, K


# ------------------------------------------------------------------------------------------ torch versions
_CHUNK = 16   # experts per gather step of the torch repacks (bounds the temporary code tensors)


def _codes_to_kernel(words: torch.Tensor, N: int, K: int, gated: bool) -> torch.Tensor:
    """Canonical code words int32 [E, N*K/8] -> kernel-layout words int32 [E, N*K/8] (codes gathered)."""
    E = words.shape[0]
    cmap = w4_code_map(N, K, gated, words.device)
    out = torch.empty(E, N * K // 8, dtype=torch.int32, device=words.device)
    for e0 in range(0, E, _CHUNK):
        codes = unpack_int4(words[e0:e0 + _CHUNK]).to(torch.uint8)
        out[e0:e0 + _CHUNK] = pack_int4(codes[:, cmap].view(codes.shape[0], -1))
    return out


def _codes_to_canonical(wk: torch.Tensor, N: int, K: int, gated: bool) -> torch.Tensor:
    """Inverse of ``_codes_to_kernel``."""
    E = wk.shape[0]
    cmap = w4_code_map(N, K, gated, wk.device)
    out = torch.empty(E, N * K // 8, dtype=torch.int32, device=wk.device)
    for e0 in range(0, E, _CHUNK):
        codes = unpack_int4(wk[e0:e0 + _CHUNK]).to(torch.uint8)
        canon = torch.empty_like(codes)
        canon[:, cmap] = codes
        out[e0:e0 + _CHUNK] = pack_int4(canon)
    return out


def repack_w4_torch(qweight: torch.Tensor, scales: torch.Tensor, gated: bool):
    E, N, K = _check_w4(qweight, scales)
    wk = _codes_to_kernel(qweight.reshape(E, -1), N, K, gated)
    sk = scales.reshape(E, -1)[:, w4_scale_map(N, K, gated, qweight.device)]
    return wk.contiguous(), sk.contiguous()


def unpack_w4_torch(wk: torch.Tensor, sk: torch.Tensor, N: int, K: int, gated: bool):
    E = wk.shape[0]
    q = _codes_to_canonical(wk, N, K, gated)
    s = torch.empty(E, N * K // 128, dtype=sk.dtype, device=sk.device)
    s[:, w4_scale_map(N, K, gated, sk.device)] = sk
    return q.view(E, N, K // 8), s.view(E, N, K // 128)


def repack_nvfp4(wp: torch.Tensor, sf: torch.Tensor, gated: bool):
    """Canonical NVFP4 experts (the reference's checkpoint format: codes uint8 [E, N, K/2], even k in the low
    nibble; E4M3 scales [E, N, K/16]) -> the kernel layout on the tensors' device: the codes in the int4 layout
    (int32 [E, N*K/8]), the scales uint8
    [E, N*K/16] per ``nvfp4_scale_map``. Returns (wk, sk)."""
    if wp.dtype != torch.uint8 or wp.dim() != 3 or sf.dtype != torch.float8_e4m3fn:
        raise RuntimeError("NVFP4 experts need codes uint8 [E, N, K/2] and float8_e4m3fn scales [E, N, K/16]")
    E, N, K2 = wp.shape
    K = 2 * K2
    if tuple(sf.shape) != (E, N, K // 16) or N % 128 or K % 128:
        raise RuntimeError(f"NVFP4 scales must be [E, N, K/16] = {(E, N, K // 16)} with N, K multiples of 128")
    words = wp.contiguous().view(torch.int32).view(E, N * K // 8)
    wk = _codes_to_kernel(words, N, K, gated)
    sk = sf.contiguous().view(torch.uint8).reshape(E, -1)[:, nvfp4_scale_map(N, K, gated, wp.device)]
    return wk.contiguous(), sk.contiguous()


def unpack_nvfp4(wk: torch.Tensor, sk: torch.Tensor, N: int, K: int, gated: bool):
    """Inverse of ``repack_nvfp4`` (exact): (codes uint8 [E, N, K/2], scales float8_e4m3fn [E, N, K/16])."""
    E = wk.shape[0]
    words = _codes_to_canonical(wk, N, K, gated)
    sf = torch.empty(E, N * K // 16, dtype=torch.uint8, device=sk.device)
    sf[:, nvfp4_scale_map(N, K, gated, sk.device)] = sk
    return words.view(torch.uint8).view(E, N, K // 2), sf.view(torch.float8_e4m3fn).view(E, N, K // 16)


def repack_bf16_torch(w: torch.Tensor, gated: bool) -> torch.Tensor:
    N, K = w.shape
    if N % 128 or K % 32:
        raise RuntimeError(f"bf16 weight needs N % 128 == 0 and K % 32 == 0, got {N}x{K}")
    return w.reshape(-1)[bf16_elem_map(N, K, gated, w.device)].contiguous()


def unpack_bf16_torch(wk: torch.Tensor, N: int, K: int, gated: bool) -> torch.Tensor:
    w = torch.empty(N * K, dtype=wk.dtype, device=wk.device)
    w[bf16_elem_map(N, K, gated, wk.device)] = wk.reshape(-1)
    return w.view(N, K)


def repack_w8_torch(q: torch.Tensor) -> torch.Tensor:
    """Canonical int8 [N, K] -> W8A8 kernel layout (same shape and dtype, bytes permuted)."""
    N, K = q.shape
    if N % 128 or K % 128:
        raise RuntimeError(f"W8A8 weight needs N % 128 == 0 and K % 128 == 0, got {N}x{K}")
    return q.reshape(-1)[w8_byte_map(N, K, q.device)].view(N, K).contiguous()


def unpack_w8_torch(qk: torch.Tensor) -> torch.Tensor:
    N, K = qk.shape
    q = torch.empty(N * K, dtype=qk.dtype, device=qk.device)
    q[w8_byte_map(N, K, qk.device)] = qk.reshape(-1)
    return q.view(N, K)


# ------------------------------------------------------------------------------------ device (C ABI) versions
def _stream(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _req_cuda(*ts):
    for t in ts:
        if not t.is_cuda or not t.is_contiguous():
            raise RuntimeError("expected contiguous CUDA tensors")


def repack_w4(qweight: torch.Tensor, scales: torch.Tensor, gated: bool):
    """Canonical int4 experts -> kernel layout on the GPU. Returns (wk int32 [E, N*K/8], sk bf16 [E, N*K/128])."""
    E, N, K = _check_w4(qweight, scales)
    _req_cuda(qweight, scales)
    wk = torch.empty(E, N * K // 8, dtype=torch.int32, device=qweight.device)
    sk = torch.empty(E, N * K // 128, dtype=torch.bfloat16, device=qweight.device)
    with torch.cuda.device(qweight.device):
        _lib.check(_lib.load().qf_w4_repack(qweight.data_ptr(), scales.data_ptr(), wk.data_ptr(), sk.data_ptr(),
                                            E, N, K, int(gated), _stream(qweight)), "w4_repack")
    return wk, sk


def unpack_w4(wk: torch.Tensor, sk: torch.Tensor, N: int, K: int, gated: bool):
    _req_cuda(wk, sk)
    E = wk.shape[0]
    q = torch.empty(E, N, K // 8, dtype=torch.int32, device=wk.device)
    s = torch.empty(E, N, K // 128, dtype=torch.bfloat16, device=wk.device)
    with torch.cuda.device(wk.device):
        _lib.check(_lib.load().qf_w4_unpack(wk.data_ptr(), sk.data_ptr(), q.data_ptr(), s.data_ptr(), E, N, K,
                                            int(gated), _stream(wk)), "w4_unpack")
    return q, s


def repack_bf16(w: torch.Tensor, gated: bool) -> torch.Tensor:
    _req_cuda(w)
    N, K = w.shape
    wk = torch.empty(N * K, dtype=torch.bfloat16, device=w.device)
    with torch.cuda.device(w.device):
        _lib.check(_lib.load().qf_bf16_repack(w.data_ptr(), wk.data_ptr(), N, K, int(gated), _stream(w)), "bf16_repack")
    return wk


def unpack_bf16(wk: torch.Tensor, N: int, K: int, gated: bool) -> torch.Tensor:
    _req_cuda(wk)
    w = torch.empty(N, K, dtype=torch.bfloat16, device=wk.device)
    with torch.cuda.device(wk.device):
        _lib.check(_lib.load().qf_bf16_unpack(wk.data_ptr(), w.data_ptr(), N, K, int(gated), _stream(wk)), "bf16_unpack")
    return w


def repack_w8(q: torch.Tensor) -> torch.Tensor:
    """Canonical int8 [N, K] -> the W8A8 kernel layout on the GPU (``qf_w8_repack``); same shape, bytes permuted.
    Synchronises the current stream when done (a load-time step)."""
    _req_cuda(q)
    if q.dtype != torch.int8 or q.dim() != 2:
        raise RuntimeError("q must be int8 [N, K]")
    N, K = q.shape
    qk = torch.empty_like(q)
    with torch.cuda.device(q.device):
        _lib.check(_lib.load().qf_w8_repack(q.data_ptr(), qk.data_ptr(), N, K, _stream(q)), "w8_repack")
        # load-time step: the GEMM requests weight tiles before its griddepcontrol.wait, so the repacked weights
        # must be complete before any GEMM launch that could follow this kernel directly
        torch.cuda.current_stream(q.device).synchronize()
    return qk


def unpack_w8(qk: torch.Tensor) -> torch.Tensor:
    _req_cuda(qk)
    N, K = qk.shape
    q = torch.empty_like(qk)
    with torch.cuda.device(qk.device):
        _lib.check(_lib.load().qf_w8_unpack(qk.data_ptr(), q.data_ptr(), N, K, _stream(qk)), "w8_unpack")
    return q
