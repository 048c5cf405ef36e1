"""Kernel-native weight layouts (host-side index maps): exact round trips and full permutations."""
import pytest
import torch

from qwenfast_b200 import formats, synthetic


@pytest.mark.parametrize("N,K,gated", [(256, 256, True), (256, 128, False), (1024, 2048, True), (2048, 512, False),
                                       (384, 384, False), (128, 640, True)])
def test_w4_round_trip(N, K, gated):
    E = 2
    q = synthetic.random_int4_words((E, N, K // 8), torch.Generator().manual_seed(N + K), "cpu")
    s = synthetic.group_scales((E, N, K // 128), torch.Generator().manual_seed(1), "cpu")
    wk, sk = formats.repack_w4_torch(q, s, gated)
    q2, s2 = formats.unpack_w4_torch(wk, sk, N, K, gated)
    assert torch.equal(q, q2) and torch.equal(s, s2)
    assert torch.equal(formats.w4_code_map(N, K, gated).sort().values, torch.arange(N * K))
    assert torch.equal(formats.w4_scale_map(N, K, gated).sort().values, torch.arange(N * K // 128))


@pytest.mark.parametrize("N,K,gated", [(1024, 2048, True), (2048, 512, False), (256, 64, True)])
def test_bf16_round_trip(N, K, gated):
    w = torch.randn(N, K).to(torch.bfloat16)
    wk = formats.repack_bf16_torch(w, gated)
    assert torch.equal(formats.unpack_bf16_torch(wk, N, K, gated), w)
    assert torch.equal(formats.bf16_elem_map(N, K, gated).sort().values, torch.arange(N * K))


def test_gate_up_rows_pair_in_fragments():
    src = formats.kernel_row_source(256, True)
    # tile 0, m16 tile 0: fragment rows 0..7 are gate rows 0..7, rows 8..15 the matching up rows 128..135; m16 tile 1
    # continues at gate row 8; tile 1 starts at gate row 64
    assert src[:16].tolist() == list(range(8)) + list(range(128, 136))
    assert src[16:18].tolist() == [8, 9] and src[24:26].tolist() == [136, 137]
    assert src[128:130].tolist() == [64, 65] and src[136] == 192


def test_pack_unpack_int4():
    codes = torch.randint(0, 16, (3, 5, 64))
    words = formats.pack_int4(codes)
    assert torch.equal(formats.unpack_int4(words).long(), codes)


def _w4_positions(N, K, gated, r, st, m, h, lane, s):
    """(kernel word index, rows A / B, first k) of tile r, stage st, m16 tile m, half h, lane, step s."""
    src = formats.kernel_row_source(N, gated)
    o = r * (128 * K // 8) + st * 2048 + ((m * 2 + h) * 32 + lane) * 4 + s
    g, t4 = lane >> 2, lane & 3
    return o, int(src[128 * r + 16 * m + g]), int(src[128 * r + 16 * m + g + 8]), 128 * st + 64 * h + 16 * t4 + 4 * s


@pytest.mark.parametrize("gated", [False, True])
def test_stage_layout_positions(gated):
    # int4: word [tile][stage][m16 tile m][half h][lane][step s] holds rows A (nibbles 0, 4, 2, 6 = k+0..k+3) and
    # B = A + 8 (nibbles 1, 5, 3, 7) of its lane's fragment
    N, K = 256, 384
    codes = torch.randint(0, 16, (1, N, K), generator=torch.Generator().manual_seed(3))
    q = formats.pack_int4(codes)
    s_ = torch.rand(1, N, K // 128).to(torch.bfloat16)
    wk, sk = formats.repack_w4_torch(q, s_, gated)
    for (r, st, m, h, lane, s) in ((0, 0, 0, 0, 0, 0), (1, 2, 7, 1, 31, 3), (0, 1, 3, 0, 13, 2), (1, 0, 5, 1, 6, 1)):
        o, ra, rb, k0 = _w4_positions(N, K, gated, r, st, m, h, lane, s)
        word = int(wk[0, o]) & 0xFFFFFFFF
        got = [(word >> (4 * i)) & 15 for i in range(8)]
        want = [int(codes[0, ra if i % 2 == 0 else rb, k0 + formats.KPOS[i]]) for i in range(8)]
        assert got == want
    # scales: stage st, [warp w][g][c] = row 16 (2w + c/2) + g + 8 (c % 2)
    src = formats.kernel_row_source(N, gated)
    w, g, c, st = 2, 5, 3, 1
    row = int(src[128 + 16 * (2 * w + 1) + g + 8])
    assert sk[0, 1 * K + 128 * st + w * 32 + g * 4 + c] == s_[0, row, st]
    # bf16: a stage is 32 k x 128 rows [m16 tile m][step s][lane][8], element 2w + h = row 16m + g + 8(w%2),
    # k = 32 st + 8 t4 + 4 s + 2 (w // 2) + h
    bm = formats.bf16_elem_map(128, 64, False)
    m, s, lane, el = 3, 1, 9, 5   # g = 2, t4 = 1, w = 2, h = 1
    assert int(bm[4096 * 1 + ((m * 2 + s) * 32 + lane) * 8 + el]) == (16 * m + 2) * 64 + (32 + 8 + 4 + 2 + 1)


@pytest.mark.parametrize("N,K", [(128, 128), (256, 2048), (384, 640)])
def test_w8_layout_round_trip_and_swizzle(N, K):
    q = torch.randint(-127, 128, (N, K), dtype=torch.int8)
    qk = formats.repack_w8_torch(q)
    assert torch.equal(formats.unpack_w8_torch(qk), q)
    assert torch.equal(formats.w8_byte_map(N, K).sort().values, torch.arange(N * K))
    # tile (0, 0): row 3's chunk 1 (k = 16..31) sits at position 1 ^ 3 = 2 of the row
    assert torch.equal(qk.reshape(-1)[3 * 128 + 2 * 16: 3 * 128 + 3 * 16], q[3, 16:32])


def test_nvfp4_kernel_layout():
    """NVFP4 experts (the reference's format) in the kernel layout: exact round trip, and each position holds what
    the kernel reads there -- the codes in the int4 fragment layout, and lane (g, t4) of consumer warp w finds the
    E4M3 scale of row 16 (2w + mm) + g + 8 ro, 16-k group 8 st + 4 h + t4 at byte (mm * 2 + h) * 2 + ro of its
    8 bytes [st][w][lane]."""
    from oracle import nvfp4_ref
    g = torch.Generator().manual_seed(5)
    E, N, K = 2, 256, 384
    for gated in (True, False):
        wp, sf = nvfp4_ref.random_nvfp4((E, N, K), g)
        wk, sk = formats.repack_nvfp4(wp, sf, gated)
        wp2, sf2 = formats.unpack_nvfp4(wk, sk, N, K, gated)
        assert torch.equal(wp2, wp) and torch.equal(sf2.view(torch.uint8), sf.view(torch.uint8))
        codes = nvfp4_ref.unpack_e2m1(wp)                      # [E, N, K]
        src = formats.kernel_row_source(N, gated)
        for e, r, st, m, h, lane, s in ((0, 0, 0, 0, 0, 0, 0), (1, 1, 2, 7, 1, 31, 3), (0, 1, 1, 2, 0, 17, 1)):
            o, ra, rb, k0 = _w4_positions(N, K, gated, r, st, m, h, lane, s)
            word = int(wk[e, o]) & 0xFFFFFFFF
            for i in range(8):
                assert (word >> (4 * i)) & 15 == int(codes[e, ra if i % 2 == 0 else rb, k0 + formats.KPOS[i]])
        sfu = sf.view(torch.uint8)
        for e, r, st, w, lane, b in ((0, 0, 0, 0, 0, 0), (1, 1, 2, 3, 31, 7), (0, 1, 1, 2, 9, 5)):
            mm, h, ro = b >> 2, (b >> 1) & 1, b & 1
            row = int(src[128 * r + 16 * (2 * w + mm) + (lane >> 2) + 8 * ro])
            got = int(sk[e, r * (128 * K // 16) + st * 1024 + (w * 32 + lane) * 8 + b])
            assert got == int(sfu[e, row, 8 * st + 4 * h + (lane & 3)])
