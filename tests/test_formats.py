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
    assert torch.equal(formats.w4_word_map(N, K, gated).sort().values, torch.arange(N * K // 8))
    assert torch.equal(formats.w4_scale_map(N, K, gated).sort().values, torch.arange(N * K // 128))


@pytest.mark.parametrize("N,K,gated", [(1024, 2048, True), (2048, 512, False), (256, 64, True)])
def test_bf16_round_trip(N, K, gated):
    w = torch.randn(N, K).to(torch.bfloat16)
    wk = formats.repack_bf16_torch(w, gated)
    assert torch.equal(formats.unpack_bf16_torch(wk, N, K, gated), w)
    assert torch.equal(formats.bf16_elem_map(N, K, gated).sort().values, torch.arange(N * K))


def test_gate_up_rows_interleave_in_lanes():
    src = formats.kernel_row_source(256, True)
    # tile 0: even lane 2j is gate row j, odd lane 2j+1 the matching up row 128 + j; tile 1 continues at gate row 64
    assert src[:6].tolist() == [0, 128, 1, 129, 2, 130]
    assert src[128:132].tolist() == [64, 192, 65, 193]


def test_pack_unpack_int4_and_nibble_order():
    codes = torch.randint(0, 16, (3, 5, 64))
    words = formats.pack_int4(codes)
    assert torch.equal(formats.unpack_int4(words).long(), codes)
    # kernel nibble order: nibble i of a kernel word holds k = [0,2,4,6,1,3,5,7][i] of its eight
    w = formats.pack_int4(torch.arange(8).view(1, 8))
    p = formats._nibble_perm(w, True)
    assert [(int(p) >> (4 * i)) & 0xF for i in range(8)] == [0, 2, 4, 6, 1, 3, 5, 7]
    assert torch.equal(formats._nibble_perm(p, False), w)


def test_stage_layout_positions():
    # int4: a stage is 128 k x 128 rows = 2048 words [half h][quad q][lane p][word j], k = 128s + 64h + 32q + 8j
    N, K = 128, 256
    wm = formats.w4_word_map(N, K, False)
    s, h, q, p, j = 1, 1, 1, 5, 2
    o = 2048 * s + 512 * (2 * h + q) + 4 * p + j
    assert int(wm[o]) == p * (K // 8) + (16 * s + 8 * h + 4 * q + j)
    # scales: [stage][lane]
    sm = formats.w4_scale_map(N, K, False)
    assert int(sm[128 * 1 + 5]) == 5 * (K // 128) + 1
    # bf16: a stage is 32 k x 128 rows [chunk c][lane p][8 elements], k = 32s + 8c + el
    bm = formats.bf16_elem_map(N, 64, False)
    assert int(bm[4096 * 1 + 1024 * 2 + 8 * 3 + 4]) == 3 * 64 + (32 + 16 + 4)


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
    the kernel reads there -- a thread of lane p in tile r reads stage st's word (quad q, word j) at
    [st][q][p][j] (nibble i = k 32q + 8j + [0,2,4,6,1,3,5,7][i]) and its eight group scales at [st][p][0..8)."""
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
        perm = formats.NIBBLE_ORDER
        for e, r, st, q, p, j in ((0, 0, 0, 0, 0, 0), (1, 1, 2, 3, 127, 3), (0, 1, 1, 2, 77, 1), (1, 0, 2, 1, 6, 2)):
            word = int(wk[e, r * (128 * K // 8) + st * 2048 + q * 512 + p * 4 + j]) & 0xFFFFFFFF
            row = int(src[128 * r + p])
            for i in range(8):
                assert (word >> (4 * i)) & 15 == int(codes[e, row, 128 * st + 32 * q + 8 * j + perm[i]])
            for gi in range(8):
                got = int(sk[e, r * (128 * K // 16) + st * 1024 + p * 8 + gi])
                assert got == int(sf.view(torch.uint8)[e, row, 8 * st + gi])
