"""INT8 dense GEMMs on the GPU vs the CPU oracle.

W8A16 (w8g, reference qf_w8g.cu): relative L2 < 4e-3 against the fp32 truth x @ (q * s)^T
(the bound of serve/qwenfast/test_w8k.py:88); w8g_unpack bit-exact.
W8A8 (config 3): the activation quantisation (xq, sx), the int32 accumulators and the bf16 outputs are all
bit-exact against the oracle (exact int64 accumulation, the same fp32 multiplies in the same order)."""
import pytest
import torch

from oracle import w8_ref
from qwenfast_b200 import formats, ops, synthetic

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("N,K", [(2048, 2048), (1280, 2560), (2560, 640), (2560, 6144), (4096, 2048), (12288, 2560),
                                 (16384, 2048), (8192, 6144), (12288, 6144), (16480, 2560), (13312, 2560),
                                 (200, 256)])
@pytest.mark.parametrize("M", [1, 2, 4, 8, 16, 64])
def test_w8g_gemm_vs_fp32_truth(cuda, N, K, M):
    g = torch.Generator(device="cpu").manual_seed(N + K + M)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    q, s = w8_ref.w8_quant(w)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    y = ops.w8g_gemm(x.to(cuda), q.to(cuda), s.to(cuda), 0)
    truth = x.float() @ w8_ref.w8g_dequant(q, s).T
    err = ((y.float().cpu() - truth).norm() / truth.norm()).item()
    assert err < 4e-3, err
    assert torch.equal(y, ops.w8g_gemm(x.to(cuda), q.to(cuda), s.to(cuda), 0)), "deterministic"


def test_w8g_strided_rows_and_group64(cuda):
    g = torch.Generator(device="cpu").manual_seed(1)
    w = (torch.randn(512, 192, generator=g) * 0.02).to(torch.bfloat16)
    q, s = w8_ref.w8_quant(w)                                   # K % 128 != 0 -> group 64
    assert s.shape[1] == 3
    xb = torch.randn(5, 256, generator=g).to(torch.bfloat16)
    x = xb.to(cuda)[:, :192]                                    # row stride 256
    y = ops.w8g_gemm(x, q.to(cuda), s.to(cuda), 0)
    truth = xb[:, :192].float() @ w8_ref.w8g_dequant(q, s).T
    assert ((y.float().cpu() - truth).norm() / truth.norm()).item() < 4e-3


@pytest.mark.parametrize("M", [3, 12])
def test_w8g_decode_group64_and_token_range(cuda, M):
    """The decode kernel (M <= 16, K % 128 == 0) with 64-k groups (a scale per half stage), a row stride above K,
    a zero token, a token scaled by 4096 and one whose first half is scaled by 2^-20 (the per-(token, 64-k) fp16
    exponent): within the reference's rel-L2 bound, and elementwise within bf16 rounding of the exact-product sum
    plus an fp32 summation allowance."""
    g = torch.Generator(device="cpu").manual_seed(7 + M)
    N, K = 1024, 2048
    q = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
    s = (torch.rand(N, K // 64, generator=g) * 1e-3 + 1e-4).to(torch.bfloat16)
    xb = torch.randn(M, K + 64, generator=g)
    xb[0] = 0.0
    xb[1] *= 4096.0
    xb[2, :K // 2] *= 2.0 ** -20
    xb = xb.to(torch.bfloat16)
    y = ops.w8g_gemm(xb.to(cuda)[:, :K], q.to(cuda), s.to(cuda), 0).float().cpu()
    deq = q.double() * s.double().repeat_interleave(64, dim=1)
    xd = xb[:, :K].double()
    truth = xd @ deq.T
    assert ((y - truth).norm() / truth.norm()).item() < 4e-3
    assert bool((y[0] == 0).all())
    allowance = 2.0 ** -8 * truth.abs() + 2.0 ** -16 * (xd.abs() @ deq.abs().T)
    assert bool(((y - truth).abs() <= allowance).all())
    assert ops.w8g_take_status() == 0


def test_w8g_unpack_exact(cuda):
    g = torch.Generator(device="cpu").manual_seed(2)
    w = (torch.randn(300, 1024, generator=g) * 0.02).to(torch.bfloat16)
    q, s = w8_ref.w8_quant(w)
    out = torch.empty(300, 1024, dtype=torch.bfloat16, device=cuda)
    ops.w8g_unpack(q.to(cuda), s.to(cuda), out)
    assert torch.equal(out.cpu(), w8_ref.w8g_dequant(q, s).to(torch.bfloat16))


@pytest.mark.parametrize("N", synthetic.W8A8_N)
@pytest.mark.parametrize("M", synthetic.W8A8_M)
def test_w8a8_bit_exact(cuda, N, M):
    K = synthetic.W8A8_K
    q, sw = synthetic.make_w8a8(N, K, seed=N)
    x = synthetic.make_w8a8_tokens(M, K, seed=M)
    xq = torch.empty(16 * K, dtype=torch.int8, device=cuda)
    sx = torch.empty(M, dtype=torch.float32, device=cuda)
    acc = torch.empty(M, N, dtype=torch.int32, device=cuda)
    qk = formats.repack_w8(q.to(cuda))
    y = ops.w8a8_gemm(x.to(cuda), qk, sw.to(cuda), xq=xq, sx=sx, acc_out=acc)
    torch.cuda.synchronize()
    yr, accr, xqr, sxr = w8_ref.w8a8_ref(x, q, sw)
    assert torch.equal(sx.cpu(), sxr)
    # packed operand: element (t, k) at (k / 16) * 256 + t * 16 + k % 16, rows t >= M zero
    xq16 = xq.view(K // 16, 16, 16).permute(1, 0, 2).reshape(16, K).cpu()
    assert torch.equal(xq16[:M], xqr)
    assert not xq16[M:].any()
    assert torch.equal(acc.cpu().long(), accr)
    assert torch.equal(y.cpu(), yr)
    assert ops.w8a8_take_status() == 0


def test_w8a8_zero_row_and_outliers(cuda):
    K, N = 2048, 2048
    q, sw = synthetic.make_w8a8(N, K, seed=9)
    x = synthetic.make_w8a8_tokens(4, K, seed=9)
    x[1] = 0
    x[2, 17] = 3000.0
    acc = torch.empty(4, N, dtype=torch.int32, device=cuda)
    y = ops.w8a8_gemm(x.to(cuda), formats.repack_w8(q.to(cuda)), sw.to(cuda), acc_out=acc)
    yr, accr, _, _ = w8_ref.w8a8_ref(x, q, sw)
    assert torch.equal(acc.cpu().long(), accr) and torch.equal(y.cpu(), yr)
    assert (y[1] == 0).all()


def test_w8_repack_matches_torch_and_round_trips(cuda):
    q, _ = synthetic.make_w8a8(384, 640, seed=5)
    qk = formats.repack_w8(q.to(cuda))
    assert torch.equal(qk.cpu(), formats.repack_w8_torch(q))
    assert torch.equal(formats.unpack_w8(qk).cpu(), q)


def test_w8a8_rejects_large_m(cuda):
    q, sw = synthetic.make_w8a8(256, 256, seed=6)
    x = synthetic.make_w8a8_tokens(17, 256, seed=6)
    with pytest.raises(RuntimeError, match="M must be"):
        ops.w8a8_gemm(x.to(cuda), formats.repack_w8(q.to(cuda)), sw.to(cuda))


@pytest.mark.parametrize("N,K,M", [(384, 640, 3), (128, 16384, 2), (1280, 4096, 16), (256, 128, 1),
                                   (16384, 2048, 4), (2560, 8192, 5)])
def test_w8a8_shapes_split_k(cuda, N, K, M):
    """The stream-K partition: odd k-tile counts, the largest K (128 runs share one tile), runs that cross tile
    boundaries with full M, runs longer than a tile, a single tile."""
    q, sw = synthetic.make_w8a8(N, K, seed=N + K)
    x = synthetic.make_w8a8_tokens(M, K, seed=M + 7)
    acc = torch.empty(M, N, dtype=torch.int32, device=cuda)
    y = ops.w8a8_gemm(x.to(cuda), formats.repack_w8(q.to(cuda)), sw.to(cuda), acc_out=acc)
    yr, accr, _, _ = w8_ref.w8a8_ref(x, q, sw)
    assert torch.equal(acc.cpu().long(), accr)
    assert torch.equal(y.cpu(), yr)
    assert ops.w8a8_take_status() == 0


def test_w8g_rpw_force_and_forbid_bits(cuda):
    """rpw 0x100 forces the tensor-memory kernel and 0x200 forbids it (qf_w8g.cu:315-318): both paths within the
    reference's bound of the fp32 truth and each deterministic; the default path at a decode shape is the forbidden
    one's (the register-fragment kernel); forbidding where only the tensor-memory kernel fits, or both bits, fails."""
    g = torch.Generator(device="cpu").manual_seed(11)
    w = (torch.randn(2048, 2048, generator=g) * 0.02).to(torch.bfloat16)
    q, s = w8_ref.w8_quant(w)
    truth_of = lambda x: x.float() @ w8_ref.w8g_dequant(q, s).T
    qd, sd = q.to(cuda), s.to(cuda)
    x = torch.randn(4, 2048, generator=g).to(torch.bfloat16)
    xd = x.to(cuda)
    ys = {r: ops.w8g_gemm(xd, qd, sd, r) for r in (0, 0x100, 0x200, 0x104)}
    for r, y in ys.items():
        truth = truth_of(x)
        assert ((y.float().cpu() - truth).norm() / truth.norm()).item() < 4e-3, r
        assert torch.equal(y, ops.w8g_gemm(xd, qd, sd, r)), r
    assert torch.equal(ys[0], ys[0x200]) and torch.equal(ys[0x100], ys[0x104])
    x32 = torch.randn(32, 2048, generator=g).to(torch.bfloat16).to(cuda)
    with pytest.raises(RuntimeError, match="forbids the tensor-memory kernel"):
        ops.w8g_gemm(x32, qd, sd, 0x200)
    with pytest.raises(RuntimeError, match="cannot both"):
        ops.w8g_gemm(xd, qd, sd, 0x300)
    assert ops.w8g_take_status() == 0


def test_w8linear_equals_w8g_gemm(cuda):
    """ops.W8Linear (the weight's checks and C-ABI arguments made once) launches what w8g_gemm launches: the same bits
    for several M, group 128 and 64, a caller-given out, a strided x, and a second stream (its own fixup buffer)."""
    g = torch.Generator(device="cpu").manual_seed(12)
    for N, K in ((2048, 2048), (12288, 2560), (264, 192), (200, 256)):   # (264, 192): group 64
        q, s = w8_ref.w8_quant((torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16))
        qd, sd = q.to(cuda), s.to(cuda)
        lin = ops.W8Linear(qd, sd)
        for M in (1, 4, 16, 64):
            x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(cuda)
            assert torch.equal(lin(x), ops.w8g_gemm(x, qd, sd))
        out = torch.empty(4, N, dtype=torch.bfloat16, device=cuda)
        xs = torch.randn(4, 2 * K, generator=g).to(torch.bfloat16).to(cuda)[:, :K]
        assert lin(xs, out) is out and torch.equal(out, ops.w8g_gemm(xs, qd, sd))
        side = torch.cuda.Stream(cuda)
        with torch.cuda.stream(side):
            y2 = lin(xs)
        side.synchronize()
        assert torch.equal(y2, out)
    with pytest.raises(RuntimeError, match="x must be"):
        lin(torch.randn(2, 128, device=cuda).to(torch.bfloat16))
    with pytest.raises(RuntimeError, match="out must be"):
        lin(torch.randn(2, 256, device=cuda).to(torch.bfloat16), torch.empty(3, 200, dtype=torch.bfloat16, device=cuda))
    assert ops.w8g_take_status() == 0


def test_w8a8linear_equals_w8a8_gemm_and_oracle(cuda):
    """ops.W8A8Linear (the weight's checks and arguments made once, per-stream scratch reused) gives the bits of
    w8a8_gemm and of the oracle: N with and without the fixup buffer (N % 128), several M in a row on one scratch,
    a caller-given out, and a second stream."""
    for N, K in ((2048, 2048), (12288, 2048), (384, 640)):
        q, sw = synthetic.make_w8a8(N, K, seed=N + 1)
        lin = ops.W8A8Linear(formats.repack_w8(q.to(cuda)), sw.to(cuda))
        for M in (1, 16, 4, 10):
            x = synthetic.make_w8a8_tokens(M, K, seed=M + N)
            y = lin(x.to(cuda))
            yr, _, _, _ = w8_ref.w8a8_ref(x, q, sw)
            assert torch.equal(y.cpu(), yr), (N, M)
            assert torch.equal(y, ops.w8a8_gemm(x.to(cuda), lin.q, lin.sw))
        out = torch.empty(M, N, dtype=torch.bfloat16, device=cuda)
        side = torch.cuda.Stream(cuda)
        side.wait_stream(torch.cuda.current_stream(cuda))
        with torch.cuda.stream(side):
            lin(x.to(cuda), out)
        side.synchronize()
        assert torch.equal(out.cpu(), yr)
    with pytest.raises(RuntimeError, match="x must be"):
        lin(torch.randn(2, 128, device=cuda).to(torch.bfloat16))
    assert ops.w8a8_take_status() == 0
