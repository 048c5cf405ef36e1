// INT8 dense projections for decode/verify rows (1..64 tokens).
//
// w8g (W8A16, reference serve/qwenfast/qf_w8g.cu): y = x @ (q * s)^T with int8 weights and one bf16 scale per group
//   of 128 (or 64) k. Weights are the A operand of mma.m16n8k16 (int8 -> bf16 is exact, |q| <= 127), tokens the B
//   operand; the fp32 partial of each 64-k chunk is scaled by its group scale.
// w8a8 (synthetic config 3, no reference kernel): per-token activation scale sx = absmax/127, xq = rint(x / sx),
//   exact int32 accumulation on mma.m16n8k32.s8, y = bf16((float(acc) * sx) * sw).
//
// Work split (both GEMMs): a CTA owns one 16-row weight tile; its 8 warps split K, each warp requests its whole
// slice (16-byte loads, streaming cache hint) before waiting on the previous kernel, and the per-warp partials are
// reduced in a fixed warp order through shared memory. Inside a 64-k chunk thread t owns k = 16t .. 16t+15 of
// weight rows g and g+8 and of token g, a permutation of k applied to both operands, so the product is the same
// sum and every load is a 16-byte vector.
#include "qf_common.cuh"

namespace {

using qf::bf16_bits;
constexpr int W8_WARPS = 8;
constexpr int W8_THREADS = W8_WARPS * 32;
constexpr int CB = 4;   // 64-k chunks per warp held in registers at once

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ uint32_t u4w(const uint4& v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }

// 4 int8 (one word) -> two bf16x2 words (bytes 0,1 -> lo; bytes 2,3 -> hi), exact.
// Each byte b is placed in the mantissa of 2^23 (float 8388608 + (b ^ 0x80)); subtracting 8388608 + 128 gives q.
// q has at most 7 significant bits, so the upper half of the fp32 pattern is q in bf16 exactly.
__device__ __forceinline__ void i8x4_bf16(uint32_t w, uint32_t& lo, uint32_t& hi) {
    const uint32_t u = w ^ 0x80808080u;
    const float f0 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440)) - 8388736.f;
    const float f1 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7441)) - 8388736.f;
    const float f2 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7442)) - 8388736.f;
    const float f3 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7443)) - 8388736.f;
    lo = __byte_perm(__float_as_uint(f0), __float_as_uint(f1), 0x7632);
    hi = __byte_perm(__float_as_uint(f2), __float_as_uint(f3), 0x7632);
}

// ------------------------------------------------------------------------------------------------ W8A16 (w8g)
template <int NT>
__global__ void __launch_bounds__(W8_THREADS)
    w8g_kernel(const __nv_bfloat16* __restrict__ x, int ldx, const int8_t* __restrict__ q,
               const uint16_t* __restrict__ s, __nv_bfloat16* __restrict__ y, int ldy, int M, int N, int K, int G) {
    __shared__ float red[W8_WARPS][16][NT * 8 + 1];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    const int row0 = blockIdx.x * 16;
    const size_t ra = (size_t)min(row0 + g, N - 1), rb = (size_t)min(row0 + g + 8, N - 1);
    const int nch = K / 64, cpw = (nch + W8_WARPS - 1) / W8_WARPS;
    const int c0 = warp * cpw, c1 = min(c0 + cpw, nch);
    const int NG = K / G;
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
    bool waited = false;
    for (int cb = c0; cb < c1; cb += CB) {
        uint4 wa[CB], wb[CB];
        uint16_t sa[CB], sb[CB];
#pragma unroll
        for (int i = 0; i < CB; ++i) {
            const int c = cb + i;
            if (c < c1) {
                wa[i] = ldg_stream(q + ra * K + 64 * c + 16 * t);
                wb[i] = ldg_stream(q + rb * K + 64 * c + 16 * t);
                sa[i] = __ldg(s + ra * NG + (64 * c) / G);
                sb[i] = __ldg(s + rb * NG + (64 * c) / G);
            }
        }
        if (!waited) { qf::pdl_wait(); waited = true; }
#pragma unroll
        for (int i = 0; i < CB; ++i) {
            const int c = cb + i;
            if (c >= c1) break;
            uint32_t A0[4], A1[4], A2[4], A3[4];   // per mma step j: a0..a3
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint32_t lo, hi;
                i8x4_bf16(u4w(wa[i], j), lo, hi);
                A0[j] = lo; A2[j] = hi;
                i8x4_bf16(u4w(wb[i], j), lo, hi);
                A1[j] = lo; A3[j] = hi;
            }
            const float fa = bf16_bits(sa[i]), fb = bf16_bits(sb[i]);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const int tok = nt * 8 + g;
                uint4 x0 = make_uint4(0, 0, 0, 0), x1 = make_uint4(0, 0, 0, 0);
                if (tok < M) {
                    const uint4* xp = reinterpret_cast<const uint4*>(x + (size_t)tok * ldx + 64 * c + 16 * t);
                    x0 = __ldg(xp);
                    x1 = __ldg(xp + 1);
                }
                float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint4& xv = j < 2 ? x0 : x1;
                    qf::mma_bf16(d, A0[j], A1[j], A2[j], A3[j], u4w(xv, (j & 1) * 2), u4w(xv, (j & 1) * 2 + 1));
                }
                acc[nt][0] = fmaf(d[0], fa, acc[nt][0]);
                acc[nt][1] = fmaf(d[1], fa, acc[nt][1]);
                acc[nt][2] = fmaf(d[2], fb, acc[nt][2]);
                acc[nt][3] = fmaf(d[3], fb, acc[nt][3]);
            }
        }
    }
    if (!waited) qf::pdl_wait();
    qf::pdl_launch_dependents();
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        red[warp][g][nt * 8 + 2 * t] = acc[nt][0];
        red[warp][g][nt * 8 + 2 * t + 1] = acc[nt][1];
        red[warp][g + 8][nt * 8 + 2 * t] = acc[nt][2];
        red[warp][g + 8][nt * 8 + 2 * t + 1] = acc[nt][3];
    }
    __syncthreads();
    for (int idx = tid; idx < 16 * M; idx += W8_THREADS) {
        const int r = idx & 15, m = idx >> 4;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < W8_WARPS; ++w) v += red[w][r][m];
        if (row0 + r < N) y[(size_t)m * ldy + row0 + r] = __float2bfloat16(v);
    }
}

__global__ void w8g_unpack_kernel(const int8_t* __restrict__ q, const uint16_t* __restrict__ s,
                                  __nv_bfloat16* __restrict__ w, long long total8, int K, int G) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total8; i += (long long)gridDim.x * blockDim.x) {
        const long long e = i * 8, row = e / K;
        const int k = (int)(e - row * K);
        const float sc = bf16_bits(s[row * (K / G) + k / G]);
        const uint2 v = *reinterpret_cast<const uint2*>(q + e);
        uint4 o;
        uint32_t* op = reinterpret_cast<uint32_t*>(&o);
        const uint32_t vv[2] = {v.x, v.y};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const float a = (float)(int8_t)((vv[h] >> (16 * j)) & 0xFF) * sc;
                const float b = (float)(int8_t)((vv[h] >> (16 * j + 8)) & 0xFF) * sc;
                __nv_bfloat162 r = __floats2bfloat162_rn(a, b);
                op[2 * h + j] = *reinterpret_cast<uint32_t*>(&r);
            }
        }
        *reinterpret_cast<uint4*>(w + e) = o;
    }
}

// ------------------------------------------------------------------------------------------------ W8A8
// One CTA per token row of the 16-token operand: absmax, sx = absmax / 127 (1 when the row is all zero),
// xq = rint(x / sx) clamped, stored packed as the tensor-core operand of the W8A8 kernel: element (t, k) at
// (k / 16) * 256 + t * 16 + k % 16 ([16-byte k chunk][16 tokens][16 B]); rows t >= M are written as zeros.
__global__ void __launch_bounds__(256) w8a8_quant_kernel(const __nv_bfloat16* __restrict__ x, int ldx, int M, int K,
                                                         int8_t* __restrict__ xqp, float* __restrict__ sx) {
    __shared__ float wmax[8];
    const int m = blockIdx.x, tid = threadIdx.x;
    // the W8A8 GEMM that follows may become resident now and prefetch its weights; it reads xq / sx only after
    // its own griddepcontrol.wait, i.e. after this grid has completed
    qf::pdl_launch_dependents();
    qf::pdl_wait();
    if (m >= M) {
        for (int k = tid * 8; k < K; k += 256 * 8)
            *reinterpret_cast<uint2*>(xqp + (size_t)(k >> 4) * 256 + m * 16 + (k & 15)) = make_uint2(0u, 0u);
        return;
    }
    const __nv_bfloat16* xr = x + (size_t)m * ldx;
    float mx = 0.f;
    for (int k = tid * 8; k < K; k += 256 * 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(xr + k);
        const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) mx = fmaxf(mx, fmaxf(fabsf(qf::bf16_lo(vv[j])), fabsf(qf::bf16_hi(vv[j]))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((tid & 31) == 0) wmax[tid >> 5] = mx;
    __syncthreads();
    float amax = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) amax = fmaxf(amax, wmax[w]);
    const float scale = amax > 0.f ? __fdiv_rn(amax, 127.f) : 1.f;
    if (tid == 0) sx[m] = scale;
    for (int k = tid * 8; k < K; k += 256 * 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(xr + k);
        const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
        uint32_t packed[2] = {0u, 0u};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int a = max(-127, min(127, __float2int_rn(__fdiv_rn(qf::bf16_lo(vv[j]), scale))));
            const int b = max(-127, min(127, __float2int_rn(__fdiv_rn(qf::bf16_hi(vv[j]), scale))));
            packed[j >> 1] |= ((uint32_t)(a & 0xFF) | ((uint32_t)(b & 0xFF) << 8)) << (16 * (j & 1));
        }
        *reinterpret_cast<uint2*>(xqp + (size_t)(k >> 4) * 256 + m * 16 + (k & 15)) = make_uint2(packed[0], packed[1]);
    }
}

template <int NT>
cudaError_t launch_w8g(const void* x, int ldx, const int8_t* q, const void* s, void* y, int ldy, int M, int N, int K,
                       int G, bool pdl, cudaStream_t st) {
    return qf::launch_ex(w8g_kernel<NT>, dim3((N + 15) / 16), dim3(W8_THREADS), 0, st, pdl,
                         static_cast<const __nv_bfloat16*>(x), ldx, q, static_cast<const uint16_t*>(s),
                         static_cast<__nv_bfloat16*>(y), ldy, M, N, K, G);
}

}  // namespace

extern "C" int qf_w8g_gemm(const void* x, int64_t ldx, const int8_t* q, const void* s, void* y, int64_t ldy, int M,
                           int N, int K, int group, int rpw, int pdl, qf_stream_t stream) {
    (void)rpw;
    QF_REQUIRE(x && q && s && y, "w8g_gemm: null pointer argument");
    QF_REQUIRE(M >= 1 && M <= QF_MAX_TOKENS, "w8g_gemm: M must be in [1, %d], got %d", QF_MAX_TOKENS, M);
    QF_REQUIRE(N >= 1 && K >= 64 && K % 64 == 0, "w8g_gemm: K must be a multiple of 64, got %d", K);
    QF_REQUIRE(group == 128 || group == 64, "w8g_gemm: group must be 128 or 64, got %d", group);
    QF_REQUIRE(K % group == 0, "w8g_gemm: K must be a multiple of the group size");
    QF_REQUIRE(ldx >= K && ldx % 8 == 0 && qf::aligned(x, 16), "w8g_gemm: x needs a row stride %% 8 == 0 and 16-byte alignment");
    QF_REQUIRE(ldy >= N && qf::aligned(q, 16), "w8g_gemm: bad y stride or unaligned q");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int nt = (M + 7) / 8;
    cudaError_t e;
    switch (nt) {
        case 1: e = launch_w8g<1>(x, (int)ldx, q, s, y, (int)ldy, M, N, K, group, pdl != 0, st); break;
        case 2: e = launch_w8g<2>(x, (int)ldx, q, s, y, (int)ldy, M, N, K, group, pdl != 0, st); break;
        case 3:
        case 4: e = launch_w8g<4>(x, (int)ldx, q, s, y, (int)ldy, M, N, K, group, pdl != 0, st); break;
        default: e = launch_w8g<8>(x, (int)ldx, q, s, y, (int)ldy, M, N, K, group, pdl != 0, st); break;
    }
    return qf::cuda_status(e, "w8g_gemm: launch");
}

extern "C" int qf_w8g_unpack(const int8_t* q, const void* s, void* w, int64_t rows, int K, int group,
                             qf_stream_t stream) {
    QF_REQUIRE(q && s && w, "w8g_unpack: null pointer argument");
    QF_REQUIRE(rows >= 0 && K % 8 == 0 && (group == 128 || group == 64) && K % group == 0, "w8g_unpack: bad shape");
    const long long total8 = rows * (long long)K / 8;
    if (total8 == 0) return QF_OK;
    long long blocks = (total8 + 255) / 256;
    if (blocks > 65535LL * 16) blocks = 65535LL * 16;
    w8g_unpack_kernel<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        q, static_cast<const uint16_t*>(s), static_cast<__nv_bfloat16*>(w), total8, K, group);
    return qf::cuda_status(cudaGetLastError(), "w8g_unpack: launch");
}

extern "C" int qf_w8a8_gemm(const void* x, int64_t ldx, const int8_t* q, const float* sw, void* y, int64_t ldy, int M,
                            int N, int K, int8_t* xq, float* sx, int32_t* acc, int32_t* acc_out, int pdl,
                            qf_stream_t stream) {
    QF_REQUIRE(x && q && sw && y && xq && sx && acc, "w8a8_gemm: null pointer argument");
    QF_REQUIRE(M >= 1 && M <= 16, "w8a8_gemm: M must be in [1, 16], got %d", M);
    QF_REQUIRE(N >= 128 && N % 128 == 0, "w8a8_gemm: N must be a multiple of 128, got %d", N);
    QF_REQUIRE(K >= 128 && K % 128 == 0 && K <= 16384, "w8a8_gemm: K must be a multiple of 128 in [128, 16384], got %d", K);
    QF_REQUIRE(ldx >= K && ldx % 8 == 0 && ldx <= INT32_MAX && qf::aligned(x, 16),
               "w8a8_gemm: x needs a row stride %% 8 == 0 and 16-byte alignment");
    QF_REQUIRE(ldy >= N && ldy <= INT32_MAX && qf::aligned(q, 16) && qf::aligned(xq, 16) && qf::aligned(acc, 16),
               "w8a8_gemm: bad y stride or unaligned q / xq / acc");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = qf::launch_ex(w8a8_quant_kernel, dim3(16), dim3(256), 0, st, pdl != 0,
                                  static_cast<const __nv_bfloat16*>(x), (int)ldx, M, K, xq, sx);
    if (e != cudaSuccess) return qf::cuda_status(e, "w8a8_gemm: quant launch");
    // tcgen05 kind::i8, stream-K over 16 KB weight tiles (w8a8tc.cu), under programmatic dependent launch of the
    // quantisation kernel: it becomes resident and requests its first weight tiles while that one runs
    e = qf::launch_w8a8_tc(xq, sx, q, sw, y, (int)ldy, acc_out, acc, M, N, K, st);
    return qf::cuda_status(e, "w8a8_gemm: launch");
}

extern "C" int qf_w8a8_fixup_elems(int N, int64_t* elems) {
    QF_REQUIRE(elems && N >= 128 && N % 128 == 0, "w8a8_fixup_elems: N must be a multiple of 128, got %d", N);
    *elems = (int64_t)qf::w8a8_fixup_elems(N);
    return QF_OK;
}

extern "C" int qf_w8_repack(const int8_t* q, int8_t* qk, int N, int K, qf_stream_t stream) {
    QF_REQUIRE(q && qk, "w8_repack: null pointer argument");
    QF_REQUIRE(N >= 128 && N % 128 == 0 && K >= 128 && K % 128 == 0, "w8_repack: need N %% 128 == 0 and K %% 128 == 0");
    return qf::cuda_status(qf::launch_w8_repack(q, qk, N, K, 0, reinterpret_cast<cudaStream_t>(stream)), "w8_repack: launch");
}

extern "C" int qf_w8_unpack(const int8_t* qk, int8_t* q, int N, int K, qf_stream_t stream) {
    QF_REQUIRE(q && qk, "w8_unpack: null pointer argument");
    QF_REQUIRE(N >= 128 && N % 128 == 0 && K >= 128 && K % 128 == 0, "w8_unpack: need N %% 128 == 0 and K %% 128 == 0");
    return qf::cuda_status(qf::launch_w8_repack(qk, q, N, K, 1, reinterpret_cast<cudaStream_t>(stream)), "w8_unpack: launch");
}

extern "C" int qf_w8a8_take_status(uint32_t* status) {
    QF_REQUIRE(status, "w8a8_take_status: null pointer argument");
    unsigned v = 0;
    const int rc = qf::cuda_status(qf::w8a8_tc_take_status(&v), "w8a8_take_status");
    *status = v;
    return rc;
}
