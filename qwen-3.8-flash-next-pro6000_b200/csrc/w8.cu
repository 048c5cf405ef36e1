// INT8 dense projections for decode/verify rows (1..64 tokens): the small kernels around the tensor-core GEMMs.
//
// w8g_unpack (reference serve/qwenfast/qf_w8g.cu:338-351): w = bf16(q * s), the group-scaled int8 weight expanded to
//   bf16 (the reference's decline path and the shared-expert conversion use it). The W8A16 GEMM itself is
//   w8g_tc.cu.
// w8a8 (synthetic config 3, no reference kernel): the per-token quantisation kernel (sx = absmax/127,
//   xq = rint(x / sx)) that writes the packed token operand of the tcgen05 kind::i8 GEMM in w8a8tc.cu, and the host
//   entry points of that GEMM.
#include "qf_common.cuh"

namespace {

using qf::bf16_bits;

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

}  // namespace

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
