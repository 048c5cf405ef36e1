// Shared device helpers for the sm_100a decode-path kernels: bf16 bit helpers, mbarrier + bulk-copy (TMA engine)
// wrappers, bounded waits, and the C-ABI error plumbing.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "qwenfast_b200.h"

namespace qf {

// ------------------------------------------------------------------------------------------------ host side
// Thread-local last-error text for qf_last_error(); every entry point returns a QF_* status code.
void set_error(const char* fmt, ...);
int cuda_status(cudaError_t e, const char* what);
int sm_count(int device);
// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device); later calls only read a cache, so
// launches made during CUDA-graph capture issue no configuration API calls.
cudaError_t ensure_smem_attr(const void* func, int bytes);
// W8A8 contraction on tcgen05 (w8a8tc.cu), launched under PDL of the quantisation kernel: xq = its packed token
// operand ([K / 16][16 tokens][16 B], tokens >= M zero), sx its scales; q in the kernel layout of qf_w8_repack;
// fix = the zero-kept split-K fixup buffer of w8a8_fixup_elems(N) int32.
size_t w8a8_fixup_elems(int N);
cudaError_t launch_w8a8_tc(const int8_t* xq, const float* sx, const int8_t* q, const float* sw, void* y, int ldy,
                           int32_t* acc_out, int32_t* fix, int M, int N, int K, cudaStream_t st);
cudaError_t w8a8_tc_take_status(unsigned* out);
// canonical [N, K] int8 <-> the W8A8 kernel layout (unpack = 1 for the inverse)
cudaError_t launch_w8_repack(const int8_t* src, int8_t* dst, int N, int K, int unpack, cudaStream_t st);
// cuTensorMapEncodeTiled through the runtime's driver entry point (resolved once per process)
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
cudaError_t encode_tiled_fn(EncodeTiled* fn);

#define QF_REQUIRE(cond, ...)                                  \
    do {                                                       \
        if (!(cond)) {                                         \
            ::qf::set_error(__VA_ARGS__);                      \
            return QF_ERR_INVALID_ARGUMENT;                    \
        }                                                      \
    } while (0)

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// Launch with the programmatic-stream-serialization attribute (PDL) when requested.
template <typename Kern, typename... Args>
cudaError_t launch_ex(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}
// The same as a cooperative launch: every CTA of the grid is resident at once (the runtime refuses a grid that cannot
// be, with cudaErrorCooperativeLaunchTooLarge), as grid-wide barriers require. Composes with PDL (measured on B200).
template <typename Kern, typename... Args>
cudaError_t launch_coop(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    attr[1].id = cudaLaunchAttributeCooperative;
    attr[1].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// ---------------------------------------------------------------------------------------------- device side
__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }
__device__ __forceinline__ float bf16_bits(uint16_t b) { return __uint_as_float(((uint32_t)b) << 16); }
__device__ __forceinline__ float bf16r(float v) { return __bfloat162float(__float2bfloat16(v)); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t ld_volatile(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// ---- mbarrier (CTA scope)
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_n(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
// 16-byte asynchronous global -> shared copy (cp.async, L2 only); src_bytes 0 writes zeros and reads nothing.
// Fences and release arrives of the issuing thread do not wait for it; cp_async_wait_all does.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Raise the phase's expected transaction bytes without arriving (the arrive comes later, e.g. after a dependency).
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Non-blocking probe of an mbarrier phase.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// try_wait that suspends the thread until the phase completes or about `hint_ns` passed, so that a waiting warp
// does not keep re-issuing barrier probes (which share the SM's memory-instruction queue with the working warps).
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}
// Bounded wait on an mbarrier phase. Returns false (and leaves the phase unconsumed) once about `limit_ns` passed.
// The bound is counted in SM cycles (clock64 reads are cheap; %globaltimer reads are not), 2 per ns: at most
// 2 x limit_ns of wall time at clocks of 1 GHz and more.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    const long long lim = (long long)(2 * limit_ns);
    while (!mbar_try_wait_hint(bar, parity, 100000u)) {
        if (clock64() - t0 > lim) return false;
    }
    return true;
}

// ---- bulk copies (TMA engine, untiled): global -> shared, completion counted on an mbarrier.
// Both addresses 16-byte aligned, size a multiple of 16 bytes.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
// ---- tensor copies (TMA engine, tiled): global -> shared through a tensor map (a __grid_constant__ parameter)
// 2-D box at (x, y) (x in elements, x * element size a multiple of 16 bytes); rows outside the tensor read zeros.
__device__ __forceinline__ void tma_tile_2d(void* dst, const void* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
// Four rows y0..y3 (any order) of a map whose box is one row high, columns from x: the rows land back to back.
__device__ __forceinline__ void tma_gather4(void* dst, const void* map, int x, int y0, int y1, int y2, int y3,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
        "%4, %5, %6}], [%7];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y0), "r"(y1), "r"(y2), "r"(y3), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
// Order this thread's earlier generic-proxy accesses (and those it acquired) before its later async-proxy ones.
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async;" ::: "memory"); }
// The same, for global memory only: orders this thread's generic-proxy view of global memory (e.g. rows acquired from
// other CTAs) before its later async-proxy (bulk / tensor copy) reads of global memory.
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// ---- named barrier over a subset of warps (non-.aligned form: callers may arrive from divergent code)
__device__ __forceinline__ void named_bar(int id, int threads) {
    asm volatile("barrier.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
// Named barrier that also ANDs a predicate over its threads: every thread gets the same result.
__device__ __forceinline__ bool named_bar_and(int id, int threads, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "barrier.red.and.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(id), "r"(threads)
        : "memory");
    return r != 0;
}
// Arrive on a named barrier without waiting for it (the producer side of a one-way hand-off).
__device__ __forceinline__ void named_bar_arrive(int id, int threads) {
    asm volatile("barrier.arrive %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---- tensor-core fragment op (register-sourced A): D += A(16x16 bf16) * B(16x8 bf16), fp32 accumulate
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The same with a zero accumulator input: D = A(16x16 bf16) * B(16x8 bf16) (starts an accumulation chain).
__device__ __forceinline__ void mma_bf16_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                           uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}

// The same two for fp16 operands: D (+)= A(16x16 f16) * B(16x8 f16), fp32 accumulate.
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_f16_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}

// int4 word -> four bf16x2 of (code - 8). The word's nibbles hold k = [0, 2, 4, 6, 1, 3, 5, 7] of eight
// consecutive k (kernel layout), so the pairs come out in natural order: (k0,k1) (k2,k3) (k4,k5) (k6,k7).
// (0x4300 | n) is the bf16 value 128 + n; subtracting 136 leaves n - 8, exactly.
__device__ __forceinline__ void dequant_w4(uint32_t q, uint32_t (&p)[4]) {
    const uint32_t MASK = 0x000F000Fu, MAGIC = 0x43004300u, BIAS = 0x43084308u;   // bf16 136.0 in both halves
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint32_t v;
        const uint32_t s = q >> (4 * i);
        asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(v) : "r"(s), "r"(MASK), "r"(MAGIC));   // (s & MASK) | MAGIC
        __nv_bfloat162 r = __hsub2(*reinterpret_cast<__nv_bfloat162*>(&v),
                                   *reinterpret_cast<const __nv_bfloat162*>(&BIAS));
        p[i] = *reinterpret_cast<uint32_t*>(&r);
    }
}

}  // namespace qf

namespace qf {
// ------------------------------------------------------------------------------------ tcgen05 / TMEM (sm_100a)
// Tensor memory is allocated per CTA by one full warp; the address written to shared memory is (lane << 16) | column.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// 32x32b shape: thread i of the warp accesses lane (taddr.lane + i); the warp's lane base is 32 * (warp % 4).
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
                 "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
        "[%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}
// Shared-memory matrix descriptor, K-major, no swizzle: 8-row core matrices of 16-byte rows; lbo = byte distance
// between the two 16-byte k-chunks of one k16 step, sbo = byte distance between 8-row groups; version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc(const void* p, uint32_t lbo, uint32_t sbo) {
    uint64_t d = (uint64_t)((smem_u32(p) >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    return d;
}
// Instruction descriptor kind::f16: bf16 A and B (K-major), fp32 D, M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// D[tmem] (+)= A[tmem] * B[smem]^T, issued by one thread.
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
        "r"(a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// One arrive on `bar` once every tcgen05.mma this thread issued before has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// int4 word -> four bf16x2 of the biased codes 128 + code (one lop3 each, exact); the caller removes the bias
// (128 + the zero point 8 = 136 times the k-sum of the other operand).
__device__ __forceinline__ void biased_w4(uint32_t q, uint32_t* p) {
    const uint32_t MASK = 0x000F000Fu, MAGIC = 0x43004300u;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t s = q >> (4 * i);
        asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(p[i]) : "r"(s), "r"(MASK), "r"(MAGIC));
    }
}
// Instruction descriptor kind::f16 with fp16 A and B (K-major), fp32 D, M x N.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// bf16 pair -> fp16 pair of the values times `mul` (a power of two); exact when the products are fp16 values.
__device__ __forceinline__ uint32_t bf16x2_to_f16x2_scaled(uint32_t v, float mul) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(__uint_as_float(v & 0xFFFF0000u) * mul), "f"(__uint_as_float(v << 16) * mul));
    return r;
}
// int4 word -> four bf16x2 of the signed codes code - 8 (lop3 to 128 + code, then one bf16x2 subtract; exact).
__device__ __forceinline__ void signed_w4(uint32_t q, uint32_t* p) {
    biased_w4(q, p);
#pragma unroll
    for (int i = 0; i < 4; ++i) asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(p[i]) : "r"(p[i]), "r"(0x43084308u));
}
}  // namespace qf

namespace qf {
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr)
                 : "memory");
}
}  // namespace qf

namespace qf {
// Bring [src, src + bytes) into L2 ahead of its use (bulk prefetch through the copy engine; nothing is written to
// shared memory). src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// NVFP4 (e2m1 codes with one E4M3 scale per 16 k) -> bf16, exactly.
// An E4M3 byte's fields placed at the low end of a bf16's exponent and mantissa (sign at bit 15, the 7 exponent and
// mantissa bits at 4..10) read as a bf16 of 2^-120 times its value -- a bf16 subnormal for an E4M3 subnormal -- so one
// multiply by 2^120 gives the scale (exact). The result is the scale in both halves.
__device__ __forceinline__ uint32_t e4m3_scale_bf16x2(uint32_t b) {
    const uint32_t bits = ((b & 0x80u) << 8) | ((b & 0x7Fu) << 4);
    uint32_t s;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(s) : "r"(bits | (bits << 16)), "r"(0x7B807B80u));   // 2^120
    return s;
}
// One word of eight e2m1 codes (nibble i = k index [0,2,4,6,1,3,5,7][i], the int4 kernel layout) -> four bf16x2 of
// the weights code * scale (scale: a bf16x2 from e4m3_scale_bf16x2), pair j = k 2j (low half), 2j + 1 (high half).
// The code's sign goes to bit 15 and its exponent and mantissa bits to 6..8: a bf16 of 2^-126 times the code's value
// (0.5 a bf16 subnormal); times 2^126, then times the scale -- both exact (e2m1 x E4M3 has at most 6 significant
// bits).
__device__ __forceinline__ void nvfp4_w4(uint32_t q, uint32_t scale, uint32_t* p) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t a = (6 - 4 * j) >= 0 ? (q << (6 - 4 * j)) : (q >> (4 * j - 6));   // exponent, mantissa -> 6..8
        const uint32_t b = q << (12 - 4 * j);                                              // sign -> 15
        const uint32_t bits = (a & 0x01C001C0u) | (b & 0x80008000u);
        uint32_t v;
        asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(v) : "r"(bits), "r"(0x7E807E80u));   // 2^126
        asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(p[j]) : "r"(v), "r"(scale));
    }
}
}  // namespace qf
