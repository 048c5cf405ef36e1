// MoE router for decode/verify batches (1..64 tokens): router GEMM + softmax + top-k + renormalise, one launch.
//
//   logits[t, e] = bf16(x[t] . w[e])          fp32 products and sums on the tensor cores
//   p[t, e]      = softmax_e(logits[t])        fp32, max-subtracted
//   ids[t]       = the k largest logits, lower expert id first among equal values
//   weights[t]   = p[t, ids] / sum(p[t, ids]) when renormalising (sum > 0), else p[t, ids]
// Selection semantics follow serve/qwenfast/qf_router.cu:3-6, 103-157 (NaN ranks as -1e30, -0 == +0).
//
// Layout of the work: a CTA owns 16 router rows (one m16 tile, experts as the A operand) and 16 warps split the
// hidden dimension; tokens are the n8 operand. Each warp requests its whole weight slice before waiting on the
// previous kernel (PDL), so the 2 MB weight stream overlaps the producer of x. Per-warp fp32 partials are summed
// in a fixed warp order through shared memory, so the logits do not depend on timing. The last CTA to finish
// (ticket counter, re-armed by that CTA) runs the top-k, one warp per token.
#include <mutex>

#include "qf_common.cuh"
#include "topk.cuh"

namespace {

using qf::bf16_lo;
constexpr int RW = 16;         // warps per CTA
constexpr int RT = RW * 32;    // threads per CTA
constexpr int REXP = 16;       // router rows per CTA
constexpr int MAXNT = QF_MAX_TOKENS / 8;

__device__ __forceinline__ uint4 ldg_nc_v4(const uint4* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

template <int BPW>
__global__ void __launch_bounds__(RT, 1)
    router_topk_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                       __nv_bfloat16* __restrict__ logits, float* __restrict__ weights, int* __restrict__ ids,
                       float* __restrict__ scratch, unsigned* __restrict__ counter, int rows, int H, int E, int topk,
                       int renorm) {
    extern __shared__ float red[];   // [RW][REXP][rp]
    __shared__ unsigned s_last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    const int e0 = blockIdx.x * REXP;
    const int nblk = H / 32;
    const int b0 = warp * BPW;
    const int ntile = (rows + 7) >> 3, rp = ntile * 8;

    // this warp's 32-k blocks of router rows e0+g and e0+g+8 (thread t holds k = 32b + 8t .. +8)
    uint4 wa[BPW], wb[BPW];
    const uint4* ra = reinterpret_cast<const uint4*>(w + (size_t)(e0 + g) * H) + t;
    const uint4* rb = reinterpret_cast<const uint4*>(w + (size_t)(e0 + g + 8) * H) + t;
#pragma unroll
    for (int i = 0; i < BPW; ++i) {
        if (b0 + i < nblk) {
            wa[i] = ldg_nc_v4(ra + 4 * (b0 + i));
            wb[i] = ldg_nc_v4(rb + 4 * (b0 + i));
        } else {
            wa[i] = wb[i] = make_uint4(0, 0, 0, 0);
        }
    }
    qf::pdl_wait();
    qf::pdl_launch_dependents();

    float d[MAXNT][4];
    // token tiles two at a time: their x fragments are all requested before the first mma uses one
#pragma unroll
    for (int np = 0; np < MAXNT; np += 2) {
        if (np < ntile) {
            uint4 xv[2][BPW];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int tok = (np + h) * 8 + g;
                const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)(tok < rows ? tok : 0) * H) + t;
#pragma unroll
                for (int i = 0; i < BPW; ++i)
                    xv[h][i] = (tok < rows && b0 + i < nblk) ? __ldcg(xr + 4 * (b0 + i)) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int nt = np + h;
                d[nt][0] = d[nt][1] = d[nt][2] = d[nt][3] = 0.f;
#pragma unroll
                for (int i = 0; i < BPW; ++i) {
                    if (b0 + i < nblk) {
                        qf::mma_bf16(d[nt], wa[i].x, wb[i].x, wa[i].y, wb[i].y, xv[h][i].x, xv[h][i].y);
                        qf::mma_bf16(d[nt], wa[i].z, wb[i].z, wa[i].w, wb[i].w, xv[h][i].z, xv[h][i].w);
                    }
                }
            }
        }
    }
#pragma unroll
    for (int nt = 0; nt < MAXNT; ++nt) {
        if (nt < ntile) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int r = g + ((i & 2) ? 8 : 0), tok = nt * 8 + 2 * t + (i & 1);
                red[(warp * REXP + r) * rp + tok] = d[nt][i];
            }
        }
    }
    __syncthreads();
    for (int idx = tid; idx < REXP * rows; idx += RT) {
        const int r = idx % REXP, tok = idx / REXP;
        float s = 0.f;
#pragma unroll
        for (int ww = 0; ww < RW; ++ww) s += red[(ww * REXP + r) * rp + tok];
        const __nv_bfloat16 bv = __float2bfloat16(s);
        logits[(size_t)tok * E + e0 + r] = bv;
        scratch[(size_t)tok * E + e0 + r] = __bfloat162float(bv);
    }

    // ---- last CTA: softmax + top-k per token
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        s_last = atomicAdd(counter, 1u) == gridDim.x - 1;
    }
    __syncwarp();
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (tid == 0) *counter = 0u;
    for (int tok = warp; tok < rows; tok += RW)
        qf::topk_row_any(scratch + (size_t)tok * E, E, topk, renorm, weights + (size_t)tok * topk,
                         ids + (size_t)tok * topk);
}

template <int BPW>
int launch_router(const void* x, const void* w, int rows, int H, int E, int topk, int renorm, float* weights,
                  int32_t* ids, void* logits, float* scratch, int32_t* counter, int pdl, cudaStream_t stream) {
    const int rp = ((rows + 7) / 8) * 8;
    const size_t smem = (size_t)RW * REXP * rp * sizeof(float);
    auto kern = router_topk_kernel<BPW>;
    cudaError_t e = qf::ensure_smem_attr(reinterpret_cast<const void*>(kern), RW * REXP * QF_MAX_TOKENS * 4);
    if (e != cudaSuccess) return qf::cuda_status(e, "router_topk: cudaFuncSetAttribute");
    e = qf::launch_ex(kern, dim3(E / REXP), dim3(RT), smem, stream, pdl != 0,
                      reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<const __nv_bfloat16*>(w),
                      reinterpret_cast<__nv_bfloat16*>(logits), weights, reinterpret_cast<int*>(ids), scratch,
                      reinterpret_cast<unsigned*>(counter), rows, H, E, topk, renorm);
    return qf::cuda_status(e, "router_topk: launch");
}

}  // namespace

namespace {
// Argument checks of both router entry points, made before anything is enqueued on the stream.
int router_args(const void* x, const void* w, int rows, int hidden, int experts, int topk, const float* topk_weights,
                const int32_t* topk_ids, const void* logits, const float* scratch, int64_t scratch_numel,
                const int32_t* counter) {
    QF_REQUIRE(x && w && topk_weights && topk_ids && logits && scratch && counter,
               "router_topk: null pointer argument");
    QF_REQUIRE(rows >= 1 && rows <= QF_MAX_TOKENS, "router_topk: rows must be in [1, %d], got %d", QF_MAX_TOKENS,
               rows);
    QF_REQUIRE(hidden >= 256 && hidden % 256 == 0 && hidden <= 4096,
               "router_topk: hidden must be a multiple of 256 in [256, 4096], got %d", hidden);
    QF_REQUIRE(experts >= 16 && experts % 16 == 0 && experts <= QF_MAX_EXPERTS,
               "router_topk: experts must be a multiple of 16 in [16, %d], got %d", QF_MAX_EXPERTS, experts);
    QF_REQUIRE(topk >= 1 && topk <= QF_MAX_TOPK && topk <= experts, "router_topk: topk must be in [1, %d], got %d",
               QF_MAX_TOPK, topk);
    QF_REQUIRE(scratch_numel >= (int64_t)rows * experts, "router_topk: scratch needs %lld floats, got %lld",
               (long long)rows * experts, (long long)scratch_numel);
    QF_REQUIRE(qf::aligned(x, 16) && qf::aligned(w, 16), "router_topk: x and w must be 16-byte aligned");
    return QF_OK;
}
}  // namespace

extern "C" int qf_router_topk(const void* x, const void* w, int rows, int hidden, int experts, int topk,
                              int renormalize, float* topk_weights, int32_t* topk_ids, void* logits, float* scratch,
                              int64_t scratch_numel, int32_t* counter, int pdl, qf_stream_t stream) {
    const int rc = router_args(x, w, rows, hidden, experts, topk, topk_weights, topk_ids, logits, scratch,
                               scratch_numel, counter);
    if (rc != QF_OK) return rc;
    const int bpw = (hidden / 32 + RW - 1) / RW;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (bpw <= 1) return launch_router<1>(x, w, rows, hidden, experts, topk, renormalize, topk_weights, topk_ids,
                                          logits, scratch, counter, pdl, st);
    if (bpw <= 2) return launch_router<2>(x, w, rows, hidden, experts, topk, renormalize, topk_weights, topk_ids,
                                          logits, scratch, counter, pdl, st);
    if (bpw <= 4) return launch_router<4>(x, w, rows, hidden, experts, topk, renormalize, topk_weights, topk_ids,
                                          logits, scratch, counter, pdl, st);
    return launch_router<8>(x, w, rows, hidden, experts, topk, renormalize, topk_weights, topk_ids, logits, scratch,
                            counter, pdl, st);
}

// ============================================================================================================
// Router entry point that allocates nothing.
//
// Some hosts cannot hand this library device memory for scratch: a plugin that is enqueued by an inference engine
// whose memory pool is sized once at start-up, or a launcher running while a CUDA graph is being captured, where a
// cudaMalloc would either fail, synchronise the device, or invalidate the capture. For them the router's two scratch
// buffers (the fp32 copy of the logits the top-k reads and the ticket counter of the last-CTA hand-off) live in the
// file-scope device array below instead of in caller-owned tensors. The caller still passes x, w and the three
// outputs. Limit: rows * experts <= 64 * 1024 (256 KB of fp32, plus one counter word); every GPU that loads the
// library keeps this array until the process exits.
//
// Set-up: the first call in a CUDA context (the device's primary context, as the runtime uses it, or another context
// the host made current) resolves the array's device address in that context with cudaGetSymbolAddress and caches it
// under the context's unique id; make that first call before any stream capture. A later call in a different context
// (after cudaDeviceReset, or on another context of the same device) resolves the address again. Each call checks its
// arguments, then clears the counter with cudaMemsetAsync on the caller's stream and launches the same kernel as
// qf_router_topk; a call that fails its checks enqueues nothing.
// All calls in a context share the array and it keeps the last call's contents, so calls that can overlap on the GPU
// (different streams, or no ordering between them) race with each other; order them on one stream.
namespace {
constexpr int NOALLOC_SCRATCH_FLOATS = QF_MAX_TOKENS * QF_MAX_EXPERTS;
// [0, NOALLOC_SCRATCH_FLOATS): logits scratch; the next word: ticket counter
static __device__ __align__(256) uint32_t g_router_noalloc[NOALLOC_SCRATCH_FLOATS + 64];

struct NoAllocSlot {
    bool ready;
    unsigned long long ctx_id;   // unique id of the context the address belongs to
    float* scratch;
    int32_t* counter;
};
std::mutex g_noalloc_mu;
NoAllocSlot g_noalloc_slot[64];

// Unique id of the calling thread's current CUDA context (driver cuCtxGetCurrent + cuCtxGetId, reached through the
// runtime's driver entry-point query, so the library still links against the runtime only). Ids are never reused,
// unlike context handles.
int current_context_id(unsigned long long* id) {
    using GetCurrent = int (*)(void**);
    using GetId = int (*)(void*, unsigned long long*);
    static GetCurrent get_current = nullptr;
    static GetId get_id = nullptr;
    if (get_current == nullptr || get_id == nullptr) {
        void* f0 = nullptr;
        void* f1 = nullptr;
        cudaDriverEntryPointQueryResult q0, q1;
        cudaError_t e = cudaGetDriverEntryPoint("cuCtxGetCurrent", &f0, cudaEnableDefault, &q0);
        if (e == cudaSuccess) e = cudaGetDriverEntryPoint("cuCtxGetId", &f1, cudaEnableDefault, &q1);
        if (e != cudaSuccess) return qf::cuda_status(e, "router_topk_noalloc: cudaGetDriverEntryPoint");
        QF_REQUIRE(q0 == cudaDriverEntryPointSuccess && q1 == cudaDriverEntryPointSuccess && f0 && f1,
                   "router_topk_noalloc: the driver does not provide cuCtxGetCurrent / cuCtxGetId");
        get_current = reinterpret_cast<GetCurrent>(f0);
        get_id = reinterpret_cast<GetId>(f1);
    }
    void* ctx = nullptr;
    QF_REQUIRE(get_current(&ctx) == 0, "router_topk_noalloc: cuCtxGetCurrent failed");
    if (ctx == nullptr) {
        // no context is current on this thread yet: the runtime's primary context of the current device becomes
        // current (a context the host made current itself is never replaced)
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e == cudaSuccess) e = cudaSetDevice(dev);
        if (e != cudaSuccess) return qf::cuda_status(e, "router_topk_noalloc: initialising the primary context");
        QF_REQUIRE(get_current(&ctx) == 0 && ctx != nullptr, "router_topk_noalloc: no current CUDA context");
    }
    QF_REQUIRE(get_id(ctx, id) == 0, "router_topk_noalloc: cuCtxGetId failed");
    return QF_OK;
}
}  // namespace

extern "C" int qf_router_topk_noalloc(const void* x, const void* w, int rows, int hidden, int experts, int topk,
                                      int renormalize, float* topk_weights, int32_t* topk_ids, void* logits, int pdl,
                                      qf_stream_t stream) {
    QF_REQUIRE(rows >= 1 && experts >= 1 && (int64_t)rows * experts <= NOALLOC_SCRATCH_FLOATS,
               "router_topk_noalloc: rows * experts must be at most %d (static scratch), got %d * %d",
               NOALLOC_SCRATCH_FLOATS, rows, experts);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return qf::cuda_status(e, "router_topk_noalloc: cudaGetDevice");
    QF_REQUIRE(dev >= 0 && dev < 64, "router_topk_noalloc: device ordinal %d out of range", dev);
    unsigned long long ctx_id = 0;
    int rc = current_context_id(&ctx_id);
    if (rc != QF_OK) return rc;
    NoAllocSlot slot;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        if (!g_noalloc_slot[dev].ready || g_noalloc_slot[dev].ctx_id != ctx_id) {
            void* base = nullptr;
            e = cudaGetSymbolAddress(&base, g_router_noalloc);
            if (e != cudaSuccess) return qf::cuda_status(e, "router_topk_noalloc: cudaGetSymbolAddress");
            g_noalloc_slot[dev].scratch = static_cast<float*>(base);
            g_noalloc_slot[dev].counter = reinterpret_cast<int32_t*>(static_cast<uint32_t*>(base) + NOALLOC_SCRATCH_FLOATS);
            g_noalloc_slot[dev].ctx_id = ctx_id;
            g_noalloc_slot[dev].ready = true;
        }
        slot = g_noalloc_slot[dev];
    }
    rc = router_args(x, w, rows, hidden, experts, topk, topk_weights, topk_ids, logits, slot.scratch,
                     NOALLOC_SCRATCH_FLOATS, slot.counter);
    if (rc != QF_OK) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    e = cudaMemsetAsync(slot.counter, 0, sizeof(int32_t), st);
    if (e != cudaSuccess) return qf::cuda_status(e, "router_topk_noalloc: clearing the counter");
    return qf_router_topk(x, w, rows, hidden, experts, topk, renormalize, topk_weights, topk_ids, logits, slot.scratch,
                          NOALLOC_SCRATCH_FLOATS, slot.counter, pdl, stream);
}
