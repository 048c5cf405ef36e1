// W8A8 INT8 GEMM for decode token counts (M <= 16) on the 5th-generation tensor cores.
//
//   y[t, n] = bf16((float(acc[t, n]) * sx[t]) * sw[n]),   acc[t, n] = sum_k xq[t, k] * q[n, k]   (exact int32)
//
// BASELINE config 3 (K = 2048, N up to 12288). There is no reference kernel for W8A8; the definition is the
// configuration's. The per-token quantisation (sx, and xq packed as the tensor-core operand) is the small kernel in
// w8.cu; this kernel runs under its programmatic dependent launch.
//
// B200 structure (a weight stream: the contraction is ~1/16 of an int8 tensor-core tile per byte)
//   * Work unit = one 16 KB weight tile (128 rows x 128 k), stored contiguously by qf_w8_repack in the K-major
//     128-byte-swizzle operand layout (row r at r * 128, its 16-byte k chunk c at position c ^ (r % 8)); units are
//     numbered tile-row-major, so unit u is the u-th 16 KB of the repacked weight.
//   * Stream-K: one CTA per SM (grid = min(SMs, units)) takes an equal contiguous run of units. Every SM streams,
//     whatever N / 128 is, and a run may start or end inside a 128-row tile (a "segment" is the part of a run in
//     one tile).
//   * 92 KB of shared memory, so two CTAs fit on an SM: the next GEMM's CTAs become resident while this one
//     drains (programmatic dependent launch of the quantisation kernel, which triggers at entry) and prefetch
//     their first weight tiles -- consecutive decode GEMMs keep HBM busy across kernel boundaries.
//   * Warp 5 (one lane) streams each unit's weight tile, plus its 2 KB token operand slab (16 tokens x 128 k
//     int8, [8 k chunks][16 tokens][16 B], tokens >= M zero), into a 5-slot ring with 1-D bulk copies. It
//     initialises its own barriers and requests the first weight tiles at entry, before the TMEM allocation and
//     before griddepcontrol.wait (the weights are load-time data); the slabs follow the wait.
//   * Warp 4 (one lane) issues tcgen05.mma.kind::i8 (M128 x N16 x K32: A = the weight tile, B = the slab, s32 D
//     in 16 TMEM columns), four per unit, accumulating a segment in one of two TMEM buffers.
//   * Warps 0-3 (thread = weight row) read a finished segment back. A segment that covers its whole tile writes
//     y directly. A tile split over several runs is finished by its owner, the run that holds the tile's first
//     unit (the end of that run, so usually the last to finish): every other run adds its int32 partials into a
//     global fixup buffer (red.add) and counts its units with a release; the owner waits (bounded; all runs of
//     the grid are resident) until the others are counted (acquire), loads their sums, adds its own, writes y
//     and leaves zeros behind. Integer addition is exact and order-free: the result does not depend on the
//     partition or the arrival order.
//   * Every mbarrier wait is bounded; a wait that runs out leaves the outputs undefined, sets the status word and
//     makes the CTA wait (bounded) for its outstanding copies and MMAs before it exits.
#include "qf_common.cuh"

namespace {

constexpr int TC_THREADS = 192;               // warps 0-3 read back, warp 4 MMA issue, warp 5 copies
constexpr int TC_RING = 5;                    // ring slots (weight tile + token slab); 2 CTAs per SM fit
constexpr int TILE_K = 128;                   // k per unit (one 128-byte swizzle row of int8)
constexpr int TILE_N = 128;                   // weight rows per tile (the mma's M)
constexpr int TILE_BYTES = TILE_N * TILE_K;   // 16 KB
constexpr int TOK = 16;                       // token columns (the mma's N); tokens >= M are zero in the slab
constexpr int SLAB_BYTES = TILE_K * TOK;      // 2 KB token operand of one unit: [8 k chunks][16 tokens][16 B]
constexpr int OFF_RING = 0;                                     // 1024-aligned slots (128-byte swizzle atoms)
constexpr int OFF_SLAB = OFF_RING + TC_RING * TILE_BYTES;
constexpr int OFF_SCALE = OFF_SLAB + TC_RING * SLAB_BYTES;      // float [16] per-token scale
constexpr int OFF_FLAG = OFF_SCALE + TOK * 4;                   // int: the owner's wait is over
constexpr int OFF_BAR = OFF_FLAG + 16;   // full[ring], empty[ring], sdone[2], sfree[2], mend, tmem addr
constexpr int TC_SMEM = OFF_BAR + (2 * TC_RING + 5) * 8 + 16 + 1024;   // + slack to align the base to 1024
constexpr uint64_t TC_WAIT_NS = 2000000000ull;
// instruction descriptor, kind::i8: s32 D (bits 4-5 = 2), s8 A and B (bits 7-9, 10-12 = 1), K-major A and B,
// N >> 3 at bit 17, M >> 4 at bit 24
constexpr uint32_t IDESC_I8 = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TOK >> 3) << 17) |
                              ((uint32_t)(TILE_N >> 4) << 24);

// K-major, 128-byte swizzle shared-memory descriptor: 8-row x 128-byte atoms, stride 1024 B between 8-row groups;
// the start must be 1024-aligned and advances by the k offset in bytes (>> 4) inside an atom.
__device__ __forceinline__ uint64_t sw128_desc(const void* p) {
    uint64_t d = (uint64_t)((qf::smem_u32(p) >> 4) & 0x3FFFu);
    d |= (uint64_t)1 << 16;              // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;    // stride byte offset
    d |= (uint64_t)1 << 46;              // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;              // layout: 128-byte swizzle
    return d;
}

__device__ __forceinline__ void mma_i8(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(adesc), "l"(bdesc), "r"(IDESC_I8), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void red_add_s32(int32_t* p, int32_t v) {
    asm volatile("red.relaxed.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int32_t ld_relaxed_s32(const int32_t* p) {
    int32_t v;
    asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Release add (the writes this thread observed, including those of the CTA ordered before it by a barrier, are
// visible before the add).
__device__ __forceinline__ void red_add_release(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// A CTA's run of units [u0, u1) splits into segments at tile boundaries; both the MMA issuer and the readback
// warps walk the same sequence.
struct Segment {
    int u, end;   // units [u, end) of tile `tile`
    int tile;
};
__device__ __forceinline__ Segment segment_at(int u, int u1, int KT) {
    Segment s;
    s.u = u;
    s.tile = u / KT;
    s.end = min(u1, (s.tile + 1) * KT);
    return s;
}

__device__ __forceinline__ void write_y(__nv_bfloat16* y, int ldy, int32_t* acc_out, int N, int n, int M,
                                        const int32_t (&a)[TOK], const float* scl, float wsc) {
#pragma unroll
    for (int t = 0; t < TOK; ++t) {
        if (t >= M) break;
        y[(size_t)t * ldy + n] = __float2bfloat16(__fmul_rn(__fmul_rn(__int2float_rn(a[t]), scl[t]), wsc));
        if (acc_out) acc_out[(size_t)t * N + n] = a[t];
    }
}

__global__ void __launch_bounds__(TC_THREADS, 2) w8a8_tc_kernel(const int8_t* __restrict__ qk,
                                                               const int8_t* __restrict__ xq,
                                                               const float* __restrict__ sx,
                                                               const float* __restrict__ sw,
                                                               __nv_bfloat16* __restrict__ y, int ldy,
                                                               int32_t* __restrict__ acc_out,
                                                               int32_t* __restrict__ fix, int M, int N, int K,
                                                               unsigned* __restrict__ err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // the 128-byte-swizzle tiles need a 1024-aligned base (the swizzle pattern repeats every 1024 bytes)
    uint8_t* smem = smem_raw + ((1024u - (qf::smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* ring = smem + OFF_RING;
    uint8_t* slab = smem + OFF_SLAB;
    float* scl = reinterpret_cast<float*>(smem + OFF_SCALE);
    volatile int* last_flag = reinterpret_cast<volatile int*>(smem + OFF_FLAG);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    uint64_t* empty = full + TC_RING;
    uint64_t* sdone = empty + TC_RING;
    uint64_t* sfree = sdone + 2;
    uint64_t* mend = sfree + 2;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(mend + 1);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int KT = K / TILE_K;
    const long long units = (long long)(N / TILE_N) * KT;   // < 2^30 (host check)
    const int u0 = (int)(units * blockIdx.x / gridDim.x), u1 = (int)(units * (blockIdx.x + 1) / gridDim.x);
    const int nu = u1 - u0;
    int32_t* fix_acc = fix;                                          // [16][N] partial sums (kept zero)
    uint32_t* fix_cnt = reinterpret_cast<uint32_t*>(fix + (size_t)TOK * N);   // [N / 128] units counted

    // Programmatic dependent launch: the next kernel in the stream reads nothing of this one before its own
    // griddepcontrol.wait, so it may be scheduled early -- once warps 0-3 are past their own wait (below).
    if (warp >= 4) qf::pdl_launch_dependents();
    if (warp == 5) {
        // ---------------------------------------------------------------- producer: weight tiles (+ slabs)
        if (lane == 0) {
            for (int i = 0; i < TC_RING; ++i) {
                qf::mbar_init(full + i, 1);
                qf::mbar_init(empty + i, 1);
            }
            qf::mbar_fence_init();
        }
        __syncwarp();
        qf::named_bar_arrive(2, TC_THREADS);   // hands the initialised ring barriers to warps 0-4
        if (lane == 0) {
            constexpr uint32_t TX = TILE_BYTES + SLAB_BYTES;
            const uint64_t pol = qf::policy_evict_first();
            const int pre = nu < TC_RING ? nu : TC_RING;
            // the weights are load-time data: request the first tiles before griddepcontrol.wait
            for (int i = 0; i < pre; ++i) {
                qf::mbar_arrive_expect_tx(full + i, TX);
                qf::bulk_g2s_hint(ring + i * TILE_BYTES, qk + (size_t)(u0 + i) * TILE_BYTES, TILE_BYTES, full + i, pol);
            }
            qf::pdl_wait();
            qf::fence_proxy_async();   // the slabs were written through the generic proxy
            for (int i = 0; i < pre; ++i)
                qf::bulk_g2s(slab + i * SLAB_BYTES, xq + (size_t)((u0 + i) % KT) * SLAB_BYTES, SLAB_BYTES, full + i);
            int issued = pre;
            for (int i = TC_RING; i < nu; ++i) {
                const int slot = i % TC_RING;
                if (!qf::mbar_wait(empty + slot, ((i / TC_RING) - 1) & 1, TC_WAIT_NS)) {
                    atomicOr(err, 1u);
                    break;
                }
                const int u = u0 + i;
                qf::mbar_arrive_expect_tx(full + slot, TX);
                qf::bulk_g2s_hint(ring + slot * TILE_BYTES, qk + (size_t)u * TILE_BYTES, TILE_BYTES, full + slot, pol);
                qf::bulk_g2s(slab + slot * SLAB_BYTES, xq + (size_t)(u % KT) * SLAB_BYTES, SLAB_BYTES, full + slot);
                ++issued;
            }
            // no copy may still be writing this CTA's shared memory when it exits (the MMA issuer may have given
            // up): each slot holds at most one unconsumed copy, its latest phase, so wait (bounded) for the last
            // ones issued -- off the critical path, the issue loop ends long before the CTA does
            for (int i = issued > TC_RING ? issued - TC_RING : 0; i < issued; ++i)
                qf::mbar_wait(full + i % TC_RING, (i / TC_RING) & 1, TC_WAIT_NS);
        }
        __syncwarp();
        __syncthreads();
        return;
    }
    if (tid == 0) {
        for (int b = 0; b < 2; ++b) {
            qf::mbar_init(sdone + b, 1);
            qf::mbar_init(sfree + b, 4);   // one arrive per readback warp
        }
        qf::mbar_init(mend, 1);
        qf::mbar_fence_init();
    }
    if (warp == 0) {
        qf::tmem_alloc(tslot, 32);
        qf::tmem_relinquish();
    }
    qf::tc_fence_before();
    qf::named_bar(2, TC_THREADS);
    qf::tc_fence_after();
    const uint32_t tmem = *tslot;

    if (warp == 4) {
        if (lane == 0) {
            // ---------------------------------------------------------------- MMA issuer
            bool ok = true;
            int i = 0, seg = 0;
            for (int u = u0; ok && u < u1; ++seg) {
                const Segment sg = segment_at(u, u1, KT);
                const int b = seg & 1;
                if (seg >= 2) {
                    if (!qf::mbar_wait(sfree + b, ((seg >> 1) - 1) & 1, TC_WAIT_NS)) {
                        atomicOr(err, 2u);
                        ok = false;
                        break;
                    }
                    qf::tc_fence_after();
                }
                const uint32_t d = tmem + 16u * b;
                for (; u < sg.end; ++u, ++i) {
                    const int slot = i % TC_RING;
                    if (!qf::mbar_wait(full + slot, (i / TC_RING) & 1, TC_WAIT_NS)) {
                        atomicOr(err, 1u);
                        ok = false;
                        break;
                    }
                    qf::tc_fence_after();
                    const uint64_t adesc = sw128_desc(ring + slot * TILE_BYTES);
                    // B: k chunks 256 B apart, 8-token groups 128 B apart; one k32 step = 2 chunks (+512 B)
                    const uint64_t bdesc = qf::smem_desc(slab + slot * SLAB_BYTES, TOK * 16, 128);
#pragma unroll
                    for (int j = 0; j < TILE_K / 32; ++j)
                        mma_i8(d, adesc + 2 * j, bdesc + (uint64_t)((2 * j * TOK * 16) >> 4), (u != sg.u) || j != 0);
                    qf::mma_commit(empty + slot);
                }
                if (ok) qf::mma_commit(sdone + b);
            }
            qf::mma_commit(mend);   // every MMA issued above has completed once this arrives
        }
        __syncwarp();
    } else {
        // -------------------------------------------------------------------- warps 0-3: thread = weight row
        qf::pdl_wait();
        if (tid < TOK) scl[tid] = tid < M ? sx[tid] : 0.f;
        qf::pdl_launch_dependents();
        qf::named_bar(1, 128);
        const int row = 32 * warp + lane;
        // a wait that ran out leaves this warp's values undefined but keeps it in step: every thread still passes
        // every named barrier below, and the warp stops waiting after its first timeout
        bool bad = false;
        int seg = 0;
        for (int u = u0; u < u1; ++seg) {
            const Segment sg = segment_at(u, u1, KT);
            u = sg.end;
            const int b = seg & 1;
            const int n = sg.tile * TILE_N + row;
            const bool partial = sg.end - sg.u != KT;
            // a tile split over several runs is finished by its owner, the run holding the tile's first unit
            const bool owner = partial && sg.u % KT == 0;
            const unsigned others_units = (unsigned)(KT - (sg.end - sg.u));
            int32_t others[TOK];
            bool have = false;   // owner: the other contributions are complete and their sums are in `others`
            if (owner) {
                // early look, while this segment's MMAs may still run
                if (tid == 0) *last_flag = qf::ld_acquire(fix_cnt + sg.tile) == others_units;
                qf::named_bar(1, 128);
                have = *last_flag != 0;
                if (have) {
#pragma unroll
                    for (int t = 0; t < TOK; ++t) others[t] = t < M ? ld_relaxed_s32(fix_acc + (size_t)t * N + n) : 0;
                }
            }
            if (!bad) bad = !__all_sync(0xffffffffu, qf::mbar_wait(sdone + b, (seg >> 1) & 1, TC_WAIT_NS));
            uint32_t v[16] = {};
            if (!bad) {
                qf::tc_fence_after();
                qf::tmem_ld16(tmem + ((uint32_t)(32 * warp) << 16) + 16u * b, v);
                qf::tmem_wait_ld();
                qf::tc_fence_before();
                __syncwarp();
                if (lane == 0) qf::mbar_arrive(sfree + b);
            } else if (lane == 0) {
                atomicOr(err, 2u);
            }
            const float wsc = sw[n];
            int32_t a[TOK];
#pragma unroll
            for (int t = 0; t < TOK; ++t) a[t] = (int32_t)v[t];
            if (!partial) {
                write_y(y, ldy, acc_out, N, n, M, a, scl, wsc);   // the whole tile: no other CTA contributes
                continue;
            }
            if (!owner) {
                // publish the partials, then count them with a release (ordered after every thread's adds by the
                // barrier); the owner takes it from there
#pragma unroll
                for (int t = 0; t < TOK; ++t)
                    if (t < M) red_add_s32(fix_acc + (size_t)t * N + n, a[t]);
                qf::named_bar(1, 128);
                if (tid == 0) red_add_release(fix_cnt + sg.tile, (unsigned)(sg.end - sg.u));
                continue;
            }
            if (!have) {
                // the other runs of this tile are all resident (this grid fits the GPU and every CTA starts before
                // any dependent grid): wait (bounded) until their units are counted
                qf::named_bar(1, 128);   // every thread has read the early flag
                if (tid == 0) {
                    const long long t0 = clock64();
                    bool done = false;
                    while (!(done = qf::ld_acquire(fix_cnt + sg.tile) == others_units) &&
                           clock64() - t0 < (long long)(2 * TC_WAIT_NS))
                        __nanosleep(64);
                    if (!done) atomicOr(err, 8u);
                    *last_flag = 1;
                }
                qf::named_bar(1, 128);
#pragma unroll
                for (int t = 0; t < TOK; ++t) others[t] = t < M ? ld_relaxed_s32(fix_acc + (size_t)t * N + n) : 0;
            }
            // finish the tile from the others' sums and this run's own partials; leave zeros behind
#pragma unroll
            for (int t = 0; t < TOK; ++t) {
                a[t] += others[t];
                if (t < M) fix_acc[(size_t)t * N + n] = 0;
            }
            write_y(y, ldy, acc_out, N, n, M, a, scl, wsc);
            if (tid == 0) fix_cnt[sg.tile] = 0u;
            qf::named_bar(1, 128);   // last_flag is rewritten by the next segment
        }
    }

    qf::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        if (!qf::mbar_wait(mend, 0, TC_WAIT_NS)) atomicOr(err, 4u);
        qf::tc_fence_after();
        qf::tmem_dealloc(tmem, 32);
    }
}

// weight repacking: canonical [N, K] int8 <-> tiles [N/128][K/128][128 rows][128 B] (rows' 16-byte chunks swizzled)
__device__ __forceinline__ long long w8_canon_index(long long o, int K) {
    const long long tile = o / TILE_BYTES;
    const int within = (int)(o - tile * TILE_BYTES);
    const int kst = K / TILE_K;
    const long long r = tile / kst;
    const int ks = (int)(tile - r * kst);
    const int rr = within >> 7, c = ((within >> 4) & 7) ^ (rr & 7), b = within & 15;
    return (r * TILE_N + rr) * (long long)K + ks * TILE_K + c * 16 + b;
}

__global__ void w8_repack_kernel(const int8_t* __restrict__ src, int8_t* __restrict__ dst, long long total, int K,
                                 int unpack) {
    for (long long o = blockIdx.x * (long long)blockDim.x + threadIdx.x; o < total; o += (long long)gridDim.x * blockDim.x) {
        const long long c = w8_canon_index(o, K);
        if (!unpack) dst[o] = src[c];
        else dst[c] = src[o];
    }
}

__device__ unsigned g_w8a8_tc_err;

}  // namespace

namespace qf {

size_t w8a8_fixup_elems(int N) { return (size_t)TOK * N + N / TILE_N; }

cudaError_t launch_w8a8_tc(const int8_t* xq, const float* sx, const int8_t* q, const float* sw, void* y, int ldy,
                           int32_t* acc_out, int32_t* fix, int M, int N, int K, cudaStream_t st) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    e = ensure_smem_attr(reinterpret_cast<const void*>(w8a8_tc_kernel), TC_SMEM);
    if (e != cudaSuccess) return e;
    unsigned* err = nullptr;
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&err), g_w8a8_tc_err);
    if (e != cudaSuccess) return e;
    const long long units = (long long)(N / TILE_N) * (K / TILE_K);
    if (units >= (1ll << 30)) return cudaErrorInvalidValue;
    const int sms = sm_count(dev);
    const int grid = (int)(units < sms ? units : sms);
    return launch_ex(w8a8_tc_kernel, dim3(grid), dim3(TC_THREADS), TC_SMEM, st, true, q, xq, sx, sw,
                     static_cast<__nv_bfloat16*>(y), ldy, acc_out, fix, M, N, K, err);
}

// Reads and clears the kernel's sticky wait-timeout bits (1: a ring / operand wait, 2: a segment wait, 4: the final
// MMA wait, 8: the wait for the other runs of a split tile).
cudaError_t w8a8_tc_take_status(unsigned* out) {
    cudaError_t e = cudaMemcpyFromSymbol(out, g_w8a8_tc_err, sizeof(unsigned));
    if (e != cudaSuccess) return e;
    const unsigned zero = 0;
    return cudaMemcpyToSymbol(g_w8a8_tc_err, &zero, sizeof(unsigned));
}

cudaError_t launch_w8_repack(const int8_t* src, int8_t* dst, int N, int K, int unpack, cudaStream_t st) {
    const long long total = (long long)N * K;
    long long blocks = (total + 255) / 256;
    if (blocks > 65535LL * 8) blocks = 65535LL * 8;
    w8_repack_kernel<<<(unsigned)blocks, 256, 0, st>>>(src, dst, total, K, unpack);
    return cudaGetLastError();
}

}  // namespace qf
