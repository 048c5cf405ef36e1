// W8A16 group-scaled INT8 GEMM for decode token counts on the 5th-generation tensor cores.
//
//   y[t, n] = bf16( sum_g s[n, g] * sum_{k in group g} q[n, k] * x[t, k] )     fp32 accumulation, group 128 or 64
//
// Replaces `w8g_gemm` (serve/qwenfast/qf_w8g.cu:303-336): the same operands -- bf16 activations x [M, K], the
// canonical int8 weight q [N, K] and its bf16 group scales s [N, K / group] -- and the same arithmetic up to fp32
// association (every product is exact here, see below).
//
// B200 structure (a weight stream: decode M is 1..64 against N x K int8 weights)
//   * Work unit = 128 weight rows x 64 k (8 KB of int8, half a 128-group or one 64-group). The weight stays in its
//     canonical row-major layout: each unit arrives by one TMA 2-D tiled load (box 64 B x 128 rows, 64-byte swizzle,
//     so that the 128 threads that read one row each hit distinct shared-memory banks).
//   * Stream-K: up to 4 CTAs per SM (NT = 16; 2 for wider token groups), every CTA one pipeline over an equal
//     contiguous run of at least ~4 units (when there are units for one run per SM), numbered tile-row-major
//     (unit u = tile (u / KT), k-unit (u % KT), KT = K / 64). A run may start or end inside a tile; a "segment" is
//     the part of a run in one tile. (cudaOccupancyMaxActiveBlocksPerMultiprocessor reports one CTA per SM for any
//     kernel that allocates tensor memory; four of these 128-column CTAs do run concurrently on a B200 SM, measured.)
//   * Exact fp16 tensor-core operands, so that every product is exact and only the fp32 sums round:
//       - weights: int8 q -> fp16 exactly: the byte (q + 128) placed under the fp16 exponent of 1024 (one prmt per
//         pair) gives 1024 + q + 128, and one fp16x2 subtract of 1152 leaves q;
//       - tokens: fp16(x * 2^-e), e = floor(log2 max|x|) - 14 over the token's 64-k slice of the unit (the eight
//         lanes that stage the slice agree on it with three shuffles): exact, the slice's maximum lands in
//         [2^14, 2^15) and a bf16 value loses bits only below 2^-38 of it;
//       - read-back of each unit's fp32 D: acc[t] += D[t] * (s[n, g] * 2^e[t]).
//   * Warps 0-3 (thread = weight row): dequantise the unit into the TMEM A operand (tcgen05.st), stage the fp16
//     token slice into the shared-memory B operand (K-major, no swizzle: [k chunk][token][16 B]), hand the unit to
//     the MMA warp, then read back the previous unit. Warp 4 (one lane): tcgen05.mma kind::f16 M128 x NT x K16, four
//     per unit, into one of two TMEM accumulators; tcgen05.commit. Warp 5 (one lane): the TMA ring; it requests the
//     first units before griddepcontrol.wait (weights are load-time data).
//   * A tile split over several runs (at most the two ends of a run) is finished without any waiting: each of its
//     runs stores its fp32 partial sums to its own slot of the fixup buffer, fences and counts itself on the tile's
//     counter; the run that counts last adds all the parts in run order -- the same sum whichever run is last -- and
//     writes y. No run waits for another, so the grid need not be co-resident.
//   * Every wait is bounded; a wait that runs out sets a bit of the sticky status word (qf_w8g_take_status) and
//     the CTA drains (the affected outputs are undefined).
#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

#include "qf_common.cuh"

namespace {

constexpr int G_THREADS = 192;             // warps 0-3 consumers, warp 4 MMA issue, warp 5 TMA producer
constexpr int G_UK = 64;                   // k per unit
constexpr int G_UN = 128;                  // weight rows per tile (the MMA's M)
constexpr int G_UBYTES = G_UN * G_UK;      // 8 KB of int8 weights per unit
constexpr int G_RING = 6;                  // ring slots
constexpr uint64_t G_WAIT_NS = 2000000000ull;

template <int NT>
struct Cfg {
    static constexpr int BBYTES = NT * G_UK * 2;                  // fp16 token operand of a unit: [8][NT][16 B]
    static constexpr int OFF_RING = 0;                            // 1024-aligned slots
    static constexpr int OFF_B = OFF_RING + G_RING * G_UBYTES;
    static constexpr int OFF_F = OFF_B + 2 * BBYTES;              // float [2][NT] per-token factors 2^e
    static constexpr int OFF_BAR = OFF_F + 2 * NT * 4;            // full[ring], empty[ring], abr[2], mmab[2], mend
    static constexpr int OFF_MISC = OFF_BAR + (2 * G_RING + 5) * 8;   // tmem address, owner flag
    static constexpr int SMEM = OFF_MISC + 16 + 1024;             // + slack to align the base to 1024
    static constexpr uint32_t TM_A = 0;                           // 2 x 32 columns (64 k of fp16 per row)
    static constexpr uint32_t TM_D = 64;                          // 2 x NT columns
    static constexpr uint32_t TM_COLS = (TM_D + 2 * NT) <= 128 ? 128 : 256;
    static constexpr int MINB = NT == 16 ? 4 : 2;                 // CTAs per SM
    static constexpr uint32_t IDESC = qf::idesc_f16(G_UN, NT);
};

// int8 word (4 consecutive k) -> two fp16x2 of the values, exactly: the biased bytes (q + 128) go under the fp16
// exponent of 1024 (prmt with the high bytes 0x64), then 1152 = 1024 + 128 is subtracted.
__device__ __forceinline__ void i8x4_to_f16(uint32_t w, uint32_t& lo, uint32_t& hi) {
    const uint32_t u = w ^ 0x80808080u;
    const uint32_t a = __byte_perm(u, 0x64646464u, 0x4140), b = __byte_perm(u, 0x64646464u, 0x4342);
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(lo) : "r"(a), "r"(0x64806480u));
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(hi) : "r"(b), "r"(0x64806480u));
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, %3}], "
        "[%4], %5;" ::"r"(qf::smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(qf::smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ void red_release(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// unit range of run b of `runs` over `units`, and the run that holds unit u
__device__ __forceinline__ int run_start(long long units, int b, int runs) { return (int)(units * b / runs); }
__device__ __forceinline__ int run_of(long long units, int u, int runs) {
    int r = (int)(((long long)u * runs) / units);
    while (r + 1 < runs && run_start(units, r + 1, runs) <= u) ++r;
    while (r > 0 && run_start(units, r, runs) > u) --r;
    return r;
}

template <int NT>
__global__ void __launch_bounds__(G_THREADS, Cfg<NT>::MINB)
    w8g_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __nv_bfloat16* __restrict__ x, int ldx,
                  const uint16_t* __restrict__ s, __nv_bfloat16* __restrict__ y, int ldy, float* __restrict__ fixp,
                  uint32_t* __restrict__ fixc, int M, int N, int K, int G, int t0, unsigned* __restrict__ err) {
    using C = Cfg<NT>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (qf::smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* ring = smem + C::OFF_RING;
    uint8_t* bop = smem + C::OFF_B;
    float* fsc = reinterpret_cast<float*>(smem + C::OFF_F);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* empty = full + G_RING;
    uint64_t* abr = empty + G_RING;
    uint64_t* mmab = abr + 2;
    uint64_t* mend = mmab + 2;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
    volatile int* lastf = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int KT = K / G_UK;
    const long long units = (long long)((N + G_UN - 1) / G_UN) * KT;   // a last tile past N: rows of zeros
    const int runs = gridDim.x;
    const int u0 = run_start(units, blockIdx.x, runs), u1 = run_start(units, blockIdx.x + 1, runs);
    const int nu = u1 - u0;
    const int GS = K / G;   // scales per row

    if (tid == 0) {
        for (int i = 0; i < G_RING; ++i) {
            qf::mbar_init(full + i, 1);
            qf::mbar_init(empty + i, 4);   // one arrive per consumer warp
        }
        for (int b = 0; b < 2; ++b) {
            qf::mbar_init(abr + b, 4);
            qf::mbar_init(mmab + b, 1);
        }
        qf::mbar_init(mend, 1);
        qf::mbar_fence_init();
    }
    if (warp == 0) {
        qf::tmem_alloc(tslot, C::TM_COLS);
        qf::tmem_relinquish();
    }
    qf::tc_fence_before();
    __syncthreads();
    qf::tc_fence_after();
    const uint32_t tmem = *tslot;

    if (warp == 5) {
        // ---------------------------------------------------------------- producer: TMA ring of weight units
        if (lane == 0) {
            const uint64_t pol = qf::policy_evict_first();
            const int pre = nu < G_RING ? nu : G_RING;
            for (int i = 0; i < pre; ++i) {   // load-time data: requested before the wait on the previous kernel
                const int u = u0 + i;
                qf::mbar_arrive_expect_tx(full + i, G_UBYTES);
                tma_load_2d(ring + i * G_UBYTES, &qmap, (u % KT) * G_UK, (u / KT) * G_UN, full + i, pol);
            }
            qf::pdl_wait();
            qf::pdl_launch_dependents();
            int issued = pre;
            for (int i = G_RING; i < nu; ++i) {
                const int slot = i % G_RING;
                if (!qf::mbar_wait(empty + slot, ((i / G_RING) - 1) & 1, G_WAIT_NS)) {
                    atomicOr(err, 1u);
                    break;
                }
                const int u = u0 + i;
                qf::mbar_arrive_expect_tx(full + slot, G_UBYTES);
                tma_load_2d(ring + slot * G_UBYTES, &qmap, (u % KT) * G_UK, (u / KT) * G_UN, full + slot, pol);
                ++issued;
            }
            // no copy may still be writing this CTA's shared memory when it exits: wait (bounded) for the last ones
            for (int i = issued > G_RING ? issued - G_RING : 0; i < issued; ++i)
                qf::mbar_wait(full + i % G_RING, (i / G_RING) & 1, G_WAIT_NS);
        }
        __syncwarp();
    } else if (warp == 4) {
        // ---------------------------------------------------------------- MMA issuer: 4 k16 steps per unit
        const uint64_t bdesc0 = qf::smem_desc(bop, NT * 16, 128);   // k chunks NT x 16 B apart, 8-token groups 128 B
        for (int i = 0; i < nu; ++i) {
            const int b = i & 1;
            if (!qf::mbar_wait(abr + b, (i >> 1) & 1, G_WAIT_NS)) {
                if (lane == 0) atomicOr(err, 2u);
                break;
            }
            if (lane == 0) {
                qf::tc_fence_after();
                const uint32_t d = tmem + C::TM_D + (uint32_t)(NT * b);
                const uint32_t a = tmem + C::TM_A + 32u * b;
                const uint64_t bd = bdesc0 + (uint64_t)(b * (C::BBYTES >> 4));
#pragma unroll
                for (int j = 0; j < G_UK / 16; ++j)
                    qf::mma_ts(d, a + 8 * j, bd + (uint64_t)((2 * j * NT * 16) >> 4), C::IDESC, j != 0);
                qf::mma_commit(mmab + b);
            }
            __syncwarp();
        }
        if (lane == 0) qf::mma_commit(mend);   // every MMA issued above has completed once this arrives
        __syncwarp();
    } else {
        // -------------------------------------------------------------------- warps 0-3: thread = weight row
        const int row = 32 * warp + lane;              // TMEM lane = tile row (warp w owns lanes 32w .. 32w + 31)
        const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
        const uint32_t ta0 = tmem + lane_base + C::TM_A, td0 = tmem + lane_base + C::TM_D;
        // B staging: NT tokens x 8 chunks of 8 k per unit; thread tid stages chunk (tid & 7) of tokens
        // (tid >> 3) + 16 j, j < NT / 16 -- the eight lanes of a token slice are consecutive
        constexpr int NJ = NT / 16;
        const int bc = tid & 7, bn = tid >> 3;
        qf::pdl_wait();
        float acc[NT];
        uint32_t mph = 0;
        bool bad = false;
        // this thread's token chunks of unit u (requested one unit before they are staged)
        uint4 xv[NJ];
        auto load_x = [&](int u) {
            const int k0 = (u % KT) * G_UK + 8 * bc;
#pragma unroll
            for (int j = 0; j < NJ; ++j) {
                const int t = t0 + bn + 16 * j;
                xv[j] = t < M ? __ldg(reinterpret_cast<const uint4*>(x + (size_t)t * ldx + k0)) : make_uint4(0u, 0u, 0u, 0u);
            }
        };
        // stage the loaded token slice into B buffer b (and the factors 2^e into fsc[b])
        auto stage_b = [&](int b) {
#pragma unroll
            for (int j = 0; j < NJ; ++j) {
                const int n = bn + 16 * j, t = t0 + n;
                const uint4 v = xv[j];
                const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
                float mx = 0.f;
#pragma unroll
                for (int i = 0; i < 4; ++i) mx = fmaxf(mx, fmaxf(fabsf(qf::bf16_lo(vv[i])), fabsf(qf::bf16_hi(vv[i]))));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                // e = floor(log2 mx) - 14 from the exponent field (0 for zero, subnormal, inf or NaN maxima)
                const int ef = (int)((__float_as_uint(mx) >> 23) & 0xFFu);
                const int e = (ef == 0 || ef == 255) ? 0 : max(-96, min(96, ef - 127 - 14));
                const float mul = __uint_as_float((uint32_t)(127 - e) << 23);
                uint4 o;
                o.x = qf::bf16x2_to_f16x2_scaled(v.x, mul);
                o.y = qf::bf16x2_to_f16x2_scaled(v.y, mul);
                o.z = qf::bf16x2_to_f16x2_scaled(v.z, mul);
                o.w = qf::bf16x2_to_f16x2_scaled(v.w, mul);
                *reinterpret_cast<uint4*>(bop + b * C::BBYTES + (bc * NT + n) * 16) = o;
                if (bc == 0) fsc[b * NT + n] = t < M ? __uint_as_float((uint32_t)(127 + e) << 23) : 0.f;
            }
        };
        // the scale of this thread's row for unit u
        auto row_scale = [&](int u) {
            const int n = (u / KT) * G_UN + row;
            return n < N ? qf::bf16_bits(__ldg(s + (size_t)n * GS + ((u % KT) * G_UK) / G)) : 0.f;
        };
        int i = 0;
        float sc_next = nu > 0 ? row_scale(u0) : 0.f;
        if (nu > 0) {
            load_x(u0);
            stage_b(0);
            if (nu > 1) load_x(u0 + 1);
        }
        qf::named_bar(1, 128);   // every token factor of the unit is in shared memory before any read-back uses it
        while (i < nu) {
            // ------------------------------------------------------------ one segment: units [u, end) of a tile
            const int su = u0 + i;
            const int tile = su / KT;
            const int end = min(u1, (tile + 1) * KT);
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[t] = 0.f;
            bool pend = false;
            int pb = 0;
            float psc = 0.f;
            for (int u = su; u < end; ++u, ++i) {
                const int b = i & 1, slot = i % G_RING;
                const float sc = sc_next;
                if (i + 1 < nu) sc_next = row_scale(u + 1);
                if (!bad) bad = !__all_sync(0xffffffffu, qf::mbar_wait(full + slot, (i / G_RING) & 1, G_WAIT_NS));
                // dequantise this row's 64 bytes (four 16-byte chunks, at positions c ^ ((row >> 1) & 3)) into TMEM
                const uint8_t* wr = ring + slot * G_UBYTES + row * 64;
                const int sw = (row >> 1) & 3;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const uint4 q = *reinterpret_cast<const uint4*>(wr + 16 * (c ^ sw));
                    uint32_t v[8];
                    i8x4_to_f16(q.x, v[0], v[1]);
                    i8x4_to_f16(q.y, v[2], v[3]);
                    i8x4_to_f16(q.z, v[4], v[5]);
                    i8x4_to_f16(q.w, v[6], v[7]);
                    qf::tmem_st8(ta0 + 32u * b + 8 * c, v);
                }
                qf::fence_proxy_async_smem();   // the B operand was written through the generic proxy
                qf::tmem_wait_st();
                qf::tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    qf::mbar_arrive(empty + slot);
                    qf::mbar_arrive(abr + b);
                }
                if (pend) {   // read back the previous unit of this segment
                    if (!bad) bad = !__all_sync(0xffffffffu, qf::mbar_wait(mmab + pb, (mph >> pb) & 1u, G_WAIT_NS));
                    mph ^= 1u << pb;
                    qf::tc_fence_after();
                    uint32_t dv[NT];
#pragma unroll
                    for (int h = 0; h < NT; h += 16) qf::tmem_ld16(td0 + (uint32_t)(NT * pb + h), *reinterpret_cast<uint32_t(*)[16]>(dv + h));
                    qf::tmem_wait_ld();
#pragma unroll
                    for (int t = 0; t < NT; ++t) acc[t] = fmaf(__uint_as_float(dv[t]), psc * fsc[pb * NT + t], acc[t]);
                    qf::tc_fence_before();
                }
                // B buffer b ^ 1 is free (its unit was just read back, or never used): stage the next unit's tokens.
                // The barrier first: every thread has read the factors of buffer b ^ 1 (the previous unit) before any
                // thread overwrites them, and the factors staged here are read two units later, after the next
                // iteration's barrier.
                qf::named_bar(1, 128);
                if (i + 1 < nu) {
                    stage_b(b ^ 1);
                    if (i + 2 < nu) load_x(u + 2);
                }
                pend = true;
                pb = b;
                psc = sc;
            }
            // the segment's last unit
            if (pend) {
                if (!bad) bad = !__all_sync(0xffffffffu, qf::mbar_wait(mmab + pb, (mph >> pb) & 1u, G_WAIT_NS));
                mph ^= 1u << pb;
                qf::tc_fence_after();
                uint32_t dv[NT];
#pragma unroll
                for (int h = 0; h < NT; h += 16) qf::tmem_ld16(td0 + (uint32_t)(NT * pb + h), *reinterpret_cast<uint32_t(*)[16]>(dv + h));
                qf::tmem_wait_ld();
#pragma unroll
                for (int t = 0; t < NT; ++t) acc[t] = fmaf(__uint_as_float(dv[t]), psc * fsc[pb * NT + t], acc[t]);
                qf::tc_fence_before();
            }
            if (bad && lane == 0) atomicOr(err, 2u);
            // ------------------------------------------------------------ segment output
            const int n = tile * G_UN + row;
            if (end - su == KT) {   // the whole tile: no other run contributes
#pragma unroll
                for (int t = 0; t < NT; ++t)
                    if (t0 + t < M && n < N) y[(size_t)(t0 + t) * ldy + n] = __float2bfloat16(acc[t]);
                continue;
            }
            // a tile split over several runs: this run's part goes to its slot (run r owns slots 2r -- the tile of
            // its first unit -- and 2r + 1 -- the tile of its last unit); the last run of the tile to count itself
            // adds every part in run order (the same sum whichever run finishes last) and writes y
            const int slot = 2 * (int)blockIdx.x + (su == u0 ? 0 : 1);
            float* sp = fixp + (size_t)slot * NT * G_UN;
#pragma unroll
            for (int t = 0; t < NT; ++t)
                if (t0 + t < M) __stcg(sp + t * G_UN + row, acc[t]);
            __threadfence();
            const int rf = run_of(units, tile * KT, runs), rl = run_of(units, tile * KT + KT - 1, runs);
            qf::named_bar(1, 128);
            if (tid == 0) *lastf = atomicAdd(fixc + tile, 1u) == (uint32_t)(rl - rf);
            qf::named_bar(1, 128);
            if (*lastf == 0) continue;
            __threadfence();
#pragma unroll
            for (int t = 0; t < NT; ++t) acc[t] = 0.f;
            for (int r = rf; r <= rl; ++r) {
                const int rs = 2 * r + ((run_start(units, r, runs) / KT) == tile ? 0 : 1);
                const float* op = fixp + (size_t)rs * NT * G_UN;
#pragma unroll
                for (int t = 0; t < NT; ++t)
                    if (t0 + t < M) acc[t] += __ldcg(op + t * G_UN + row);
            }
#pragma unroll
            for (int t = 0; t < NT; ++t)
                if (t0 + t < M && n < N) y[(size_t)(t0 + t) * ldy + n] = __float2bfloat16(acc[t]);
            if (tid == 0) fixc[tile] = 0u;   // re-armed for the next call
            qf::named_bar(1, 128);           // lastf is rewritten by the next segment
        }
    }

    qf::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        if (!qf::mbar_wait(mend, 0, G_WAIT_NS)) atomicOr(err, 4u);
        qf::tc_fence_after();
        qf::tmem_dealloc(tmem, Cfg<NT>::TM_COLS);
    }
}

__device__ unsigned g_w8g_err;

#include "w8g_rf.cuh"

// The register-fragment kernel's launch (M <= 16, K % 128 == 0): ks stages per item chosen so that the grid covers
// the SMs about two CTAs deep with at most S_MAX splits per tile (S = ceil(K / 128 / ks)), raised while the grid is
// larger than one wave. The shared memory is sized first as for 16 staged token rows with at most 12 stages (the CTA
// placement measured best wherever that fits one wave); for up to 8 tokens, a shape that does not fit that way is
// sized by its 8 staged rows with up to KS_MAX stages (more CTAs per SM). A grid under 7/8 of a wave reduces the
// splits in a cluster per tile, a fuller one through the fixup buffer (at most `cap` slots). Returns
// cudaErrorNotSupported when no sizing gives a one-wave grid, for two token tiles over more CTAs than two per SM, or
// when the slots do not fit (the caller then uses the tensor-memory kernel).
// A decode-kernel instantiation (two token tiles, four ring stages) with its attributes set: the dynamic shared
// memory limit for its largest sizing and the largest carveout (several CTAs per SM need it).
static void* rf_kernel(bool two, bool four, cudaError_t* e) {
    using namespace w8rf;
    void* kern = two ? (four ? (void*)w8g_rf_kernel<true, NST_SHORT> : (void*)w8g_rf_kernel<true, 3>)
                     : (four ? (void*)w8g_rf_kernel<false, NST_SHORT> : (void*)w8g_rf_kernel<false, 3>);
    *e = qf::ensure_smem_attr(kern, smem_bytes(KS_MAX, 16, four ? NST_SHORT : 3));
    if (*e != cudaSuccess) return nullptr;
    static bool carveout_set[2][2] = {{false, false}, {false, false}};
    if (!carveout_set[two][four]) {
        *e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                  (int)cudaSharedmemCarveoutMaxShared);
        if (*e != cudaSuccess) return nullptr;
        carveout_set[two][four] = true;
    }
    return kern;
}

// CTAs of that instantiation one SM holds at once with `smem` bytes of dynamic shared memory, as the runtime counts
// them (registers, shared memory and its per-CTA reservation); cached per (device, instantiation, size). 0 on error.
static int rf_ctas_per_sm(bool two, bool four, int smem) {
    static std::mutex mu;
    static std::map<std::tuple<int, int, int, int>, int> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    const auto key = std::make_tuple(dev, (int)two, (int)four, smem);
    {
        std::lock_guard<std::mutex> lock(mu);
        const auto it = cache.find(key);
        if (it != cache.end()) return it->second;
    }
    cudaError_t e = cudaSuccess;
    void* kern = rf_kernel(two, four, &e);
    int n = 0;
    if (kern == nullptr || cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, w8rf::THREADS, (size_t)smem) !=
                               cudaSuccess) {
        (void)cudaGetLastError();
        return 0;
    }
    std::lock_guard<std::mutex> lock(mu);
    cache[key] = n;
    return n;
}

cudaError_t launch_w8g_rf(const void* q, const void* x, int ldx, const void* s, void* y, int ldy, float* fix,
                          uint32_t* cnt, long long cap, int M, int N, int K, int group, int sms, bool pdl, unsigned* err,
                          cudaStream_t st) {
    using namespace w8rf;
    const int tiles = (N + ROWS - 1) / ROWS, KT = K / SK;   // a last tile past N: rows of zeros
    // about two items per SM, at least ceil(KT / S_MAX) stages per item (the last split adds at most S_MAX slots)
    const long long target = 2LL * sms;
    // one wave (the CTAs resident at once on every SM, as the runtime counts them) only: grids of several waves gave run-to-run
    // differences in stress runs (cause not found), so longer splits are tried first and then the tensor-memory kernel
    int ks = 0, S = 0, smem = 0, rows_used = 16, nst = 3;
    long long wave = 0;
    auto wave_of = [&](int kk, int rows, int stages) {   // the CTAs resident at once on the whole GPU
        return (long long)sms * rf_ctas_per_sm(M > 8, stages == NST_SHORT, smem_bytes(kk, rows, stages));
    };
    auto pick = [&](int rows, int ks_max) {   // smem sized for `rows` staged token rows, at most ks_max stages
        int k = (int)std::min<long long>(ks_max, ((long long)tiles * KT + target - 1) / target);
        k = std::max(std::max(1, k), (KT + S_MAX - 1) / S_MAX);
        if (k > ks_max) return false;   // K above ks_max * S_MAX * 128
        while (k < ks_max && (long long)tiles * ((KT + k - 1) / k) > wave_of(k, rows, 3)) ++k;
        ks = k;
        S = (KT + k - 1) / k;
        wave = wave_of(k, rows, 3);
        smem = smem_bytes(k, rows, 3);
        rows_used = rows;
        return (long long)tiles * S <= wave;
    };
    if (!pick(16, 12) && !(M <= 8 && pick(8, KS_MAX))) return cudaErrorNotSupported;
    // a ring of four stages for short items, where the grid still fits one wave with it (measured: 7-16 % faster for
    // items of at most KS_SHORT stages, 3-5 % slower for longer ones)
    if (ks <= KS_SHORT && (long long)tiles * S <= wave_of(ks, rows_used, NST_SHORT)) {
        nst = NST_SHORT;
        wave = wave_of(ks, rows_used, NST_SHORT);
        smem = smem_bytes(ks, rows_used, NST_SHORT);
    }
    // two token tiles over more than two CTAs per SM: the tensor-memory kernel (one stream per SM) is faster there
    if (M > 8 && (long long)tiles * S > target) return cudaErrorNotSupported;
    // clusters when the grid fills at most 7/8 of the wave: a fuller wave leaves clusters that find no room in a GPC
    // (measured); else the fixup buffer
    const int cl = S > 1 && (long long)tiles * S * 8 <= wave * 7 ? 1 : 0;
    if (!cl && (long long)tiles * S > cap) return cudaErrorNotSupported;
    qf::EncodeTiled enc = nullptr;
    cudaError_t e = qf::encode_tiled_fn(&enc);
    if (e != cudaSuccess) return e;
    Params p{};
    const cuuint64_t gdim[2] = {(cuuint64_t)K, (cuuint64_t)N};
    const cuuint64_t gstride[1] = {(cuuint64_t)K};
    const cuuint32_t box[2] = {(cuuint32_t)SK, (cuuint32_t)ROWS};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult cr = enc(&p.wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(q), gdim, gstride, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return cudaErrorInvalidValue;
    p.x = static_cast<const __nv_bfloat16*>(x);
    p.s = static_cast<const __nv_bfloat16*>(s);
    p.y = static_cast<__nv_bfloat16*>(y);
    p.fix = fix;
    p.cnt = cnt;
    p.cl = cl;
    p.err = err;
    p.ldx = ldx; p.ldy = ldy; p.M = M; p.N = N; p.K = K; p.group = group; p.ks = ks; p.S = S; p.KT = KT;
    // (smem: the sizing picked above, at least what the kernel's layout for M uses)
    void* kern = rf_kernel(M > 8, nst == NST_SHORT, &e);
    if (kern == nullptr) return e;
    // with cl, the S splits of a tile are one cluster (S <= S_MAX = 8, the portable cluster size)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(tiles * S);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cl ? (unsigned)S : 1u;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    void* args[] = {&p};
    return cudaLaunchKernelExC(&cfg, kern, args);
}

template <int NT>
cudaError_t launch_w8g_tc(const CUtensorMap& map, const void* x, int ldx, const void* s, void* y, int ldy,
                          float* fixp, uint32_t* fixc, int M, int N, int K, int G, int t0, long long units, int sms,
                          bool pdl, unsigned* err, cudaStream_t st) {
    auto kern = w8g_tc_kernel<NT>;
    cudaError_t e = qf::ensure_smem_attr(reinterpret_cast<const void*>(kern), Cfg<NT>::SMEM);
    if (e != cudaSuccess) return e;
    // Cfg::MINB runs per SM (no run ever waits for another, so residency does not matter), at most one per unit;
    // several CTAs per SM need the largest shared-memory carveout (without the hint the driver may pick a smaller one)
    static bool carveout_set[3] = {false, false, false};
    const int ix = NT == 16 ? 0 : (NT == 32 ? 1 : 2);
    if (!carveout_set[ix]) {
        e = cudaFuncSetAttribute(reinterpret_cast<const void*>(kern), cudaFuncAttributePreferredSharedMemoryCarveout,
                                 (int)cudaSharedmemCarveoutMaxShared);
        if (e != cudaSuccess) return e;
        carveout_set[ix] = true;
    }
    // runs of at least ~4 units where the weight allows one run per SM (a run's fixed costs -- ring start, its
    // partial tiles -- then stay small next to its stream), up to MINB runs per SM
    const long long gmax = (long long)sms * Cfg<NT>::MINB;
    long long g = (units + 3) / 4;
    if (g < sms) g = sms;
    if (g > gmax) g = gmax;
    if (g > units) g = units;
    const int grid = (int)g;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(G_THREADS);
    cfg.dynamicSmemBytes = Cfg<NT>::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, map, static_cast<const __nv_bfloat16*>(x), ldx,
                              static_cast<const uint16_t*>(s), static_cast<__nv_bfloat16*>(y), ldy, fixp, fixc, M, N,
                              K, G, t0, err);
}

}  // namespace

cudaError_t qf::encode_tiled_fn(EncodeTiled* fn) {
    static EncodeTiled cached = nullptr;
    if (cached == nullptr) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q);
        if (e != cudaSuccess) return e;
        if (q != cudaDriverEntryPointSuccess || f == nullptr) return cudaErrorNotSupported;
        cached = reinterpret_cast<EncodeTiled>(f);
    }
    *fn = cached;
    return cudaSuccess;
}

extern "C" int qf_w8g_fixup_elems(int N, int64_t* elems) {
    QF_REQUIRE(elems && N >= 8 && N % 8 == 0, "w8g_fixup_elems: N must be a multiple of 8, got %d", N);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return qf::cuda_status(e, "w8g_fixup_elems: cudaGetDevice");
    const int sms = qf::sm_count(dev);
    QF_REQUIRE(sms > 0, "w8g_fixup_elems: cannot query the SM count");
    // two float partial slots per run (runs: 4 per SM for up to 16 tokens, 2 per SM with 64 tokens x 128 rows per
    // slot for more), then one counter per 128-row tile
    *elems = (int64_t)sms * 2 * 4 * 16 * G_UN;
    if ((int64_t)sms * 2 * 2 * 64 * G_UN > *elems) *elems = (int64_t)sms * 2 * 2 * 64 * G_UN;
    *elems += (N + G_UN - 1) / G_UN;
    return QF_OK;
}

extern "C" int qf_w8g_gemm(const void* x, int64_t ldx, const int8_t* q, const void* s, void* y, int64_t ldy, int M,
                           int N, int K, int group, int rpw, float* fix, int64_t fix_elems, int pdl,
                           qf_stream_t stream) {
    // rpw: the reference's path bits (qf_w8g.cu:315-318) -- 0x100 forces its tensor-core kernel, 0x200 forbids it;
    // here they force / forbid the tensor-memory kernel (the register-fragment kernel otherwise takes decode shapes).
    // The low byte (the reference's rows per warp of its CUDA-core kernel) has no counterpart.
    const bool force_tm = (rpw & 0x100) != 0, forbid_tm = (rpw & 0x200) != 0;
    QF_REQUIRE(!(force_tm && forbid_tm), "w8g_gemm: rpw cannot both force (0x100) and forbid (0x200) the tensor-memory kernel");
    QF_REQUIRE(x && q && s && y && fix, "w8g_gemm: null pointer argument");
    QF_REQUIRE(M >= 1 && M <= QF_MAX_TOKENS, "w8g_gemm: M must be in [1, %d], got %d", QF_MAX_TOKENS, M);
    QF_REQUIRE(N >= 8 && N % 8 == 0, "w8g_gemm: N must be a multiple of 8, got %d", N);
    QF_REQUIRE(K >= 64 && K % 64 == 0 && K <= (1 << 20), "w8g_gemm: K must be a multiple of 64, got %d", K);
    QF_REQUIRE(group == 128 || group == 64, "w8g_gemm: group must be 128 or 64, got %d", group);
    QF_REQUIRE(K % group == 0, "w8g_gemm: K must be a multiple of the group size");
    QF_REQUIRE(ldx >= K && ldx % 8 == 0 && ldx <= INT32_MAX && qf::aligned(x, 16),
               "w8g_gemm: x needs a row stride %% 8 == 0 and 16-byte alignment");
    QF_REQUIRE(ldy >= N && ldy <= INT32_MAX && qf::aligned(q, 16) && qf::aligned(fix, 16),
               "w8g_gemm: bad y stride or unaligned q / fix");
    int64_t need = 0;
    int rc = qf_w8g_fixup_elems(N, &need);
    if (rc != QF_OK) return rc;
    QF_REQUIRE(fix_elems >= need, "w8g_gemm: the fixup buffer needs %lld floats, got %lld", (long long)need,
               (long long)fix_elems);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return qf::cuda_status(e, "w8g_gemm: cudaGetDevice");
    unsigned* err = nullptr;
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&err), g_w8g_err);
    if (e != cudaSuccess) return qf::cuda_status(e, "w8g_gemm: status word");
    const int sms = qf::sm_count(dev);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    float* fixp = fix;
    const int ntiles = (N + G_UN - 1) / G_UN;
    uint32_t* fixc = reinterpret_cast<uint32_t*>(fix + (need - ntiles));
    if (!force_tm && M <= 16 && K % w8rf::SK == 0) {   // decode token counts: the register-fragment kernel
        e = launch_w8g_rf(q, x, (int)ldx, s, y, (int)ldy, fixp, fixc, (need - ntiles) / w8rf::PART, M, N, K, group,
                          sms, pdl != 0, err, st);
        if (e != cudaErrorNotSupported) return qf::cuda_status(e, "w8g_gemm: launch");
    }
    if (forbid_tm) {
        qf::set_error("w8g_gemm: rpw 0x200 forbids the tensor-memory kernel, and the register-fragment kernel does not "
                      "take M %d, N %d, K %d (it needs M <= 16, K %% 128 == 0 and a one-wave split)", M, N, K);
        return QF_ERR_UNSUPPORTED;
    }
    qf::EncodeTiled enc = nullptr;
    e = qf::encode_tiled_fn(&enc);
    if (e != cudaSuccess) return qf::cuda_status(e, "w8g_gemm: cuTensorMapEncodeTiled entry point");
    // the canonical weight as a 2-D tensor (K bytes per row); one box = one unit (64 k x 128 rows), 64-byte swizzle
    CUtensorMap map;
    const cuuint64_t gdim[2] = {(cuuint64_t)K, (cuuint64_t)N};
    const cuuint64_t gstride[1] = {(cuuint64_t)K};
    const cuuint32_t box[2] = {(cuuint32_t)G_UK, (cuuint32_t)G_UN};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult cr = enc(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(q), gdim, gstride, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    QF_REQUIRE(cr == CUDA_SUCCESS, "w8g_gemm: cuTensorMapEncodeTiled failed (%d)", (int)cr);
    const long long units = (long long)ntiles * (K / G_UK);
    const int NT = M <= 16 ? 16 : (M <= 32 ? 32 : 64);
    if (NT == 16) e = launch_w8g_tc<16>(map, x, (int)ldx, s, y, (int)ldy, fixp, fixc, M, N, K, group, 0, units, sms, pdl != 0, err, st);
    else if (NT == 32) e = launch_w8g_tc<32>(map, x, (int)ldx, s, y, (int)ldy, fixp, fixc, M, N, K, group, 0, units, sms, pdl != 0, err, st);
    else e = launch_w8g_tc<64>(map, x, (int)ldx, s, y, (int)ldy, fixp, fixc, M, N, K, group, 0, units, sms, pdl != 0, err, st);
    return qf::cuda_status(e, "w8g_gemm: launch");
}

extern "C" int qf_w8g_take_status(uint32_t* status) {
    QF_REQUIRE(status, "w8g_take_status: null pointer argument");
    unsigned v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_w8g_err, sizeof(unsigned));
    if (e != cudaSuccess) return qf::cuda_status(e, "w8g_take_status");
    const unsigned zero = 0;
    e = cudaMemcpyToSymbol(g_w8g_err, &zero, sizeof(unsigned));
    *status = v;
    return qf::cuda_status(e, "w8g_take_status");
}
