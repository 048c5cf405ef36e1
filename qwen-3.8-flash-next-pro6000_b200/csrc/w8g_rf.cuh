// W8A16 group-scaled INT8 GEMM for decode token counts (M <= 16) on register fragments: mma.sync m16n8k16 with fp16
// operands, fp32 accumulation. Included by w8g_tc.cu (it shares that file's status word and helpers); qf_w8g_gemm
// routes M <= 16 with K % 128 == 0 here and everything else to the tensor-memory kernel.
//
//   y[t, n] = bf16( sum over 64-k halves h of  s[n, g(h)] * 2^e[t, h] * sum_{k in h} q[n, k] * x16[t, k] )
//
// where x16[t, k] = fp16(x[t, k] * 2^-e[t, h]) and e[t, h] = floor(log2 max|x[t, h]|) - 14 (clamped), so the slice's
// largest value lands in [2^14, 2^15): the conversion is exact down to 2^-31 of that maximum, and the int8 weights are
// exact in fp16 (i8x4_to_f16), so every product is exact and only the fp32 sums round -- the arithmetic of
// serve/qwenfast/qf_w8g.cu:47-139 (fp32 group sums times the group scale) up to fp32 association.
//
// Structure (a weight stream, like the decode MoE kernel's register path):
//   * One CTA per item = (128-row tile, split of the K stages): the tiles' K / 128 stages are cut into S splits of ks
//     stages each, S chosen so that the grid covers the GPU about two CTAs deep (S <= S_MAX). 160 threads: warps 0-3 consume,
//     warp 4 (one lane) is the producer.
//   * Producer: a ring of 16 KB weight stages, 3 deep (4 for items of at most 5 stages), each 128 rows x 128 k, one
//     TMA 2-D tile with 128-byte swizzle (the four 16-byte chunks a lane reads are spread over all banks), requested
//     before griddepcontrol.wait (the weights are load-time data).
//   * Consumers, first: the item's token slices (fp16 with the per-(token, 64-k) exponent, 16-byte chunks swizzled by
//     token) and group scales into shared memory; then per stage and 64-k half, warp w runs the m16 tiles 2w, 2w + 1:
//     one 16-byte load per row and half gives the four k16 steps of that row (k = 64 h + 16 t4 + 4 s + 0..3 in the
//     mma columns 2 t4, 2 t4 + 1, 2 t4 + 8, 2 t4 + 9, the same permutation for the tokens), a second n8 token tile
//     only above 8 tokens. Each half's fp32 partial is scaled by s[row] * 2^e[token] into the accumulators.
//   * When the grid is one wave, the S splits of one tile run as one thread-block cluster: each CTA leaves its fp32
//     partial in its shared memory, and cluster rank 0 adds the S partials in split order through distributed shared
//     memory and writes y (no global round trip). Larger grids (cluster placement costs them more than it saves)
//     reduce through the fixup buffer instead: each item stores its partial to its own slot and counts itself on the
//     tile's counter; the item that counts last adds all slots in split order and re-arms the counter. Either way
//     the sum is the same whichever split finishes last.
//   * Every wait is bounded; a wait that runs out sets a bit of the status word (qf_w8g_take_status).
#pragma once

namespace w8rf {

constexpr int THREADS = 160;
constexpr int ROWS = 128;                 // weight rows per tile
constexpr int SK = 128;                   // k per stage
constexpr int STAGE = ROWS * SK;          // 16 KB of int8
constexpr int NST_SHORT = 4;              // ring stages for items of at most KS_SHORT stages (else 3)
constexpr int KS_SHORT = 5;
constexpr int KS_MAX = 16;                // stages per item
constexpr int S_MAX = 8;                  // splits per tile
constexpr int PART = 16 * ROWS;           // floats of one fixup slot (16 per consumer thread)
constexpr uint64_t WAIT_NS = 2000000000ull;

// shared memory (base aligned to 1024 for the swizzled TMA tiles), nst = the ring stages, mt = the staged token
// rows (8, or 16 with the second n8 token tile): ring [nst][STAGE] | tokens [ks][2 halves][mt][128 B] (fp16) |
// factors float [ks][2][mt] | scales float [ks][2][ROWS] | full[nst], empty[nst] | flag
__host__ __device__ constexpr int off_tok(int nst) { return nst * STAGE; }
__host__ __device__ constexpr int off_fac(int ks, int mt, int nst) { return off_tok(nst) + ks * 2 * mt * 128; }
__host__ __device__ constexpr int off_sc(int ks, int mt, int nst) { return off_fac(ks, mt, nst) + ks * 2 * mt * 4; }
__host__ __device__ constexpr int off_bar(int ks, int mt, int nst) { return off_sc(ks, mt, nst) + ks * 2 * ROWS * 4; }
__host__ __device__ constexpr int smem_bytes(int ks, int mt, int nst) {
    return off_bar(ks, mt, nst) + 2 * nst * 8 + 16 + 1024;
}

struct Params {
    CUtensorMap wmap;   // q [N, K] uint8; box 128 k x 128 rows, 128-byte swizzle
    const __nv_bfloat16* x;
    const __nv_bfloat16* s;
    __nv_bfloat16* y;
    float* fix;         // split partials (cl == 0): one PART slot per item, then
    uint32_t* cnt;      // one counter per tile, left at zero
    unsigned* err;
    int ldx, ldy, M, N, K, group, ks, S, KT;
    int cl;             // 1: the splits of a tile are one thread-block cluster and reduce through its shared memory
};

__device__ __forceinline__ float pow2f(int k) { return __uint_as_float((uint32_t)(127 + k) << 23); }

// thread-block cluster helpers: a full barrier (release / acquire), this CTA's rank, another rank's address of a
// shared-memory location, and a 16-byte load from it
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t map_rank(uint32_t addr, int rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr)
                 : "memory");
    return v;
}

template <bool TWO, int NST>
__global__ void __launch_bounds__(THREADS) w8g_rf_kernel(const __grid_constant__ Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ks = p.ks;
    uint8_t* ring = smem;
    constexpr int MT = TWO ? 16 : 8;   // staged token rows
    uint8_t* tok = smem + off_tok(NST);
    float* fac = reinterpret_cast<float*>(smem + off_fac(ks, MT, NST));
    float* sc = reinterpret_cast<float*>(smem + off_sc(ks, MT, NST));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + off_bar(ks, MT, NST));
    uint64_t* empty = full + NST;
    int* flag = reinterpret_cast<int*>(empty + NST);
    const int item = blockIdx.x, tile = item / p.S, split = item - tile * p.S;
    const int j0 = split * ks, nks = min(ks, p.KT - j0);   // this item's stages: K stages j0 .. j0 + nks - 1
    if (tid == 0) {
        for (int i = 0; i < NST; ++i) {
            qf::mbar_init(full + i, 1);
            qf::mbar_init(empty + i, 4);
        }
        qf::mbar_fence_init();
    }
    __syncthreads();

    if (warp == 4) {
        // ------------------------------------------------------------------ producer (one lane)
        if (lane == 0) {
            const uint64_t pol = qf::policy_evict_first();
            for (int j = 0; j < nks; ++j) {
                const int st = j % NST;
                if (j >= NST && !qf::mbar_wait(empty + st, ((j / NST) - 1) & 1, WAIT_NS)) atomicOr(p.err, 16u);
                qf::mbar_arrive_expect_tx(full + st, STAGE);
                tma_load_2d(ring + st * STAGE, &p.wmap, (j0 + j) * SK, tile * ROWS, full + st, pol);
            }
        }
        if (p.S == 1 || !p.cl) return;
        // splits reduced in the cluster: this warp joins the cluster barriers below
        cluster_sync();
        cluster_sync();
        return;
    }

    // ---------------------------------------------------------------------- consumers (128 threads)
    qf::pdl_wait();   // x comes from the previous kernel
    const int M = p.M, kb = j0 * SK;
    // token slices: 8 threads per (stage, half, token) slice of 64 k, thread c the 16-byte chunk c (k 8c .. 8c + 7)
    {
        const int c = tid & 7, nsl = nks * 2 * M;
        for (int sl0 = 0; sl0 < nsl; sl0 += ROWS / 8 * 4) {
            uint4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {   // four slices in flight per thread
                const int sl = sl0 + u * (ROWS / 8) + (tid >> 3);
                v[u] = make_uint4(0u, 0u, 0u, 0u);
                if (sl < nsl) {
                    const int t = sl % M, jh = sl / M;   // jh = stage * 2 + half
                    v[u] = __ldcg(reinterpret_cast<const uint4*>(p.x + (size_t)t * p.ldx + kb + jh * 64 + c * 8));
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int sl = sl0 + u * (ROWS / 8) + (tid >> 3);   // uniform within each group of 8 lanes
                const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
                uint32_t mx = 0u;   // largest |x| as a bit pattern (monotone for non-negative floats)
#pragma unroll
                for (int i = 0; i < 4; ++i) mx = max(mx, max((w[i] << 16) & 0x7FFF0000u, w[i] & 0x7FFF0000u));
#pragma unroll
                for (int o = 1; o < 8; o <<= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                if (sl < nsl) {
                    const int t = sl % M, jh = sl / M;
                    const int ex = mx == 0u ? 0 : max(-110, min(110, (int)(mx >> 23) - 127 - 14));
                    const float mul = pow2f(-ex);
                    uint32_t o[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const __half2 h2 = __floats2half2_rn(qf::bf16_lo(w[i]) * mul, qf::bf16_hi(w[i]) * mul);
                        o[i] = *reinterpret_cast<const uint32_t*>(&h2);
                    }
                    *reinterpret_cast<uint4*>(tok + jh * (MT * 128) + t * 128 + ((c ^ (t & 7)) * 16)) =
                        make_uint4(o[0], o[1], o[2], o[3]);
                    if (c == 0) fac[jh * MT + t] = pow2f(ex);
                }
            }
        }
        // group scales of row tid (one per half: a 128-group gives both halves the same scale), all requested at once
        const __nv_bfloat16* srow = p.s + (size_t)min(tile * ROWS + tid, p.N - 1) * (p.K / p.group);   // rows past N: 0
        __nv_bfloat16 sv[2 * KS_MAX];
#pragma unroll
        for (int jh = 0; jh < 2 * KS_MAX; ++jh)
            if (jh < 2 * nks) sv[jh] = tile * ROWS + tid < p.N ? srow[(kb + jh * 64) / p.group] : __float2bfloat16(0.f);
#pragma unroll
        for (int jh = 0; jh < 2 * KS_MAX; ++jh)
            if (jh < 2 * nks) sc[jh * ROWS + tid] = __bfloat162float(sv[jh]);
    }
    qf::named_bar(1, ROWS);

    const int rw = warp, g = lane >> 2, t4 = lane & 3;
    float acc[4][4];   // acc[2 m + n][i]: row 16 (2 rw + m) + g + 8 (i / 2), token 8 n + 2 t4 + (i % 2)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    bool ok = true;
    for (int j = 0; j < nks; ++j) {
        const int st = j % NST;
        if (ok && !qf::mbar_wait(full + st, (j / NST) & 1, WAIT_NS)) {
            atomicOr(p.err, 32u);
            ok = false;
        }
        const uint8_t* wb = ring + st * STAGE;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint8_t* tb = tok + (j * 2 + h) * (MT * 128);
            const uint4 x0a = *reinterpret_cast<const uint4*>(tb + g * 128 + (((2 * t4) ^ g) * 16));
            const uint4 x0b = *reinterpret_cast<const uint4*>(tb + g * 128 + (((2 * t4 + 1) ^ g) * 16));
            uint4 x1a = make_uint4(0u, 0u, 0u, 0u), x1b = x1a;
            if constexpr (TWO) {
                x1a = *reinterpret_cast<const uint4*>(tb + (8 + g) * 128 + (((2 * t4) ^ g) * 16));
                x1b = *reinterpret_cast<const uint4*>(tb + (8 + g) * 128 + (((2 * t4 + 1) ^ g) * 16));
            }
            const uint32_t xw0[8] = {x0a.x, x0a.y, x0a.z, x0a.w, x0b.x, x0b.y, x0b.z, x0b.w};
            const uint32_t xw1[8] = {x1a.x, x1a.y, x1a.z, x1a.w, x1b.x, x1b.y, x1b.z, x1b.w};
            const float* fh = fac + (j * 2 + h) * MT;
            const float f00 = fh[2 * t4], f01 = fh[2 * t4 + 1];
            const float f10 = TWO ? fh[8 + 2 * t4] : 0.f, f11 = TWO ? fh[9 + 2 * t4] : 0.f;
#pragma unroll
            for (int m = 0; m < 2; ++m) {
                const int r0 = 16 * (2 * rw + m) + g;
                const uint4 wa = *reinterpret_cast<const uint4*>(wb + r0 * SK + (((4 * h + t4) ^ g) * 16));
                const uint4 wc = *reinterpret_cast<const uint4*>(wb + (r0 + 8) * SK + (((4 * h + t4) ^ g) * 16));
                const uint32_t aw[4] = {wa.x, wa.y, wa.z, wa.w}, cw[4] = {wc.x, wc.y, wc.z, wc.w};
                float d0[4], d1[4];
#pragma unroll
                for (int s = 0; s < 4; ++s) {
                    uint32_t a0, a2, a1, a3;
                    i8x4_to_f16(aw[s], a0, a2);   // row r0: k + 0|1, k + 2|3
                    i8x4_to_f16(cw[s], a1, a3);   // row r0 + 8
                    if (s == 0) {
                        qf::mma_f16_z(d0, a0, a1, a2, a3, xw0[0], xw0[1]);
                        if constexpr (TWO) qf::mma_f16_z(d1, a0, a1, a2, a3, xw1[0], xw1[1]);
                    } else {
                        qf::mma_f16(d0, a0, a1, a2, a3, xw0[2 * s], xw0[2 * s + 1]);
                        if constexpr (TWO) qf::mma_f16(d1, a0, a1, a2, a3, xw1[2 * s], xw1[2 * s + 1]);
                    }
                }
                const float* sh = sc + (j * 2 + h) * ROWS;
                const float s0 = sh[r0], s1 = sh[r0 + 8];
                acc[2 * m][0] = fmaf(d0[0], s0 * f00, acc[2 * m][0]);
                acc[2 * m][1] = fmaf(d0[1], s0 * f01, acc[2 * m][1]);
                acc[2 * m][2] = fmaf(d0[2], s1 * f00, acc[2 * m][2]);
                acc[2 * m][3] = fmaf(d0[3], s1 * f01, acc[2 * m][3]);
                if constexpr (TWO) {
                    acc[2 * m + 1][0] = fmaf(d1[0], s0 * f10, acc[2 * m + 1][0]);
                    acc[2 * m + 1][1] = fmaf(d1[1], s0 * f11, acc[2 * m + 1][1]);
                    acc[2 * m + 1][2] = fmaf(d1[2], s1 * f10, acc[2 * m + 1][2]);
                    acc[2 * m + 1][3] = fmaf(d1[3], s1 * f11, acc[2 * m + 1][3]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) qf::mbar_arrive(empty + st);
    }
    qf::pdl_launch_dependents();

    // ---------------------------------------------------------------------- epilogue
    const int ctid = tid;
    auto store_y = [&](const float (&a)[4][4]) {
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
            for (int n = 0; n < (TWO ? 2 : 1); ++n)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int t = 8 * n + 2 * t4 + (i & 1);
                    const int yrow = tile * ROWS + 16 * (2 * rw + m) + g + 8 * (i >> 1);
                    if (t < M && yrow < p.N) p.y[(size_t)t * p.ldy + yrow] = __float2bfloat16(a[2 * m + n][i]);
                }
    };
    if (p.S == 1) {
        store_y(acc);
        return;
    }
    if (!p.cl) {
        // splits in separate CTAs (grids of several waves): each item stores its fp32 partial to its fixup slot and
        // counts itself on the tile's counter; the item that counts last adds the slots in split order (the same
        // sum whichever split comes last), writes y and re-arms the counter
        float* mine = p.fix + (size_t)item * PART + ctid * 16;
#pragma unroll
        for (int j = 0; j < 4; ++j)
            __stcg(reinterpret_cast<float4*>(mine + 4 * j), make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]));
        __threadfence();
        qf::named_bar(1, ROWS);
        if (ctid == 0) {
            const bool last = atomicAdd(p.cnt + tile, 1u) == (uint32_t)(p.S - 1);
            if (last) {
                __threadfence();
                p.cnt[tile] = 0u;
            }
            *flag = last ? 1 : 0;
        }
        qf::named_bar(1, ROWS);
        if (*flag == 0) return;
        __threadfence();
        float tot[4][4];
        const float* part = p.fix + (size_t)tile * p.S * PART + ctid * 16;
#pragma unroll
        for (int ps = 0; ps < 2; ++ps) {   // two passes of 8 floats, every split's loads in flight
            float4 q[S_MAX][2];
#pragma unroll
            for (int sp = 0; sp < S_MAX; ++sp)
                if (sp < p.S) {
#pragma unroll
                    for (int j = 0; j < 2; ++j)
                        q[sp][j] = __ldcg(reinterpret_cast<const float4*>(part + (size_t)sp * PART + 4 * (2 * ps + j)));
                }
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                float4 a = q[0][j];
#pragma unroll
                for (int sp = 1; sp < S_MAX; ++sp)
                    if (sp < p.S) {
                        a.x += q[sp][j].x; a.y += q[sp][j].y; a.z += q[sp][j].z; a.w += q[sp][j].w;
                    }
                tot[2 * ps + j][0] = a.x; tot[2 * ps + j][1] = a.y; tot[2 * ps + j][2] = a.z; tot[2 * ps + j][3] = a.w;
            }
        }
        store_y(tot);
        return;
    }
    // several splits of this tile run as one thread-block cluster (cluster rank = split): each CTA leaves its fp32
    // partial in its own shared memory (the ring, free once every consumer warp is past its last stage), and rank 0
    // adds the S partials in split order through distributed shared memory -- the same sum for every schedule
    qf::named_bar(1, ROWS);
    float* red = reinterpret_cast<float*>(ring) + ctid * 16;
#pragma unroll
    for (int j = 0; j < 4; ++j)
        *reinterpret_cast<float4*>(red + 4 * j) = make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
    cluster_sync();
    if (cluster_rank() == 0) {
        float tot[4][4];
        const uint32_t mine = qf::smem_u32(red);
#pragma unroll
        for (int ps = 0; ps < 2; ++ps) {   // two passes of 8 floats, every split's loads in flight
            float4 q[S_MAX][2];
#pragma unroll
            for (int sp = 0; sp < S_MAX; ++sp)
                if (sp < p.S) {
                    const uint32_t ra = map_rank(mine, sp);
#pragma unroll
                    for (int j = 0; j < 2; ++j) q[sp][j] = ld_cluster_f4(ra + 16u * (2 * ps + j));
                }
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                float4 a = q[0][j];
#pragma unroll
                for (int sp = 1; sp < S_MAX; ++sp)
                    if (sp < p.S) {
                        a.x += q[sp][j].x; a.y += q[sp][j].y; a.z += q[sp][j].z; a.w += q[sp][j].w;
                    }
                tot[2 * ps + j][0] = a.x; tot[2 * ps + j][1] = a.y; tot[2 * ps + j][2] = a.z; tot[2 * ps + j][3] = a.w;
            }
        }
        store_y(tot);
    }
    cluster_sync();   // every CTA keeps its shared memory until rank 0 has read it
}

}  // namespace w8rf
