// Decode-size (1..64 tokens) W4A16 routed experts + shared expert + top-k combine in ONE persistent launch.
//
// Reference behaviour: serve/qwenfast/qf_a16moe.cu (persistent mode :342-837, host :852-922): gemm1 (gate_up) +
// SwiGLU, gemm2 (down) with the top-k weight, a top-k-ordered combine per 128-column tile, and the sigmoid-gated
// shared expert. Rounding points (qf_a16moe.cu:2-4):
//   h  = bf16(silu(bf16(bf16(acc_gate) * gs13)) * bf16(bf16(acc_up) * gs13))
//   y  = bf16(bf16(acc_down) * bf16(gs2 * bf16(topk_w)))            one slot per (token, top-k position)
//   out = bf16(sigmoid(x . w_gate) * shared + bf16(sum_kpos y))      fp32 sum in top-k order
// Expert weights are int4 codes (zero point 8) with one bf16 scale per 128 k: each 128-k group is reduced on the
// tensor cores in fp32 and then scaled once (exact products, no per-weight scale multiply).
//
// B200 structure
//   * 2 CTAs per SM (296), 9 warps each: warp 8 lane 0 is the producer, warp 8 lane 1 the signal agent, warps 0..7
//     are consumers.
//   * Work items, claimed in order from a global queue:
//       GL  shared-expert gate logits          S1  shared gate_up tile, one of 4 k-splits, one 16-token group
//       G1  expert u gate_up tile + group      S1F shared gate_up split-K sum + SwiGLU
//       S2  shared down tile + group           G2  expert u down tile + group
//       CB  top-k combine of one 128-column tile (+ gated shared term)
//     An item only depends on items claimed before it, so the queue cannot deadlock.
//   * The producer streams each item through an NST-stage shared-memory ring with 1-D bulk copies (TMA engine,
//     mbarrier completion): per stage 16 KB of weights (128 rows x 256 k int4, or x 64 k bf16), their scales, and
//     the matching k-slice of the item's token rows (x for gate_up, h for down). Every cross-CTA dependency
//     (gate_up -> down, split-K -> finalize -> shared down, all producers of a column tile -> combine) is waited on
//     by the producer (bounded) before it fills the stage, so consumers never spin on other CTAs.
//   * Consumers signal completed items through a CTA-local ring; the agent lane turns each record into one gpu-scope
//     release (fence + atomic add) on the control block. Consumer warps never execute a gpu-scope fence.
//   * Contraction on the 5th-generation tensor cores (tcgen05). int4 tiles: every consumer thread owns one TMEM lane
//     (= one weight row of the 128-row tile) and one 128-k half of the stage; it turns each int4 word into four
//     bf16x2 of the biased codes (128 + code; one lop3 each) and stores them to TMEM (tcgen05.st) as the A operand.
//     The gathered token rows are re-laid by the consumers into the canonical K-major shared-memory layout (B,
//     N = 16). One elected thread issues tcgen05.mma kind::f16 (A in TMEM, B in SMEM, fp32 D in TMEM) per k16 step
//     plus one against a constant -136 A tile that removes the bias, then tcgen05.commit. Each 128-k group has its
//     own D region; its fp32 partial is read back (tcgen05.ld) and scaled once by the row's group scale.
//     bf16 tiles (shared expert): the stage itself is the A operand (SMEM descriptor), D accumulates in TMEM over the
//     whole item. gate_up tiles interleave gate row j (even lane) and up row j (odd lane): SwiGLU is one shuffle.
//   * The routing plan (unique experts, per-expert token lists, group offsets) is rebuilt identically by every CTA
//     from topk_ids with shared-memory atomics (token bit masks), so no CTA waits for a plan.
//   * Every wait is bounded (globaltimer); a wait that runs out sets QF_MOE_ERR_* in ctrl and the kernel drains.
#include "qf_common.cuh"

namespace {

using qf::bf16_bits;
using qf::bf16_hi;
using qf::bf16_lo;
using qf::bf16r;

constexpr int NCW = 8;                        // consumer warps
constexpr int MOE_THREADS = (NCW + 1) * 32;   // + the producer / agent warp
constexpr int CONS_THREADS = NCW * 32;
constexpr int CTAS_PER_SM = 2;
constexpr int TG = 16;                        // tokens per token group (two n8 tiles)
constexpr int NST = 3;                        // pipeline stages per CTA
constexpr int NEPI = 8;                       // completion-record ring
constexpr int W4_KC = 256;                    // int4 k per stage
constexpr int BF_KC = 64;                     // bf16 k per stage
constexpr int STAGE_W = 16384;                // weight bytes of a full stage
constexpr int STAGE_S = 512;                  // scale bytes of a full int4 stage
constexpr int STAGE_X = TG * (W4_KC + 8) * 2; // token rows of a stage (row stride kc + 8 elements)
constexpr int STAGE_BYTES = STAGE_W + STAGE_S + STAGE_X;
constexpr int NSPLIT = 4;                     // split-K of the shared expert's gate_up
constexpr int MAXSLOTS = QF_MAX_TOKENS * QF_MAX_TOPK;
constexpr uint64_t DEP_WAIT_NS = 1000000000ull;    // cross-CTA dependency waits
constexpr uint64_t PIPE_WAIT_NS = 4000000000ull;   // ring waits (longer: they cover the dependency waits)

// control block words
enum : int {
    C_QUEUE = 0,
    C_EXIT = 1,
    C_GLF = 2,
    C_ERR = QF_MOE_CTRL_ERR,
    C_CNT = 8,      // [64] column-tile arrivals
    C_SDONE = 72,   // [4] finished shared gate_up tiles per token group
    C_SPLIT = 80,   // [64] split-K arrivals per (shared tile, token group)
    C_DONE = 160,   // [QF_MAX_EXPERTS] finished gate_up items per unique expert
};
static_assert(C_DONE + QF_MAX_EXPERTS <= QF_MOE_CTRL_WORDS, "ctrl layout");

enum : int { K_STOP = 0, K_GL, K_S1, K_G1, K_S1F, K_S2, K_G2, K_CB };

struct StageDesc {
    int16_t kind, u, tile, tg, split, kidx, nk, kc, ntok, pad[3];
};
struct EpiRec {     // one completion record: add `add` to ctrl[idx] (idx < 0: nothing; kind STOP ends the agent)
    int idx, add;
};

struct Params {
    const __nv_bfloat16* x;
    const int* ids;
    const float* tw;
    const uint8_t* w13;
    const uint16_t* s13;
    const uint16_t* gs13;
    const uint8_t* w2;
    const uint16_t* s2;
    const uint16_t* gs2;
    const __nv_bfloat16* wgate;
    const __nv_bfloat16* shared;
    const uint8_t* shw13;
    const uint8_t* shw2;
    __nv_bfloat16* hbuf;
    __nv_bfloat16* ybuf;
    float* gl;
    uint32_t* ctrl;
    float* pbuf;
    __nv_bfloat16* hsh;
    __nv_bfloat16* sbuf;
    __nv_bfloat16* out;
    long long* dbg;
    int M, H, I, E, topk, Is, mode, elo, ehi;
};

// shared memory map (dynamic)
constexpr int BST_BYTES = TG * (W4_KC / 8) * 16;                      // B operand [k chunk][16 tokens][16 B]
constexpr int OFF_RING = 0;
constexpr int OFF_BST = OFF_RING + NST * STAGE_BYTES;
constexpr int OFF_BAR = OFF_BST + BST_BYTES;                          // full[NST], empty[NST], efull[NEPI], eempty[NEPI], mma
constexpr int OFF_DESC = OFF_BAR + (2 * NST + 2 * NEPI + 2) * 8;
constexpr int OFF_EPI = OFF_DESC + NST * (int)sizeof(StageDesc);
constexpr int OFF_PLAN = OFF_EPI + NEPI * (int)sizeof(EpiRec);
constexpr int PLAN_ULIST = 0;                                         // int16 [QF_MAX_EXPERTS]
constexpr int PLAN_GPRE = PLAN_ULIST + QF_MAX_EXPERTS * 2;            // int16 [QF_MAX_EXPERTS + 1]
constexpr int PLAN_TOFF = PLAN_GPRE + (QF_MAX_EXPERTS + 8) * 2;
constexpr int PLAN_TLIST = PLAN_TOFF + (QF_MAX_EXPERTS + 8) * 2;      // int16 [MAXSLOTS]
constexpr int PLAN_SIDS = PLAN_TLIST + MAXSLOTS * 2;                  // int16 [MAXSLOTS] copy of topk_ids
constexpr int PLAN_MISC = PLAN_SIDS + MAXSLOTS * 2;                   // int32 [64]
constexpr int PLAN_BYTES = PLAN_MISC + 64 * 4;
constexpr int MOE_SMEM = OFF_PLAN + PLAN_BYTES;
static_assert(CTAS_PER_SM * (MOE_SMEM + 1024) <= 228 * 1024, "two CTAs per SM must fit in shared memory");
// plan-build scratch aliases the ring (the producer starts after the plan is built)
constexpr int SCR_MASK = 0;                                        // uint64 [E]
constexpr int SCR_EXF = SCR_MASK + QF_MAX_EXPERTS * 8;             // int16 [E] x 3 (flag, count, groups) in-chunk
constexpr int SCR_TOFFE = SCR_EXF + 3 * QF_MAX_EXPERTS * 2;        // int16 [E] token offset per expert id
constexpr int SCR_CHUNK = SCR_TOFFE + QF_MAX_EXPERTS * 2;          // int32 [32] x 3 chunk totals
static_assert(SCR_CHUNK + 3 * 32 * 4 <= NST * STAGE_BYTES, "plan scratch");

enum : int { MISC_U = 0, MISC_NTOK = 1, MISC_GT = 2, MISC_FLAG = 3, MISC_DBGN = 5, MISC_TMEM = 6 };

// tensor memory map (columns of this CTA's allocation; fp32 / bf16x2 per 32-bit column, lane = tile row)
constexpr uint32_t TM_COLS = 256;
constexpr uint32_t TM_A = 0;       // 128 columns: A tile of one 256-k int4 stage (16 k16 steps x 8 columns)
constexpr uint32_t TM_D = 128;     // 2 x 16 columns: fp32 partial of each 128-k group (bf16 items: running sum)
constexpr uint32_t TM_C = 160;     // 8 columns: constant -136 A tile (bias removal)
constexpr uint32_t IDESC = qf::idesc_bf16(128, TG);

// Errors that stop the pipeline (waits that ran out). An out-of-range expert id is reported but not fatal: the
// slot is skipped and the rest of the layer is computed.
constexpr uint32_t HARD_ERR = QF_MOE_ERR_TIMEOUT | QF_MOE_ERR_PIPELINE;

__device__ __forceinline__ void set_err(uint32_t* ctrl, uint32_t bits) { atomicOr(ctrl + C_ERR, bits); }
__device__ __forceinline__ bool hard_error(uint32_t* ctrl) { return (qf::ld_volatile(ctrl + C_ERR) & HARD_ERR) != 0u; }

// Bounded wait until ctrl[idx] >= target (acquire). Gives up early when another CTA already recorded a hard error.
__device__ bool wait_counter(uint32_t* ctrl, int idx, uint32_t target) {
    if (qf::ld_acquire(ctrl + idx) >= target) return true;
    const uint64_t t0 = qf::globaltimer();
    while (qf::ld_acquire(ctrl + idx) < target) {
        if (hard_error(ctrl)) return false;
        if (qf::globaltimer() - t0 > DEP_WAIT_NS) {
            set_err(ctrl, QF_MOE_ERR_TIMEOUT);
            return false;
        }
        __nanosleep(64);
    }
    return true;
}

struct Layout {   // per-launch derived sizes, identical in every thread
    int R1, R2, Rs1, ngs, U, Gt, has_gate, has_shw;
    int b_s1, b_g1, b_s1f, b_s2, b_g2, b_cb, total;
    uint32_t tile_target;
};

__device__ __forceinline__ int find_u(const int16_t* gpre, int U, int key) {   // largest u with gpre[u] <= key
    int lo = 0, hi = U - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (gpre[mid] <= key) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// ---------------------------------------------------------------------------------------------- consumer math
// Copy the stage's token rows (row-major, stride kc + 8 elements) into the canonical K-major B layout
// [k chunk of 8][token (16)][16 bytes] (8-token core matrices: SBO = 128 B, k-chunk stride LBO = 256 B).
__device__ __forceinline__ void reshuffle_b(const uint8_t* stage, uint8_t* bst, int kc, int ntok, int ctid) {
    const int xrb = (kc + 8) * 2;
    const uint8_t* xs = stage + STAGE_W + STAGE_S;
    const int nch = kc >> 3;
    for (int idx = ctid; idx < nch * ntok; idx += CONS_THREADS) {
        const int c = idx / ntok, n = idx - c * ntok;
        *reinterpret_cast<uint4*>(bst + (c * TG + n) * 16) = *reinterpret_cast<const uint4*>(xs + n * xrb + c * 16);
    }
    qf::fence_proxy_async_smem();   // the tensor cores read bst through the async proxy
}

// Dequantise this thread's row of its 128-k half of an int4 stage into TMEM (biased codes, natural k order):
// word w of the half (k = 8w .. 8w+7) becomes columns TM_A + 64 * half + 4w .. +4.
__device__ __forceinline__ void stage_w4_to_tmem(const uint8_t* stage, uint32_t tmem, int half, int quarter, int lane) {
    const int row = 32 * quarter + lane;
    const uint8_t* ws = stage + ((half * 4) * 128 + row) * 16;
    const uint32_t lane_base = (uint32_t)(32 * quarter) << 16;
#pragma unroll
    for (int qd = 0; qd < 4; ++qd) {
        const uint4 w = *reinterpret_cast<const uint4*>(ws + qd * 128 * 16);
        uint32_t v[16];
        qf::biased_w4(w.x, v + 0);
        qf::biased_w4(w.y, v + 4);
        qf::biased_w4(w.z, v + 8);
        qf::biased_w4(w.w, v + 12);
        qf::tmem_st16(tmem + lane_base + TM_A + 64 * half + 16 * qd, v);
    }
}

// Combine of one 128-column tile for all tokens: out = bf16(gate * shared + bf16(sum_kpos y)), 8 columns a thread.
__device__ void combine_tile(const Params& p, const Layout& L, const int16_t* sids, int c, int ctid) {
    const int H = p.H, topk = p.topk;
    for (int q = ctid; q < p.M * 16; q += CONS_THREADS) {
        const int t = q >> 4, n = 128 * c + 8 * (q & 15);
        float a[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) a[j] = 0.f;
        for (int kp = 0; kp < topk; ++kp) {
            const int s = t * topk + kp;
            const int e = sids[s];
            if (e < 0 || e < p.elo || e >= p.ehi) continue;
            const uint4 v = __ldcg(reinterpret_cast<const uint4*>(p.ybuf + (size_t)s * H + n));
            const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                a[2 * j] += bf16_lo(vv[j]);
                a[2 * j + 1] += bf16_hi(vv[j]);
            }
        }
        float r[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) r[j] = bf16r(a[j]);
        if (L.has_gate) {
            const float gate = 1.f / (1.f + __expf(-__ldcg(p.gl + t)));
            uint4 sv;
            if (L.has_shw) sv = __ldcg(reinterpret_cast<const uint4*>(p.sbuf + (size_t)t * H + n));
            else sv = __ldcg(reinterpret_cast<const uint4*>(p.shared + (size_t)t * H + n));
            const uint32_t ss[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                r[2 * j] = fmaf(gate, bf16_lo(ss[j]), r[2 * j]);
                r[2 * j + 1] = fmaf(gate, bf16_hi(ss[j]), r[2 * j + 1]);
            }
        }
        uint4 o;
        uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            __nv_bfloat162 b2 = __floats2bfloat162_rn(r[2 * j], r[2 * j + 1]);
            op[j] = *reinterpret_cast<uint32_t*>(&b2);
        }
        *reinterpret_cast<uint4*>(p.out + (size_t)t * H + n) = o;
    }
}

__global__ void __launch_bounds__(MOE_THREADS, CTAS_PER_SM) moe_persistent_kernel(const __grid_constant__ Params p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* ring = smem + OFF_RING;
    uint8_t* bst = smem + OFF_BST;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    uint64_t* empty = full + NST;
    uint64_t* efull = empty + NST;
    uint64_t* eempty = efull + NEPI;
    uint64_t* mma_bar = eempty + NEPI;
    StageDesc* desc = reinterpret_cast<StageDesc*>(smem + OFF_DESC);
    EpiRec* epi = reinterpret_cast<EpiRec*>(smem + OFF_EPI);
    uint8_t* plan = smem + OFF_PLAN;
    int16_t* ulist = reinterpret_cast<int16_t*>(plan + PLAN_ULIST);
    int16_t* gpre = reinterpret_cast<int16_t*>(plan + PLAN_GPRE);
    int16_t* toff = reinterpret_cast<int16_t*>(plan + PLAN_TOFF);
    int16_t* tlist = reinterpret_cast<int16_t*>(plan + PLAN_TLIST);
    int16_t* sids = reinterpret_cast<int16_t*>(plan + PLAN_SIDS);
    int* misc = reinterpret_cast<int*>(plan + PLAN_MISC);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int M = p.M, E = p.E, topk = p.topk, nslots = M * topk;
    uint32_t* ctrl = p.ctrl;

    if (tid == 0) {
        for (int i = 0; i < NST; ++i) {
            qf::mbar_init(full + i, 1);
            qf::mbar_init(empty + i, NCW);
        }
        for (int i = 0; i < NEPI; ++i) {
            qf::mbar_init(efull + i, NCW);
            qf::mbar_init(eempty + i, 1);
        }
        qf::mbar_init(mma_bar, 1);
        qf::mbar_fence_init();
        misc[MISC_DBGN] = 0;
    }
    if (warp == 0) {   // tensor memory: one warp allocates for the CTA (two CTAs per SM take 256 columns each)
        qf::tmem_alloc(reinterpret_cast<uint32_t*>(misc + MISC_TMEM), TM_COLS);
        qf::tmem_relinquish();
    }
    __syncwarp();
    // Everything below reads data of the previous kernel (topk ids, x) or the control block it may re-arm.
    qf::pdl_wait();

    // ------------------------------------------------------------------ routing plan (all 288 threads)
    {
        uint64_t* mask = reinterpret_cast<uint64_t*>(ring + SCR_MASK);
        int16_t* exf = reinterpret_cast<int16_t*>(ring + SCR_EXF);
        int16_t* exc = exf + QF_MAX_EXPERTS;
        int16_t* exg = exc + QF_MAX_EXPERTS;
        int16_t* toffe = reinterpret_cast<int16_t*>(ring + SCR_TOFFE);
        int* chunk = reinterpret_cast<int*>(ring + SCR_CHUNK);
        for (int e = tid; e < E; e += MOE_THREADS) mask[e] = 0ull;
        __syncthreads();
        bool bad = false;
        for (int s = tid; s < nslots; s += MOE_THREADS) {
            const int e = p.ids[s];
            if (e < 0 || e >= E) {
                bad = true;
                sids[s] = -1;
                continue;
            }
            sids[s] = (int16_t)e;
            if (e < p.elo || e >= p.ehi) continue;
            atomicOr(reinterpret_cast<unsigned long long*>(mask + e), 1ull << (s / topk));
        }
        if (bad) set_err(ctrl, QF_MOE_ERR_BAD_EXPERT);
        __syncthreads();
        const int nch = (E + 31) >> 5;
        for (int c = warp; c < nch; c += NCW + 1) {
            const int e = 32 * c + lane;
            const uint64_t m = e < E ? mask[e] : 0ull;
            const int f = m != 0ull, cnt = __popcll(m), ng = (cnt + TG - 1) / TG;
            int sf = f, sc = cnt, sg = ng;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int a = __shfl_up_sync(0xffffffffu, sf, o), b = __shfl_up_sync(0xffffffffu, sc, o),
                          d = __shfl_up_sync(0xffffffffu, sg, o);
                if (lane >= o) { sf += a; sc += b; sg += d; }
            }
            if (e < E) { exf[e] = (int16_t)(sf - f); exc[e] = (int16_t)(sc - cnt); exg[e] = (int16_t)(sg - ng); }
            if (lane == 31) { chunk[c] = sf; chunk[32 + c] = sc; chunk[64 + c] = sg; }
        }
        __syncthreads();
        if (warp == 0) {
            int vf = lane < nch ? chunk[lane] : 0, vc = lane < nch ? chunk[32 + lane] : 0,
                vg = lane < nch ? chunk[64 + lane] : 0;
            int sf = vf, sc = vc, sg = vg;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int a = __shfl_up_sync(0xffffffffu, sf, o), b = __shfl_up_sync(0xffffffffu, sc, o),
                          d = __shfl_up_sync(0xffffffffu, sg, o);
                if (lane >= o) { sf += a; sc += b; sg += d; }
            }
            __syncwarp();
            if (lane < nch) { chunk[lane] = sf - vf; chunk[32 + lane] = sc - vc; chunk[64 + lane] = sg - vg; }
            if (lane == 31) { misc[MISC_U] = sf; misc[MISC_NTOK] = sc; misc[MISC_GT] = sg; }
        }
        __syncthreads();
        for (int e = tid; e < E; e += MOE_THREADS) {
            if (mask[e] != 0ull) {
                const int c = e >> 5;
                const int u = chunk[c] + exf[e];
                ulist[u] = (int16_t)e;
                toff[u] = (int16_t)(chunk[32 + c] + exc[e]);
                gpre[u] = (int16_t)(chunk[64 + c] + exg[e]);
                toffe[e] = toff[u];
            }
        }
        if (tid == 0) {
            toff[misc[MISC_U]] = (int16_t)misc[MISC_NTOK];
            gpre[misc[MISC_U]] = (int16_t)misc[MISC_GT];
        }
        __syncthreads();
        for (int s = tid; s < nslots; s += MOE_THREADS) {
            const int e = sids[s];
            if (e < 0 || e < p.elo || e >= p.ehi) continue;
            const int t = s / topk, kp = s - t * topk;
            bool first = true;
            for (int k2 = 0; k2 < kp; ++k2) first &= sids[t * topk + k2] != e;
            if (first) {
                const int j = __popcll(mask[e] & ((1ull << t) - 1ull));
                tlist[toffe[e] + j] = (int16_t)s;
            }
        }
        __syncthreads();
    }
    qf::pdl_launch_dependents();
    const uint32_t tmem = (uint32_t)misc[MISC_TMEM];

    Layout L;
    L.R1 = (2 * p.I) / 128;
    L.R2 = p.H / 128;
    L.has_shw = p.shw13 != nullptr;
    L.has_gate = (p.shared != nullptr || L.has_shw) ? 1 : 0;
    L.Rs1 = L.has_shw ? (2 * p.Is) / 128 : 0;
    L.ngs = (M + TG - 1) / TG;
    L.U = misc[MISC_U];
    L.Gt = misc[MISC_GT];
    L.b_s1 = L.has_gate ? 1 : 0;
    L.b_g1 = L.b_s1 + (L.has_shw ? L.Rs1 * NSPLIT * L.ngs : 0);
    L.b_s1f = L.b_g1 + L.R1 * L.Gt;
    L.b_s2 = L.b_s1f + (L.has_shw ? L.Rs1 * L.ngs : 0);
    L.b_g2 = L.b_s2 + (L.has_shw ? L.R2 * L.ngs : 0);
    L.b_cb = L.b_g2 + L.R2 * L.Gt;
    L.total = L.b_cb + L.R2;
    L.tile_target = (uint32_t)(L.Gt + (L.has_shw ? L.ngs : 0));

    if (warp == NCW) {
        if (lane == 0) {
            // ========================================================== producer (one thread)
            const uint64_t pol = qf::policy_evict_first();
            int st = 0;
            uint32_t ph = 0;
            int next = (int)atomicAdd(ctrl + C_QUEUE, 1u);
            for (;;) {
                int item = next;
                if (hard_error(ctrl)) item = L.total;
                if (item < L.total) next = (int)atomicAdd(ctrl + C_QUEUE, 1u);   // claim ahead; in-order per CTA
                int kind = K_STOP, u = 0, tile = 0, tg = 0, split = 0, nk = 1, ntok = 0, e = 0;
                if (item >= L.total) {
                    kind = K_STOP;
                } else if (item < L.b_s1) {
                    kind = K_GL;
                } else if (item < L.b_g1) {
                    const int j = item - L.b_s1;
                    kind = K_S1;
                    tg = j % L.ngs;
                    split = (j / L.ngs) % NSPLIT;
                    tile = j / (L.ngs * NSPLIT);
                    nk = (p.H / NSPLIT) / BF_KC;
                    ntok = min(TG, M - TG * tg);
                } else if (item < L.b_s1f || (item >= L.b_g2 && item < L.b_cb)) {
                    const bool down = item >= L.b_g2;
                    const int j = item - (down ? L.b_g2 : L.b_g1);
                    const int R = down ? L.R2 : L.R1;
                    u = find_u(gpre, L.U, j / R);
                    const int ngu = gpre[u + 1] - gpre[u];
                    const int jj = j - R * gpre[u];
                    tile = jj / ngu;
                    tg = jj - tile * ngu;
                    kind = down ? K_G2 : K_G1;
                    e = ulist[u];
                    const int K = down ? p.I : p.H;
                    nk = (K + W4_KC - 1) / W4_KC;
                    ntok = min(TG, (toff[u + 1] - toff[u]) - TG * tg);
                } else if (item < L.b_s2) {
                    const int j = item - L.b_s1f;
                    kind = K_S1F;
                    tg = j % L.ngs;
                    tile = j / L.ngs;
                    ntok = min(TG, M - TG * tg);
                } else if (item < L.b_g2) {
                    const int j = item - L.b_s2;
                    kind = K_S2;
                    tg = j % L.ngs;
                    tile = j / L.ngs;
                    nk = p.Is / BF_KC;
                    ntok = min(TG, M - TG * tg);
                } else {
                    kind = K_CB;
                    tile = item - L.b_cb;
                }
                // dependencies of items without copies are resolved before their (empty) stage is published
                if (kind == K_S1F) wait_counter(ctrl, C_SPLIT + tile * L.ngs + tg, (uint32_t)NSPLIT);
                if (kind == K_CB) {
                    wait_counter(ctrl, C_CNT + tile, L.tile_target);
                    if (L.has_gate) wait_counter(ctrl, C_GLF, 1u);
                }
                for (int kidx = 0; kidx < nk; ++kidx) {
                    if (!qf::mbar_wait(empty + st, ph ^ 1u, PIPE_WAIT_NS)) set_err(ctrl, QF_MOE_ERR_PIPELINE);
                    uint8_t* sb = ring + st * STAGE_BYTES;
                    uint8_t* sw = sb;
                    uint8_t* ssc = sb + STAGE_W;
                    uint8_t* sx = sb + STAGE_W + STAGE_S;
                    int kc = 0;
                    uint32_t bytes = 0;
                    if (kind == K_G1 || kind == K_G2) {
                        const int K = kind == K_G1 ? p.H : p.I;
                        kc = min(W4_KC, K - W4_KC * kidx);
                        bytes = 128 * kc / 2 + kc * 2 + ntok * kc * 2;
                    } else if (kind == K_S1 || kind == K_S2) {
                        kc = BF_KC;
                        bytes = STAGE_W + ntok * kc * 2;
                    }
                    StageDesc d;
                    d.kind = (int16_t)kind; d.u = (int16_t)u; d.tile = (int16_t)tile; d.tg = (int16_t)tg;
                    d.split = (int16_t)split; d.kidx = (int16_t)kidx; d.nk = (int16_t)nk; d.kc = (int16_t)kc;
                    d.ntok = (int16_t)ntok;
                    desc[st] = d;
                    if (bytes == 0) {
                        qf::mbar_arrive(full + st);
                    } else {
                        qf::mbar_arrive_expect_tx(full + st, bytes);
                        const int xrb = (kc + 8) * 2;
                        if (kind == K_G1 || kind == K_G2) {
                            const bool down = kind == K_G2;
                            const int K = down ? p.I : p.H;
                            const int N = down ? p.H : 2 * p.I;
                            const uint8_t* wbase = (down ? p.w2 : p.w13) + (size_t)e * ((size_t)N * K / 2) +
                                                   (size_t)tile * (128 * (size_t)K / 2) + (size_t)kidx * STAGE_W;
                            const uint16_t* sbase = (down ? p.s2 : p.s13) + (size_t)e * ((size_t)N * K / 128) +
                                                    (size_t)tile * K + (size_t)kidx * 256;
                            qf::bulk_g2s_hint(sw, wbase, 128 * kc / 2, full + st, pol);
                            qf::bulk_g2s_hint(ssc, sbase, kc * 2, full + st, pol);
                            if (down && kidx == 0) {
                                wait_counter(ctrl, C_DONE + u, (uint32_t)(L.R1 * (gpre[u + 1] - gpre[u])));
                                qf::fence_proxy_async();
                            }
                            const int tbase = toff[u] + TG * tg;
                            for (int j = 0; j < ntok; ++j) {
                                const int s = tlist[tbase + j];
                                const __nv_bfloat16* src = down ? p.hbuf + (size_t)s * p.I + W4_KC * kidx
                                                                : p.x + (size_t)(s / topk) * p.H + W4_KC * kidx;
                                qf::bulk_g2s(sx + j * xrb, src, kc * 2, full + st);
                            }
                        } else {
                            const bool down = kind == K_S2;
                            const int K = down ? p.Is : p.H;
                            const int k0 = down ? BF_KC * kidx : split * (p.H / NSPLIT) + BF_KC * kidx;
                            const uint8_t* wbase = (down ? p.shw2 : p.shw13) + (size_t)tile * (128 * (size_t)K * 2) +
                                                   (size_t)(k0 / BF_KC) * STAGE_W;
                            qf::bulk_g2s_hint(sw, wbase, STAGE_W, full + st, pol);
                            if (down && kidx == 0) {
                                wait_counter(ctrl, C_SDONE + tg, (uint32_t)L.Rs1);
                                qf::fence_proxy_async();
                            }
                            for (int j = 0; j < ntok; ++j) {
                                const int tok = TG * tg + j;
                                const __nv_bfloat16* src =
                                    down ? p.hsh + (size_t)tok * p.Is + k0 : p.x + (size_t)tok * p.H + k0;
                                qf::bulk_g2s(sx + j * xrb, src, kc * 2, full + st);
                            }
                        }
                    }
                    if (++st == NST) { st = 0; ph ^= 1u; }
                }
                if (kind == K_STOP) break;
            }
        } else if (lane == 1) {
            // ========================================================== signal agent (one thread)
            // Consumer warps arrive on efull[slot] after their item's global stores; this thread then makes those
            // stores visible at gpu scope (fence) and publishes the item's counter increment.
            int es = 0;
            uint32_t eph = 0;
            for (;;) {
                if (!qf::mbar_wait(efull + es, eph, PIPE_WAIT_NS)) {
                    set_err(ctrl, QF_MOE_ERR_PIPELINE);
                    break;
                }
                const EpiRec r = epi[es];
                if (r.idx == -2) break;   // consumers stopped
                if (r.idx >= 0) {
                    __threadfence();
                    atomicAdd(ctrl + r.idx, (uint32_t)r.add);
                }
                qf::mbar_arrive(eempty + es);
                if (++es == NEPI) { es = 0; eph ^= 1u; }
            }
        }
        __syncwarp();
    } else {
        // ============================================================== consumers (8 warps, 2 warpgroups)
        const int ctid = tid;                 // 0..255
        const int wg = warp >> 2;             // warpgroup: which 128-k half of an int4 stage this thread dequantises
        const int quarter = warp & 3;         // TMEM lane quarter
        const int row = 32 * quarter + lane;  // tile row (= TMEM lane) owned by this thread
        const uint32_t lane_base = (uint32_t)(32 * quarter) << 16;
        float* red = reinterpret_cast<float*>(bst);   // [128 rows][16] partial exchange between the warpgroups
        int st = 0, es = 0;
        uint32_t ph = 0, eph = 0, mph = 0;
        float acc[TG];
        // optional timeline: (globaltimer << 12) | tag, up to 32 per CTA (tags: item kinds, 14 plan built, 15 exit)
        auto stamp = [&](int tag) {
            if (p.dbg != nullptr && ctid == 0 && misc[MISC_DBGN] < 32) {
                p.dbg[blockIdx.x * 32 + misc[MISC_DBGN]] = (long long)((qf::globaltimer() << 12) | (uint64_t)tag);
                misc[MISC_DBGN] += 1;
            }
        };
        // hand one completion record to the agent (record written by thread 0; all eight warps arrive)
        auto signal = [&](int idx, int add) {
            if (ctid == 0) {
                if (!qf::mbar_wait(eempty + es, eph ^ 1u, PIPE_WAIT_NS)) set_err(ctrl, QF_MOE_ERR_PIPELINE);
                epi[es].idx = idx;
                epi[es].add = add;
            }
            __syncwarp();
            if (lane == 0) qf::mbar_arrive(efull + es);
            if (++es == NEPI) { es = 0; eph ^= 1u; }
        };
        // the constant -136 A tile: written once by the first warpgroup (lanes 0..127, 8 columns)
        if (wg == 0) {
            uint32_t v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = 0xC308C308u;   // bf16 -136.0 in both halves
            qf::tmem_st8(tmem + lane_base + TM_C, v);
            qf::tmem_wait_st();
        }
        qf::tc_fence_before();
        qf::named_bar(1, CONS_THREADS);
        stamp(14);
        for (;;) {
            if (!qf::mbar_wait(full + st, ph, PIPE_WAIT_NS)) {
                set_err(ctrl, QF_MOE_ERR_PIPELINE);
                signal(-2, 0);
                break;
            }
            const StageDesc d = desc[st];
            if (d.kind == K_STOP) {
                stamp(15);
                signal(-2, 0);
                break;
            }
            if (d.kidx == 0) {
#pragma unroll
                for (int n = 0; n < TG; ++n) acc[n] = 0.f;
                stamp(d.kind);
            }
            uint8_t* sb = ring + st * STAGE_BYTES;
            const bool w4 = d.kind == K_G1 || d.kind == K_G2;
            const bool bf = d.kind == K_S1 || d.kind == K_S2;
            if (w4 || bf) {
                const int ngrp = w4 ? (d.kc >> 7) : 0;
                float sc = 0.f;
                reshuffle_b(sb, bst, d.kc, d.ntok, ctid);
                if (w4 && wg < ngrp) {
                    stage_w4_to_tmem(sb, tmem, wg, quarter, lane);
                    const uint16_t* ss = reinterpret_cast<const uint16_t*>(sb + STAGE_W);
                    sc = bf16_bits(ss[row * ngrp + wg]);
                    qf::tmem_wait_st();
                }
                qf::tc_fence_before();
                if (w4) {   // the stage's bytes now live in TMEM and bst: hand the ring slot back
                    __syncwarp();
                    if (lane == 0) qf::mbar_arrive(empty + st);
                }
                qf::named_bar(1, CONS_THREADS);
                if (ctid == 0) {
                    qf::tc_fence_after();
                    if (w4) {
                        for (int j = 0; j < (d.kc >> 4); ++j) {
                            const uint32_t dcol = tmem + TM_D + 16 * (j >> 3);
                            const uint64_t bd = qf::smem_desc(bst + 2 * j * 256, 256, 128);
                            qf::mma_ts(dcol, tmem + TM_C, bd, IDESC, (j & 7) != 0);
                            qf::mma_ts(dcol, tmem + TM_A + 8 * j, bd, IDESC, 1u);
                        }
                    } else {
                        for (int j = 0; j < 4; ++j)
                            qf::mma_ss(tmem + TM_D, qf::smem_desc(sb + 2 * j * 2048, 2048, 128),
                                       qf::smem_desc(bst + 2 * j * 256, 256, 128), IDESC, (d.kidx > 0 || j > 0));
                    }
                    qf::mma_commit(mma_bar);
                }
                __syncwarp();
                if (!qf::mbar_wait(mma_bar, mph, PIPE_WAIT_NS)) set_err(ctrl, QF_MOE_ERR_PIPELINE);
                mph ^= 1u;
                qf::tc_fence_after();
                if (bf) {   // the stage was the A operand: release it only now
                    __syncwarp();
                    if (lane == 0) qf::mbar_arrive(empty + st);
                }
                if (w4 && wg < ngrp) {
                    uint32_t v[16];
                    qf::tmem_ld16(tmem + lane_base + TM_D + 16 * wg, v);
                    qf::tmem_wait_ld();
#pragma unroll
                    for (int n = 0; n < TG; ++n) acc[n] = fmaf(__uint_as_float(v[n]), sc, acc[n]);
                }
                qf::tc_fence_before();
            } else {
                __syncwarp();
                if (lane == 0) qf::mbar_arrive(empty + st);
            }
            if (++st == NST) { st = 0; ph ^= 1u; }
            if (d.kidx != d.nk - 1) continue;

            // ------------------------------------------------------------ epilogues (item complete)
            if (w4) {   // fixed-order sum of the two warpgroups' halves into warpgroup 0
                if (wg == 1) {
#pragma unroll
                    for (int n = 0; n < TG; n += 4)
                        *reinterpret_cast<float4*>(red + row * TG + n) = make_float4(acc[n], acc[n + 1], acc[n + 2], acc[n + 3]);
                }
                qf::named_bar(1, CONS_THREADS);
                if (wg == 0) {
#pragma unroll
                    for (int n = 0; n < TG; n += 4) {
                        const float4 o = *reinterpret_cast<const float4*>(red + row * TG + n);
                        acc[n] += o.x; acc[n + 1] += o.y; acc[n + 2] += o.z; acc[n + 3] += o.w;
                    }
                }
                qf::named_bar(1, CONS_THREADS);
            } else if (bf && wg == 0) {
                uint32_t v[16];
                qf::tmem_ld16(tmem + lane_base + TM_D, v);
                qf::tmem_wait_ld();
#pragma unroll
                for (int n = 0; n < TG; ++n) acc[n] = __uint_as_float(v[n]);
                qf::tc_fence_before();
            }
            if (d.kind == K_GL) {
                for (int tok = warp; tok < M; tok += NCW) {
                    const uint4* xr = reinterpret_cast<const uint4*>(p.x + (size_t)tok * p.H);
                    const uint4* wr = reinterpret_cast<const uint4*>(p.wgate);
                    float a = 0.f;
                    for (int i = lane; i < p.H / 8; i += 32) {
                        const uint4 xv = __ldcg(xr + i), wv = __ldg(wr + i);
                        const uint32_t xx[4] = {xv.x, xv.y, xv.z, xv.w}, ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            a = fmaf(bf16_lo(xx[j]), bf16_lo(ww[j]), a);
                            a = fmaf(bf16_hi(xx[j]), bf16_hi(ww[j]), a);
                        }
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
                    if (lane == 0) p.gl[tok] = a;
                }
                signal(C_GLF, 1);
            } else if (d.kind == K_G1 || d.kind == K_S1F) {
                // rows interleave gate (even lane) and up (odd lane) of intermediate column j = row / 2;
                // even lanes finish tokens 0..7, odd lanes tokens 8..15
                if (d.kind == K_S1F && wg == 0) {
                    const float* pb = p.pbuf + (size_t)((d.tile * L.ngs + d.tg) * NSPLIT) * 2048 + row * TG;
#pragma unroll
                    for (int n = 0; n < TG; ++n) acc[n] = 0.f;
#pragma unroll
                    for (int sp = 0; sp < NSPLIT; ++sp) {   // fixed split order: the sum does not depend on timing
#pragma unroll
                        for (int n = 0; n < TG; n += 4) {
                            const float4 q = __ldcg(reinterpret_cast<const float4*>(pb + (size_t)sp * 2048 + n));
                            acc[n] += q.x; acc[n + 1] += q.y; acc[n + 2] += q.z; acc[n + 3] += q.w;
                        }
                    }
                }
                if (wg == 0) {
                    const bool odd = lane & 1;
                    float oth[TG];
#pragma unroll
                    for (int n = 0; n < TG; ++n) oth[n] = __shfl_xor_sync(0xffffffffu, acc[n], 1);
                    const int col = 64 * d.tile + (row >> 1);
                    if (d.kind == K_G1) {
                        const int u = d.u, e = ulist[u];
                        const float gs = p.gs13 ? bf16_bits(p.gs13[e]) : 1.f;
                        const int tbase = toff[u] + TG * d.tg;
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const int n = odd ? 8 + i : i;
                            const float g0 = odd ? oth[8 + i] : acc[i], u0 = odd ? acc[8 + i] : oth[i];
                            if (n < d.ntok) {
                                const float gv = bf16r(bf16r(g0) * gs);
                                const float uv = bf16r(bf16r(u0) * gs);
                                p.hbuf[(size_t)tlist[tbase + n] * p.I + col] =
                                    __float2bfloat16(gv / (1.f + __expf(-gv)) * uv);
                            }
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const int n = odd ? 8 + i : i;
                            const float g0 = odd ? oth[8 + i] : acc[i], u0 = odd ? acc[8 + i] : oth[i];
                            if (n < d.ntok) {
                                const float gv = bf16r(g0), uv = bf16r(u0);
                                p.hsh[(size_t)(TG * d.tg + n) * p.Is + col] =
                                    __float2bfloat16(gv / (1.f + __expf(-gv)) * uv);
                            }
                        }
                    }
                }
                signal(d.kind == K_G1 ? C_DONE + d.u : C_SDONE + d.tg, 1);
            } else if (d.kind == K_S1) {
                if (wg == 0) {
                    float* pb = p.pbuf + (size_t)((d.tile * L.ngs + d.tg) * NSPLIT + d.split) * 2048 + row * TG;
#pragma unroll
                    for (int n = 0; n < TG; n += 4)
                        __stcg(reinterpret_cast<float4*>(pb + n), make_float4(acc[n], acc[n + 1], acc[n + 2], acc[n + 3]));
                }
                signal(C_SPLIT + d.tile * L.ngs + d.tg, 1);
            } else if (d.kind == K_G2) {
                if (wg == 0) {
                    const int u = d.u, e = ulist[u];
                    const float g2 = p.gs2 ? bf16_bits(p.gs2[e]) : 1.f;
                    const int n0 = 128 * d.tile + row;
                    const int tbase = toff[u] + TG * d.tg;
#pragma unroll
                    for (int n = 0; n < TG; ++n) {
                        if (n >= d.ntok) break;
                        const int s0 = tlist[tbase + n];
                        const int tok = s0 / topk;
                        const float v = bf16r(acc[n]);
                        for (int kp = s0 - tok * topk; kp < topk; ++kp) {
                            const int s = tok * topk + kp;
                            if (sids[s] != e) continue;
                            const float w = bf16r(g2 * bf16r(__ldcg(p.tw + s)));
                            p.ybuf[(size_t)s * p.H + n0] = __float2bfloat16(v * w);
                        }
                    }
                }
                signal(C_CNT + d.tile, 1);
            } else if (d.kind == K_S2) {
                if (wg == 0) {
                    const int n0 = 128 * d.tile + row;
#pragma unroll
                    for (int n = 0; n < TG; ++n)
                        if (n < d.ntok) p.sbuf[(size_t)(TG * d.tg + n) * p.H + n0] = __float2bfloat16(acc[n]);
                }
                signal(C_CNT + d.tile, 1);
            } else if (d.kind == K_CB) {
                // the producer acquired every producer of this tile (and the gate logits) before publishing it
                combine_tile(p, L, sids, d.tile, ctid);
                signal(-1, 0);
            }
        }
    }

    // ------------------------------------------------------------------ exit: the last CTA re-arms ctrl
    __syncthreads();
    if (warp == 0) {   // every mma this CTA issued has completed (each commit was waited for)
        qf::tc_fence_after();
        qf::tmem_dealloc(tmem, TM_COLS);
    }
    if (tid == 0) {
        __threadfence();
        misc[MISC_FLAG] = atomicAdd(ctrl + C_EXIT, 1u) == gridDim.x - 1;
    }
    __syncwarp();
    __syncthreads();
    if (misc[MISC_FLAG]) {
        __threadfence();
        for (int i = tid; i < QF_MOE_CTRL_WORDS; i += MOE_THREADS)
            if (i != C_ERR) ctrl[i] = 0u;
    }
}

// ------------------------------------------------------------------------------------------ weight repacking
// Kernel layouts (one expert matrix [N, K]; see qwenfast_b200/formats.py for the same maps in torch):
//   row order inside a 128-row tile r: plain -> 128r + lane; gate_up ("gated") -> even lane 2j = gate row 64r + j,
//   odd lane 2j+1 = up row N/2 + 64r + j, so a SwiGLU pair sits in neighbouring lanes of one warp.
//   int4 stage (256 k, 16 KB): [half h (128 k)][quad q][lane (128)][4 words], word j of quad q holding
//   k = 256st + 128h + 32q + 8j .. +8 with nibble i = k index [0,2,4,6,1,3,5,7][i]; scales [lane][h].
//   bf16 stage (64 k, 16 KB): [k chunk c (8)][lane (128)][8 elements] = the canonical K-major no-swizzle tile.
__device__ __forceinline__ int kernel_row_to_src(int pos, int N, int gated) {
    if (!gated) return pos;
    const int r = pos >> 7, rho = pos & 127;
    return (rho & 1) ? N / 2 + 64 * r + (rho >> 1) : 64 * r + (rho >> 1);
}

// word o of an expert's kernel-layout matrix -> (source row, source word along K)
__device__ __forceinline__ void w4_word_src(long long o, int N, int K, int gated, int& row, int& kw) {
    const long long per_tile = 128LL * K / 8;
    const int r = (int)(o / per_tile);
    const int ot = (int)(o - r * per_tile);
    const int st = ot / 4096;
    const int os = ot - 4096 * st;
    const int j = os & 3, rho = (os >> 2) & 127, hq = os >> 9;
    kw = 32 * st + 16 * (hq >> 2) + 4 * (hq & 3) + j;
    row = kernel_row_to_src(128 * r + rho, N, gated);
}

__device__ __forceinline__ void w4_scale_src(long long o, int N, int K, int gated, int& row, int& grp) {
    const int r = (int)(o / K);
    const int ot = (int)(o - (long long)r * K);
    const int st = ot / 256;
    const int kc = min(256, K - 256 * st);
    const int os = ot - 256 * st;
    const int ngrp = kc / 128;
    grp = 2 * st + os % ngrp;
    row = kernel_row_to_src(128 * r + os / ngrp, N, gated);
}

__device__ __forceinline__ uint32_t nib_perm(uint32_t v, bool forward) {
    // forward: nibble i <- k index [0,2,4,6,1,3,5,7][i]; backward: inverse
    const int fwd[8] = {0, 2, 4, 6, 1, 3, 5, 7};
    uint32_t o = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        if (forward) o |= ((v >> (4 * fwd[i])) & 0xFu) << (4 * i);
        else o |= ((v >> (4 * i)) & 0xFu) << (4 * fwd[i]);
    }
    return o;
}

__global__ void w4_repack_kernel(const uint32_t* __restrict__ src, const uint16_t* __restrict__ ssrc,
                                 uint32_t* __restrict__ dst, uint16_t* __restrict__ sdst, int E, int N, int K,
                                 int gated, int unpack) {
    const long long words = (long long)N * K / 8, ents = (long long)N * K / 128;
    const long long total = (long long)E * words;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const long long e = i / words, o = i - e * words;
        int row, kw;
        w4_word_src(o, N, K, gated, row, kw);
        const long long si = e * words + (long long)row * (K / 8) + kw;
        if (!unpack) dst[i] = nib_perm(src[si], true);
        else dst[si] = nib_perm(src[i], false);
        if (o < ents) {
            int srow, grp;
            w4_scale_src(o, N, K, gated, srow, grp);
            const long long ssi = e * ents + (long long)srow * (K / 128) + grp;
            const long long di = e * ents + o;
            if (!unpack) sdst[di] = ssrc[ssi];
            else sdst[ssi] = ssrc[di];
        }
    }
}

__global__ void bf16_repack_kernel(const uint16_t* __restrict__ src, uint16_t* __restrict__ dst, int N, int K,
                                   int gated, int unpack) {
    const long long total = (long long)N * K;
    for (long long o = blockIdx.x * (long long)blockDim.x + threadIdx.x; o < total; o += (long long)gridDim.x * blockDim.x) {
        const long long per_tile = 128LL * K;
        const int r = (int)(o / per_tile);
        const int ot = (int)(o - r * per_tile);
        const int st = ot >> 13, os = ot & 8191;
        const int c = os >> 10, rho = (os >> 3) & 127, el = os & 7;
        const int k = 64 * st + 8 * c + el;
        const int row = kernel_row_to_src(128 * r + rho, N, gated);
        const long long si = (long long)row * K + k;
        if (!unpack) dst[o] = src[si];
        else dst[si] = src[o];
    }
}

}  // namespace

// ================================================================================================= C ABI
extern "C" int qf_a16_moe_workspace(int M, int H, int I, int topk, int Is, int64_t* hbuf_bytes, int64_t* ybuf_bytes,
                                    int64_t* gl_numel, int64_t* ctrl_numel, int64_t* pbuf_numel,
                                    int64_t* shbuf_bytes) {
    QF_REQUIRE(M >= 1 && M <= QF_MAX_TOKENS && H > 0 && I > 0 && topk >= 1 && topk <= QF_MAX_TOPK && Is >= 0,
               "a16_moe_workspace: bad sizes");
    const int ngs = (M + TG - 1) / TG;
    if (hbuf_bytes) *hbuf_bytes = (int64_t)M * topk * I * 2;
    if (ybuf_bytes) *ybuf_bytes = (int64_t)M * (topk + 1) * H * 2;
    if (gl_numel) *gl_numel = M;
    if (ctrl_numel) *ctrl_numel = QF_MOE_CTRL_WORDS;
    if (pbuf_numel) *pbuf_numel = Is > 0 ? (int64_t)(2 * Is / 128) * ngs * NSPLIT * 2048 : 0;
    if (shbuf_bytes) *shbuf_bytes = Is > 0 ? (int64_t)M * (Is + H) * 2 : 0;
    return QF_OK;
}

extern "C" int qf_a16_moe_decode(const void* x, const int32_t* topk_ids, const float* topk_w, const int32_t* w13,
                                 const void* s13, const void* gs13, const int32_t* w2, const void* s2, const void* gs2,
                                 const void* w_gate, const void* shared, const void* sh_w13, const void* sh_w2,
                                 void* hbuf, int64_t hbuf_bytes, void* ybuf, int64_t ybuf_bytes, float* gl,
                                 int64_t gl_numel, int32_t* ctrl, int64_t ctrl_numel, float* pbuf, int64_t pbuf_numel,
                                 void* shbuf, int64_t shbuf_bytes, void* out, int M, int H, int I, int E, int topk,
                                 int Is, int phase, int mode, int expert_lo, int expert_hi, int64_t* dbg, int pdl,
                                 qf_stream_t stream) {
    QF_REQUIRE(x && topk_ids && topk_w && w13 && s13 && w2 && s2 && hbuf && ybuf && gl && ctrl && out,
               "a16_moe_decode: null pointer argument");
    QF_REQUIRE(phase == 3 || phase == 4,
               "a16_moe_decode: phase must be 3 or 4 (whole layer); split phases 1/2 are not provided, got %d", phase);
    QF_REQUIRE(mode == 0, "a16_moe_decode: mode %d not available (0 = full layer)", mode);
    QF_REQUIRE(M >= 1 && M <= QF_MAX_TOKENS, "a16_moe_decode: M must be in [1, %d], got %d", QF_MAX_TOKENS, M);
    QF_REQUIRE(H >= 128 && H % 256 == 0 && H <= 8192, "a16_moe_decode: H must be a multiple of 256 in [256, 8192], got %d", H);
    QF_REQUIRE(I >= 128 && I % 128 == 0 && I <= 8192, "a16_moe_decode: I must be a multiple of 128, got %d", I);
    QF_REQUIRE(E >= 1 && E <= QF_MAX_EXPERTS, "a16_moe_decode: E must be in [1, %d], got %d", QF_MAX_EXPERTS, E);
    QF_REQUIRE(topk >= 1 && topk <= QF_MAX_TOPK && topk <= E, "a16_moe_decode: topk must be in [1, %d], got %d",
               QF_MAX_TOPK, topk);
    QF_REQUIRE(expert_lo >= 0 && expert_lo <= expert_hi && expert_hi <= E, "a16_moe_decode: bad expert range");
    const bool has_shw = sh_w13 != nullptr || sh_w2 != nullptr;
    QF_REQUIRE(!(has_shw && shared), "a16_moe_decode: give either shared-expert weights or a precomputed shared output");
    if (has_shw) {
        QF_REQUIRE(sh_w13 && sh_w2 && pbuf && shbuf, "a16_moe_decode: shared-expert weights need sh_w13, sh_w2, pbuf, shbuf");
        QF_REQUIRE(Is >= 64 && Is % 64 == 0 && Is <= 1024, "a16_moe_decode: Is must be a multiple of 64 in [64, 1024], got %d", Is);
    }
    QF_REQUIRE(!(has_shw || shared) || w_gate, "a16_moe_decode: a shared term needs w_gate");
    int64_t need_h, need_y, need_gl, need_ctrl, need_p, need_sh;
    qf_a16_moe_workspace(M, H, I, topk, has_shw ? Is : 0, &need_h, &need_y, &need_gl, &need_ctrl, &need_p, &need_sh);
    QF_REQUIRE(hbuf_bytes >= need_h && ybuf_bytes >= need_y && gl_numel >= need_gl && ctrl_numel >= need_ctrl,
               "a16_moe_decode: scratch too small (need hbuf %lld B, ybuf %lld B, gl %lld, ctrl %lld)", (long long)need_h,
               (long long)need_y, (long long)need_gl, (long long)need_ctrl);
    QF_REQUIRE(!has_shw || (pbuf_numel >= need_p && shbuf_bytes >= need_sh),
               "a16_moe_decode: shared scratch too small (need pbuf %lld, shbuf %lld B)", (long long)need_p, (long long)need_sh);
    const void* al[] = {x, w13, s13, w2, s2, hbuf, ybuf, out, w_gate, shared, sh_w13, sh_w2, pbuf, shbuf};
    for (const void* a : al) QF_REQUIRE(a == nullptr || qf::aligned(a, 16), "a16_moe_decode: every tensor must be 16-byte aligned");

    int dev = 0;
    cudaError_t ce = cudaGetDevice(&dev);
    if (ce != cudaSuccess) return qf::cuda_status(ce, "a16_moe_decode: cudaGetDevice");
    const int sms = qf::sm_count(dev);
    QF_REQUIRE(sms > 0, "a16_moe_decode: cannot query the SM count");
    static int per_sm_cache[64] = {0};
    int per_sm = dev < 64 ? per_sm_cache[dev] : 0;
    ce = qf::ensure_smem_attr(reinterpret_cast<const void*>(moe_persistent_kernel), MOE_SMEM);
    if (ce != cudaSuccess) return qf::cuda_status(ce, "a16_moe_decode: cudaFuncSetAttribute");
    if (per_sm == 0) {
        // every CTA of the persistent grid must be resident at once: size the grid from the occupancy
        ce = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, moe_persistent_kernel, MOE_THREADS, MOE_SMEM);
        if (ce != cudaSuccess) return qf::cuda_status(ce, "a16_moe_decode: occupancy query");
        per_sm = per_sm < 1 ? 1 : (per_sm > CTAS_PER_SM ? CTAS_PER_SM : per_sm);
        if (dev < 64) per_sm_cache[dev] = per_sm;
    }

    Params p;
    p.x = static_cast<const __nv_bfloat16*>(x);
    p.ids = topk_ids;
    p.tw = topk_w;
    p.w13 = reinterpret_cast<const uint8_t*>(w13);
    p.s13 = static_cast<const uint16_t*>(s13);
    p.gs13 = static_cast<const uint16_t*>(gs13);
    p.w2 = reinterpret_cast<const uint8_t*>(w2);
    p.s2 = static_cast<const uint16_t*>(s2);
    p.gs2 = static_cast<const uint16_t*>(gs2);
    p.wgate = static_cast<const __nv_bfloat16*>(w_gate);
    p.shared = static_cast<const __nv_bfloat16*>(shared);
    p.shw13 = has_shw ? static_cast<const uint8_t*>(sh_w13) : nullptr;
    p.shw2 = has_shw ? static_cast<const uint8_t*>(sh_w2) : nullptr;
    p.hbuf = static_cast<__nv_bfloat16*>(hbuf);
    p.ybuf = static_cast<__nv_bfloat16*>(ybuf);
    p.gl = gl;
    p.ctrl = reinterpret_cast<uint32_t*>(ctrl);
    p.pbuf = pbuf;
    p.hsh = has_shw ? static_cast<__nv_bfloat16*>(shbuf) : nullptr;
    p.sbuf = has_shw ? static_cast<__nv_bfloat16*>(shbuf) + (size_t)M * Is : nullptr;
    p.out = static_cast<__nv_bfloat16*>(out);
    p.dbg = reinterpret_cast<long long*>(dbg);
    p.M = M; p.H = H; p.I = I; p.E = E; p.topk = topk; p.Is = has_shw ? Is : 0;
    p.mode = mode; p.elo = expert_lo; p.ehi = expert_hi;
    ce = qf::launch_ex(moe_persistent_kernel, dim3(sms * per_sm), dim3(MOE_THREADS), MOE_SMEM,
                       reinterpret_cast<cudaStream_t>(stream), pdl != 0, p);
    return qf::cuda_status(ce, "a16_moe_decode: launch");
}

extern "C" int qf_moe_combine(const void*, const void*, const void*, int, void*, int, int, int, int, qf_stream_t) {
    qf::set_error("moe_combine: expert-parallel combine not available in this build");
    return QF_ERR_UNSUPPORTED;
}

static int repack_grid(long long n) {
    long long b = (n + 255) / 256;
    return (int)(b < 65535 * 8 ? (b > 0 ? b : 1) : 65535 * 8);
}

extern "C" int qf_w4_repack(const int32_t* qweight, const void* scales, int32_t* wk, void* sk, int E, int N, int K,
                            int gated, qf_stream_t stream) {
    QF_REQUIRE(qweight && scales && wk && sk, "w4_repack: null pointer argument");
    QF_REQUIRE(E >= 1 && N >= 128 && N % 128 == 0 && K >= 128 && K % 128 == 0, "w4_repack: need N %% 128 == 0 and K %% 128 == 0");
    const long long n = (long long)E * N * K / 8;
    w4_repack_kernel<<<repack_grid(n), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const uint32_t*>(qweight), static_cast<const uint16_t*>(scales), reinterpret_cast<uint32_t*>(wk),
        static_cast<uint16_t*>(sk), E, N, K, gated, 0);
    return qf::cuda_status(cudaGetLastError(), "w4_repack: launch");
}

extern "C" int qf_w4_unpack(const int32_t* wk, const void* sk, int32_t* qweight, void* scales, int E, int N, int K,
                            int gated, qf_stream_t stream) {
    QF_REQUIRE(qweight && scales && wk && sk, "w4_unpack: null pointer argument");
    QF_REQUIRE(E >= 1 && N >= 128 && N % 128 == 0 && K >= 128 && K % 128 == 0, "w4_unpack: need N %% 128 == 0 and K %% 128 == 0");
    const long long n = (long long)E * N * K / 8;
    w4_repack_kernel<<<repack_grid(n), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const uint32_t*>(wk), static_cast<const uint16_t*>(sk), reinterpret_cast<uint32_t*>(qweight),
        static_cast<uint16_t*>(scales), E, N, K, gated, 1);
    return qf::cuda_status(cudaGetLastError(), "w4_unpack: launch");
}

extern "C" int qf_bf16_repack(const void* w, void* wk, int N, int K, int gated, qf_stream_t stream) {
    QF_REQUIRE(w && wk, "bf16_repack: null pointer argument");
    QF_REQUIRE(N >= 128 && N % 128 == 0 && K >= 64 && K % 64 == 0, "bf16_repack: need N %% 128 == 0 and K %% 64 == 0");
    bf16_repack_kernel<<<repack_grid((long long)N * K), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t*>(w), static_cast<uint16_t*>(wk), N, K, gated, 0);
    return qf::cuda_status(cudaGetLastError(), "bf16_repack: launch");
}

extern "C" int qf_bf16_unpack(const void* wk, void* w, int N, int K, int gated, qf_stream_t stream) {
    QF_REQUIRE(w && wk, "bf16_unpack: null pointer argument");
    QF_REQUIRE(N >= 128 && N % 128 == 0 && K >= 64 && K % 64 == 0, "bf16_unpack: need N %% 128 == 0 and K %% 64 == 0");
    bf16_repack_kernel<<<repack_grid((long long)N * K), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t*>(wk), static_cast<uint16_t*>(w), N, K, gated, 1);
    return qf::cuda_status(cudaGetLastError(), "bf16_unpack: launch");
}
