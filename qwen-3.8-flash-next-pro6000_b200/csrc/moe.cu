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
//   * One CTA per SM (148 on B200) running NVP = 3 independent pipelines. A pipeline is 5 warps: 4 consumer warps
//     and a producer warp (lane 0). One more warp (lane 0) is the signal agent of all three. The pipelines share
//     the routing plan; everything else (ring, barriers, job slots) is per pipeline.
//   * Work items, claimed in order from a global queue by each pipeline's producer:
//       GL  shared-expert gate logits          S1  shared gate_up tile, one of 4 k-splits, one 16-token group
//       G1  expert u gate_up tile + group      S1F shared gate_up split-K sum + SwiGLU
//       S2  shared down tile + group           G2  expert u down tile + group
//       CB  top-k combine of one 128-column tile for 8 tokens (+ gated shared term)
//     An item only depends on items claimed before it, by pipelines that are already running, so the queue cannot
//     deadlock for any grid size.
//   * The producer streams each item's weights through an NST-stage shared-memory ring with the TMA engine
//     (mbarrier completion): per stage 8 KB of weights (128 rows x 128 k int4, or x 32 k bf16; 1-D bulk copy), for
//     int4 the stage's 128 row scales, and the matching k-slice of the item's token rows (x for gate_up, h for down):
//     one tensor copy of up to 16 consecutive rows for the shared expert, 1-D copies of one or two gathered rows, or
//     4-row gather copies (tile::gather4) of more, for a routed expert. Every cross-CTA dependency (gate_up -> down,
//     split-K -> finalize -> shared down, all producers of a column tile -> combine) is acquired by the producer
//     (bounded wait) before it copies the dependent rows and marks the stage full, so consumers never spin on other
//     CTAs, and a stage arrives whole: the four consumer warps of a pipeline run unsynchronised through an item.
//   * Contraction: a decode item has few tokens (about one per routed expert at 10 tokens x top-10 of 512 experts),
//     so each stage is a matrix-vector product that streams 8 KB of weights for a handful of columns. The weights
//     are stored in the tensor cores' register-fragment order (m16n8k16): consumer warp w owns the two 16-row tiles
//     2w, 2w + 1 of every 128-row stage, and one 16-byte shared-memory load gives a lane the int4 codes of four
//     k16 steps of one tile. Each 32-bit word turns into the four bf16x2 A registers of one step with a shift and
//     a lop3 per register (the biased code 128 + code, exact), and feeds mma.sync m16n8k16 (bf16, fp32 accumulate)
//     once per 8 tokens; the bias is taken off once per stage by an mma of a constant fragment against the tokens. No shared-memory or tensor-memory round trip sits between the copy engine and
//     the tensor cores. (tcgen05 with N = 16 token columns spends one tensor-memory store, one 128-row MMA chain and
//     one tensor-memory load per stage whatever the token count; at decode sizes that chain, not HBM, set the rate.)
//     bf16 stages (shared expert, 32 k) are already in fragment order and feed the mma directly.
//     gate_up tiles put gate row j in fragment row g and up row j in fragment row g + 8: one thread holds both.
//   * Consumers signal completed items through a per-pipeline record ring; the agent turns each record into one
//     gpu-scope release (fence + atomic add) on the control block. Consumer warps never execute a gpu-scope fence.
//   * The routing plan (unique experts, per-expert token lists, group offsets) is rebuilt identically by every CTA
//     from topk_ids with shared-memory atomics (token bit masks), so no CTA waits for a plan.
//   * Every wait is bounded; a wait that runs out sets QF_MOE_ERR_* in ctrl and the kernel drains. The consumer
//     warps of a pipeline agree on each item's outcome through a reducing named barrier (barrier.red.and) before its
//     epilogue, so a wait that runs out in one warp ends the item in all four and no barrier is left waiting.
#include <type_traits>

#include "qf_common.cuh"
#include "topk.cuh"

namespace {

using qf::bf16_bits;
using qf::bf16_hi;
using qf::bf16_lo;
using qf::bf16r;

constexpr int NCW = 4;                        // consumer warps of a pipeline (two 16-row tiles of 128 each)
constexpr int NVP = 3;                        // pipelines per CTA
constexpr int VP_WARPS = NCW + 1;             // consumers, producer
constexpr int VP_PRODUCER = NCW;
constexpr int AGENT_WARP = NVP * VP_WARPS;
constexpr int MOE_THREADS = (NVP * VP_WARPS + 1) * 32;
constexpr int CONS_THREADS = NCW * 32;
constexpr int CTAS_PER_SM = 1;
constexpr int TG = 16;                        // tokens per token group (two n8 tiles of the mma)
constexpr int NST = 5;                        // ring stages per pipeline
constexpr int NEPI = 8;                       // completion-record ring
constexpr int W4_KC = 128;                    // int4 k per stage (one scale group)
constexpr int BF_KC = 32;                     // bf16 k per stage
constexpr int STAGE_W = 8192;                 // weight bytes of a stage (128 rows x 128 k int4 or x 32 k bf16)
constexpr int STAGE_S = 256;                  // scale bytes of an int4 stage (one per row)
constexpr int STAGE_TOK = STAGE_W + STAGE_S;  // offset of the stage's token block
// token block of a pipelined stage: [token (16)][k]. int4 stages (128 k = 256 B per row): rows copied one by one
// sit at a 272-byte stride (the 8 lanes of each 16-byte shared-memory load phase hit distinct banks), rows of a
// 4-row gather copy back to back (256 B); bf16 stages (32 k): 64 B per row, back to back (conflict-free as it is).
constexpr int BROW_W4 = 272;
constexpr int BROW_G4 = 256;
constexpr int BROW_BF = 64;
constexpr int GATHER_MIN = 3;                 // tokens from which a routed item's rows come by 4-row gathers
constexpr int STAGE_BYTES = STAGE_TOK + TG * BROW_W4;
constexpr int NSPLIT = 4;                     // split-K of the shared expert's gate_up
constexpr int G1_SPLIT = 2;                   // k halves of a routed gate_up item (finished by the later half) when
                                              // all halves fit in one wave of pipelines (small M)
constexpr int MAXSLOTS = QF_MAX_TOKENS * QF_MAX_TOPK;
constexpr int CB_TOK = 4;                     // tokens of a combine item (x 32 four-column chunks = one per thread)
constexpr int CB_BATCH = 8;                   // slot loads a combine thread keeps in flight (registers)
constexpr uint64_t DEP_WAIT_NS = 1000000000ull;    // cross-CTA dependency waits
constexpr uint64_t PIPE_WAIT_NS = 4000000000ull;   // ring waits (longer: they cover the dependency waits)

// control block words
enum : int {
    C_QUEUE = 0,
    C_EXIT = 1,
    C_GLF = 2,
    C_ERR = QF_MOE_CTRL_ERR,
    C_RBAR = 4,     // fused router: CTAs whose logits are stored (grid barrier)
    C_XBAR = 5,     // fused router with host input: CTAs whose slice of x is in device memory (grid barrier)
    C_NEVER = 6,    // diagnostic mode 2: a word nothing increments (a dependency that never arrives)
    C_TBAR = 7,     // fused router above TOPK_ALL_MAX tokens: CTAs whose share of the top-k is stored (grid barrier)
    C_CNT = 8,      // [64] column-tile arrivals
    C_SDONE = 72,   // [4] finished shared gate_up tiles per token group
    C_SPLIT = 80,   // [64] split-K arrivals per (shared tile, token group)
    C_DONE = 160,   // [QF_MAX_EXPERTS] finished gate_up items per unique expert
};
static_assert(C_DONE + QF_MAX_EXPERTS <= QF_MOE_CTRL_MIRROR, "ctrl layout");

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
    const __nv_bfloat16* rw;   // fused router: router weight [E, H]; nullptr when topk ids / weights are inputs
    __nv_bfloat16* logits;     // fused router outputs: logits bf16 [M, E], ids int32 [M, topk], weights fp32 [M, topk]
    int* ids_out;
    float* tw_out;
    int renorm;
    const __nv_bfloat16* xsrc;   // fused router: x in pinned (mapped) host memory, copied into x by the kernel, or nullptr
    int M, H, I, E, topk, Is, mode, elo, ehi;
    int phase;  // 0: the whole layer; 1: gate logits + gate_up (hbuf, gl); 2: down + combine from hbuf and gl
    int wofs;   // expert id of the first expert in w13 / s13 / w2 / s2 / gs13 / gs2 (mode 1: elo)
    const uint8_t* f13;   // NVFP4 experts (FMT 1): E4M3 group-16 scales in the layout of formats.nvfp4_scale_map
    const uint8_t* f2;
    // token-row sources of the stages' token blocks (tensor maps, encoded per launch)
    CUtensorMap xt;   // x [M, H] bf16, box 32 k x tok_box rows: the shared expert's gate_up tokens
    CUtensorMap xg;   // x [M, H] bf16, box 128 k x 1 row: a routed expert's gate_up tokens (4-row gathers)
    CUtensorMap hg;   // hbuf [M * topk, I] bf16, box 128 k x 1 row: a routed expert's down tokens (by slot)
    CUtensorMap ht;   // shared-expert h [M, Is] bf16, box 32 k x tok_box rows: its down tokens
    int tok_box;      // rows of the xt / ht boxes: min(TG, M)
};

// shared memory map (dynamic): NVP pipeline blocks, then the routing plan
constexpr int VO_RING = 0;
constexpr int VO_BAR = VO_RING + NST * STAGE_BYTES;                   // full, empty, efull, eempty
constexpr int VO_DESC = VO_BAR + (2 * NST + 2 * NEPI) * 8;
constexpr int VO_EPI = VO_DESC + NST * (int)sizeof(StageDesc);
constexpr int VO_FLAG = VO_EPI + NEPI * (int)sizeof(EpiRec);         // int: this group finishes the item
constexpr int VP_BYTES = (VO_FLAG + 4 + 127) & ~127;
constexpr int OFF_PLAN = NVP * VP_BYTES;
static_assert(STAGE_BYTES % 128 == 0 && VO_BAR % 8 == 0 && VP_BYTES % 128 == 0, "shared memory alignment");
constexpr int PLAN_ULIST = 0;                                         // int16 [QF_MAX_EXPERTS]
constexpr int PLAN_GPRE = PLAN_ULIST + QF_MAX_EXPERTS * 2;            // int16 [QF_MAX_EXPERTS + 1]
constexpr int PLAN_TOFF = PLAN_GPRE + (QF_MAX_EXPERTS + 8) * 2;
constexpr int PLAN_TLIST = PLAN_TOFF + (QF_MAX_EXPERTS + 8) * 2;      // int16 [MAXSLOTS]
constexpr int PLAN_SIDS = PLAN_TLIST + MAXSLOTS * 2;                  // int16 [MAXSLOTS] copy of topk_ids
constexpr int PLAN_DUPN = PLAN_SIDS + MAXSLOTS * 2;                   // int16 [MAXSLOTS] next slot, same token+expert
constexpr int PLAN_TW = PLAN_DUPN + MAXSLOTS * 2;                     // fp32 [MAXSLOTS] bf16-rounded topk_weights
constexpr int PLAN_QGU = PLAN_TW + MAXSLOTS * 4;                      // int16 [MAXSLOTS] token group -> its u
constexpr int PLAN_TTOK = PLAN_QGU + MAXSLOTS * 2;                    // int16 [MAXSLOTS] token of each tlist entry
constexpr int PLAN_MISC = PLAN_TTOK + MAXSLOTS * 2;                   // int32 [64]
constexpr int PLAN_LAYOUT = PLAN_MISC + 64 * 4;                       // Layout (per-launch sizes, one copy per CTA)
constexpr int PLAN_LAYOUT_BYTES = 256;
constexpr int PLAN_BYTES = PLAN_LAYOUT + PLAN_LAYOUT_BYTES;
constexpr int MOE_SMEM = OFF_PLAN + PLAN_BYTES;
static_assert(MOE_SMEM + 1024 <= 228 * 1024, "the CTA must fit in shared memory");
// plan-build scratch aliases the ring (the producer starts after the plan is built)
constexpr int SCR_MASK = 0;                                        // uint64 [E]
constexpr int SCR_EXF = SCR_MASK + QF_MAX_EXPERTS * 8;             // int16 [E] x 3 (flag, count, groups) in-chunk
constexpr int SCR_TOFFE = SCR_EXF + 3 * QF_MAX_EXPERTS * 2;        // int16 [E] token offset per expert id
constexpr int SCR_CHUNK = SCR_TOFFE + QF_MAX_EXPERTS * 2;          // int32 [32] x 3 chunk totals
constexpr int SCR_RIDS = SCR_CHUNK + 3 * 32 * 4;                   // int32 [MAXSLOTS] fused router: selected ids
constexpr int SCR_RTW = SCR_RIDS + MAXSLOTS * 4;                    // fp32 [MAXSLOTS] fused router: their weights
static_assert(SCR_RTW + MAXSLOTS * 4 <= NST * STAGE_BYTES, "plan scratch (pipeline 0's ring)");
// fused router: this CTA's router rows live in pipeline 1's ring (idle until the plan is done)
constexpr int RROWS_BYTES = NST * STAGE_BYTES;
constexpr int RPC_MAX = 8;                                          // router rows per CTA

enum : int { DBG_CONSUMERS = 30, DBG_STOP = 31, DBG_ENTRY = 0xFFF };   // timeline events (dbg)
enum : int { MISC_U = 0, MISC_NTOK = 1, MISC_GT = 2, MISC_FLAG = 3, MISC_DBGN = 5, MISC_DUPS = 7 };

// Errors that stop the pipeline (waits that ran out). An out-of-range expert id is reported but not fatal: the
// slot is skipped and the rest of the layer is computed.
constexpr uint32_t HARD_ERR = QF_MOE_ERR_TIMEOUT | QF_MOE_ERR_PIPELINE;

__device__ __forceinline__ void set_err(uint32_t* ctrl, uint32_t bits) { atomicOr(ctrl + C_ERR, bits); }
__device__ __forceinline__ bool hard_error(uint32_t* ctrl) { return (qf::ld_volatile(ctrl + C_ERR) & HARD_ERR) != 0u; }

// Bounded wait until ctrl[idx] >= target (acquire). Gives up early when another CTA already recorded a hard error.
// Bounded spin until ctrl[idx] >= target (acquire). The bound is counted in SM cycles (2 per ns: at most ~1 s at
// the B200's clocks); the sticky error word and the bound are checked every 16 polls, so that a poll costs one L2
// round trip.
__device__ bool wait_counter(uint32_t* ctrl, int idx, uint32_t target) {
    if (qf::ld_acquire(ctrl + idx) >= target) return true;
    const long long t0 = clock64();
    const long long lim = (long long)(2 * DEP_WAIT_NS);
    for (uint32_t it = 1;; ++it) {
        __nanosleep(32);
        if (qf::ld_acquire(ctrl + idx) >= target) return true;
        if ((it & 15u) == 0u) {
            if (hard_error(ctrl)) return false;
            if (clock64() - t0 > lim) {
                set_err(ctrl, QF_MOE_ERR_TIMEOUT);
                return false;
            }
        }
    }
}

// Every CTA of the launch arrives, then waits (bounded) for all: writes before the barrier are visible to loads at
// L2 level (ld.cg / cp.async.cg) after it. The counter is re-armed at the launch's exit.
__device__ void grid_barrier(uint32_t* ctrl, int idx) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(ctrl + idx, 1u);
        wait_counter(ctrl, idx, gridDim.x);   // a timeout sets the sticky error; the items then stop
    }
    __syncthreads();
}

struct Layout {   // per-launch derived sizes, identical in every thread
    int R1, R2, Rs1, ngs, ngc, U, Gt, has_gate, has_shw;
    int b_s1, b_g1, b_s1f, b_s2, b_g2, b_cb, total;
    int base, nq;                     // this launch's items are base + the queue claims 0 .. nq - 1 (phases)
    uint32_t tile_target;
    int g1s;                          // gate_up k splits this launch: G1_SPLIT or 1
    // pbuf (floats): [0, sh_off) the zero-kept gate_up half counters (uint32), sized for QF_MAX_TOKENS so that their
    // place does not depend on M (one workspace sized for the largest M serves every smaller M); then the shared
    // gate_up split-K partials, then the gate_up half partials
    size_t sh_off, g1_part_off;
};
static_assert(sizeof(Layout) <= PLAN_LAYOUT_BYTES && PLAN_LAYOUT % 8 == 0, "Layout slot in the plan");

// The per-launch sizes: computed once per CTA (after the routing plan has counted U and Gt) into shared memory,
// read from there by every role, so that they do not occupy registers of the pipelines' loops.
__device__ void make_layout(Layout& L, const Params& p, int M, int U, int Gt, int grid) {
    L.R1 = (2 * p.I) / 128;
    L.R2 = p.H / 128;
    L.has_shw = p.shw13 != nullptr;
    L.has_gate = (p.shared != nullptr || L.has_shw) ? 1 : 0;
    L.Rs1 = L.has_shw ? (2 * p.Is) / 128 : 0;
    L.ngs = (M + TG - 1) / TG;
    L.ngc = (M + CB_TOK - 1) / CB_TOK;
    L.U = U;
    L.Gt = Gt;
    L.b_s1 = L.has_gate ? 1 : 0;
    L.b_g1 = L.b_s1 + (L.has_shw ? L.Rs1 * NSPLIT * L.ngs : 0);
    // split the gate_up items only when every half still fits in one wave of pipelines: then the halves shorten
    // the critical path; with more items the split only adds the hand-off of the partials. The test uses the
    // bound M * topk on the token groups, not this launch's count, so that a shard (mode 1) decides exactly as
    // the whole layer does and the sums keep the same association.
    L.g1s = G1_SPLIT * L.R1 * M * p.topk <= grid * NVP ? G1_SPLIT : 1;
    L.b_s1f = L.b_g1 + L.R1 * L.Gt * L.g1s;
    L.b_s2 = L.b_s1f + (L.has_shw ? L.Rs1 * L.ngs : 0);
    L.b_g2 = L.b_s2 + (L.has_shw ? L.R2 * L.ngs : 0);
    L.b_cb = L.b_g2 + L.R2 * L.Gt;
    L.total = L.b_cb + L.R2 * L.ngc;
    // phase 1 ends with the gate_up items (no shared-expert weights in the split phases: b_g2 == b_s1f); phase 2
    // starts with the down items
    if (p.phase == 1) L.total = L.b_g2;
    L.base = p.phase == 2 ? L.b_g2 : 0;
    L.nq = L.total - L.base;
    L.tile_target = (uint32_t)(L.Gt + (L.has_shw ? L.ngs : 0));
    L.sh_off = ((size_t)QF_MAX_TOKENS * p.topk * L.R1 + 3) & ~(size_t)3;
    L.g1_part_off = L.sh_off + (L.has_shw ? (size_t)L.Rs1 * L.ngs * NSPLIT * 2048 : 0);
}

// ------------------------------------------------------------------------------- register-path stage contraction
// A lane (g = lane / 4, t4 = lane % 4) of consumer warp w holds the m16n8k16 fragments of m16 tiles 2w + m (m = 0, 1)
// and n8 token tiles n (n = 0, 1): accumulator d[2 m + n][i] is row 16 (2w + m) + g + 8 (i / 2) of the stage, token
// 8 n + 2 t4 + (i % 2). Inside each 64-k half of a stage the weights' k order is permuted so that the lane's four
// k16 steps use one 32-byte run of each token row: step s of half h takes k = 64 h + 16 t4 + 4 s + (0 .. 3) in mma
// columns (2 t4, 2 t4 + 1, 2 t4 + 8, 2 t4 + 9). The layouts are built by the repack kernels below.

// NVFP4 pair j of a word (nibbles j and j + 4, e2m1 codes) -> bf16x2 of code * scale (exact): sign to bit 15,
// exponent and mantissa to bits 6..8 (a bf16 of 2^-126 times the code), times 2^126, times the row's scale.
__device__ __forceinline__ uint32_t nvfp4_pair(uint32_t q, int j, uint32_t scale) {
    const uint32_t a = (6 - 4 * j) >= 0 ? (q << (6 - 4 * j)) : (q >> (4 * j - 6));
    const uint32_t b = q << (12 - 4 * j);
    const uint32_t bits = (a & 0x01C001C0u) | (b & 0x80008000u);
    uint32_t v, r;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(v) : "r"(bits), "r"(0x7E807E80u));   // 2^126
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(v), "r"(scale));
    return r;
}

// One int4 / NVFP4 stage (128 rows x 128 k) of warp rw's two m16 tiles: d = fresh fp32 partials of the stage.
// sb: the ring stage (weights in fragment order: [tile (8)][half (2)][lane (32)][4 words]); bb: the token block,
// row stride brow. TWO: the item has more than 8 tokens (second n8 tile). NVFP4 (FMT 1): fsc = the lane's eight
// E4M3 scales of the stage, byte (m * 2 + h) * 2 + (row g : 0, row g + 8 : 1) (each covers the lane's 16 k).
// int4 (FMT 0): the A registers hold the signed codes code - 8 (one lop3 to the biased code 128 + code and one
// bf16x2 subtract of 136, both exact). Every product is exact; the partials are fp32.
template <int FMT, bool TWO>
__device__ __forceinline__ void stage_w4(const uint8_t* sb, const uint8_t* bb, int brow, int rw, int lane, uint2 fsc,
                                         float (&d)[4][4]) {
    const int g = lane >> 2, t4 = lane & 3;
    // every accumulator chain starts with a zero-input mma (h = 0, s = 0): no register clearing per stage
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint8_t* tb = bb + g * brow + h * 128 + t4 * 32;
        const uint4 x0a = *reinterpret_cast<const uint4*>(tb), x0b = *reinterpret_cast<const uint4*>(tb + 16);
        uint4 x1a = make_uint4(0u, 0u, 0u, 0u), x1b = x1a;
        if constexpr (TWO) {
            x1a = *reinterpret_cast<const uint4*>(tb + 8 * brow);
            x1b = *reinterpret_cast<const uint4*>(tb + 8 * brow + 16);
        }
        const uint32_t xw0[8] = {x0a.x, x0a.y, x0a.z, x0a.w, x0b.x, x0b.y, x0b.z, x0b.w};
        const uint32_t xw1[8] = {x1a.x, x1a.y, x1a.z, x1a.w, x1b.x, x1b.y, x1b.z, x1b.w};
#pragma unroll
        for (int m = 0; m < 2; ++m) {
            const uint4 a = *reinterpret_cast<const uint4*>(sb + (((2 * rw + m) * 2 + h) * 32 + lane) * 16);
            const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
            uint32_t sA = 0u, sB = 0u;
            if constexpr (FMT == 1) {
                const uint32_t ws = (m == 0 ? fsc.x : fsc.y) >> (16 * h);
                sA = qf::e4m3_scale_bf16x2(ws & 0xFFu);
                sB = qf::e4m3_scale_bf16x2((ws >> 8) & 0xFFu);
            }
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                // A registers of step s: (row g, k+0|1) (row g+8, k+0|1) (row g, k+2|3) (row g+8, k+2|3) = the
                // word's nibble pairs (0,4) (1,5) (2,6) (3,7)
                uint32_t v[4];
                if constexpr (FMT == 0) {
                    qf::signed_w4(aw[s], v);
                } else {
#pragma unroll
                    for (int j = 0; j < 4; ++j) v[j] = nvfp4_pair(aw[s], j, (j & 1) ? sB : sA);
                }
                if (h == 0 && s == 0) {
                    qf::mma_bf16_z(d[2 * m], v[0], v[1], v[2], v[3], xw0[0], xw0[1]);
                    if constexpr (TWO) qf::mma_bf16_z(d[2 * m + 1], v[0], v[1], v[2], v[3], xw1[0], xw1[1]);
                } else {
                    qf::mma_bf16(d[2 * m], v[0], v[1], v[2], v[3], xw0[2 * s], xw0[2 * s + 1]);
                    if constexpr (TWO) qf::mma_bf16(d[2 * m + 1], v[0], v[1], v[2], v[3], xw1[2 * s], xw1[2 * s + 1]);
                }
            }
        }
    }
    if constexpr (!TWO && FMT != 0) {   // the unused token tile's accumulators (added up by the caller): zero
#pragma unroll
        for (int m = 0; m < 2; ++m) d[2 * m + 1][0] = d[2 * m + 1][1] = d[2 * m + 1][2] = d[2 * m + 1][3] = 0.f;
    }
}

// One bf16 stage (128 rows x 32 k, [tile (8)][step (2)][lane (32)][8 elements] = the A registers of each k16 step)
// of warp rw's two m16 tiles; token block row stride BROW_BF, the lane's 8 k = 8 t4 .. 8 t4 + 7 of each token.
template <bool TWO>
__device__ __forceinline__ void stage_bf16(const uint8_t* sb, const uint8_t* bb, int rw, int lane, float (&d)[4][4]) {
    const int g = lane >> 2, t4 = lane & 3;
    if constexpr (!TWO) {
#pragma unroll
        for (int m = 0; m < 2; ++m) d[2 * m + 1][0] = d[2 * m + 1][1] = d[2 * m + 1][2] = d[2 * m + 1][3] = 0.f;
    }
    const uint4 x0 = *reinterpret_cast<const uint4*>(bb + g * BROW_BF + t4 * 16);
    const uint4 x1 = TWO ? *reinterpret_cast<const uint4*>(bb + (8 + g) * BROW_BF + t4 * 16) : make_uint4(0u, 0u, 0u, 0u);
    const uint32_t xw0[4] = {x0.x, x0.y, x0.z, x0.w}, xw1[4] = {x1.x, x1.y, x1.z, x1.w};
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int s = 0; s < 2; ++s) {
            const uint4 a = *reinterpret_cast<const uint4*>(sb + (((2 * rw + m) * 2 + s) * 32 + lane) * 16);
            if (s == 0) {
                qf::mma_bf16_z(d[2 * m], a.x, a.y, a.z, a.w, xw0[0], xw0[1]);
                if constexpr (TWO) qf::mma_bf16_z(d[2 * m + 1], a.x, a.y, a.z, a.w, xw1[0], xw1[1]);
            } else {
                qf::mma_bf16(d[2 * m], a.x, a.y, a.z, a.w, xw0[2 * s], xw0[2 * s + 1]);
                if constexpr (TWO) qf::mma_bf16(d[2 * m + 1], a.x, a.y, a.z, a.w, xw1[2 * s], xw1[2 * s + 1]);
            }
        }
}

// Shared-expert gate logit of one token, x[t] . w_gate in fp32: lane-strided fma chain over 16-byte chunks, then an
// xor-tree warp sum (every lane returns it). One definition for the layer kernel and the expert-parallel combine,
// so both produce the same bits.
__device__ __forceinline__ float gate_logit(const __nv_bfloat16* xrow, const __nv_bfloat16* wgate, int H, int lane) {
    const uint4* xr = reinterpret_cast<const uint4*>(xrow);
    const uint4* wr = reinterpret_cast<const uint4*>(wgate);
    float a = 0.f;
    // two chunks' loads in flight at a time (one memory round trip per two), the fma chain in chunk order
    for (int i0 = lane; i0 < H / 8; i0 += 2 * 32) {
        uint4 xv[2], wv[2];
#pragma unroll
        for (int b = 0; b < 2; ++b) {
            const int i = i0 + 32 * b;
            xv[b] = i < H / 8 ? __ldcg(xr + i) : make_uint4(0u, 0u, 0u, 0u);
            wv[b] = i < H / 8 ? __ldg(wr + i) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int b = 0; b < 2; ++b) {
            if (i0 + 32 * b >= H / 8) break;
            const uint32_t xx[4] = {xv[b].x, xv[b].y, xv[b].z, xv[b].w}, ww[4] = {wv[b].x, wv[b].y, wv[b].z, wv[b].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                a = fmaf(bf16_lo(xx[j]), bf16_lo(ww[j]), a);
                a = fmaf(bf16_hi(xx[j]), bf16_hi(ww[j]), a);
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    return a;
}

// Add 8 bf16 slot values (one 16-byte word) to the fp32 column sums.
__device__ __forceinline__ void add8(float (&a)[8], uint4 v) {
    const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        a[2 * j] += bf16_lo(vv[j]);
        a[2 * j + 1] += bf16_hi(vv[j]);
    }
}
// out = bf16(gate * shared + bf16(a)) for 8 columns (gate applied when has_gate), where a = the fp32 sum of the
// routed slots in top-k order: the reference's combine rounding points (qf_a16moe.cu:449-461).
__device__ __forceinline__ uint4 finish8(const float (&a)[8], bool has_gate, float gl, uint4 sv) {
    float r[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = bf16r(a[j]);
    if (has_gate) {
        const float gate = 1.f / (1.f + __expf(-gl));
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
    return o;
}

__device__ __forceinline__ void add4(float (&a)[4], uint2 v) {
    a[0] += bf16_lo(v.x);
    a[1] += bf16_hi(v.x);
    a[2] += bf16_lo(v.y);
    a[3] += bf16_hi(v.y);
}
// finish8 for 4 columns (the same arithmetic per column)
__device__ __forceinline__ uint2 finish4(const float (&a)[4], bool has_gate, float gl, uint2 sv) {
    float r[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) r[j] = bf16r(a[j]);
    if (has_gate) {
        const float gate = 1.f / (1.f + __expf(-gl));
        r[0] = fmaf(gate, bf16_lo(sv.x), r[0]);
        r[1] = fmaf(gate, bf16_hi(sv.x), r[1]);
        r[2] = fmaf(gate, bf16_lo(sv.y), r[2]);
        r[3] = fmaf(gate, bf16_hi(sv.y), r[3]);
    }
    const __nv_bfloat162 b0 = __floats2bfloat162_rn(r[0], r[1]), b1 = __floats2bfloat162_rn(r[2], r[3]);
    return make_uint2(*reinterpret_cast<const uint32_t*>(&b0), *reinterpret_cast<const uint32_t*>(&b1));
}

// Combine of one 128-column tile for tokens CB_TOK g .. CB_TOK g + CB_TOK - 1: out = bf16(gate * shared +
// bf16(sum_kpos y)); a thread owns one (token, 4 columns). The shared row, the gate logit and CB_BATCH routed slots
// are requested before the first add (one L2 round trip per CB_BATCH slots); the sum runs in top-k order.
__device__ void combine_tile(const Params& p, const Layout& L, const int16_t* sids, int c, int g, int ctid) {
    const int H = p.H, topk = p.topk;
    const int t = CB_TOK * g + (ctid >> 5), n = 128 * c + 4 * (ctid & 31);
    if (t >= p.M) return;
    uint2 sv = make_uint2(0u, 0u);
    float gl = 0.f;
    if (L.has_gate) {
        gl = __ldcg(p.gl + t);
        if (L.has_shw) sv = __ldcg(reinterpret_cast<const uint2*>(p.sbuf + (size_t)t * H + n));
        else sv = __ldcg(reinterpret_cast<const uint2*>(p.shared + (size_t)t * H + n));
    }
    float a[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k0 = 0; k0 < topk; k0 += CB_BATCH) {
        uint2 v[CB_BATCH];
        bool live[CB_BATCH];
#pragma unroll
        for (int b = 0; b < CB_BATCH; ++b) {
            const int kp = k0 + b, s = t * topk + kp;
            const int e = kp < topk ? sids[s] : -1;
            live[b] = e >= 0 && e >= p.elo && e < p.ehi;
            if (live[b]) v[b] = __ldcg(reinterpret_cast<const uint2*>(p.ybuf + (size_t)s * H + n));
        }
#pragma unroll
        for (int b = 0; b < CB_BATCH; ++b)
            if (live[b]) add4(a, v[b]);
    }
    *reinterpret_cast<uint2*>(p.out + (size_t)t * H + n) = finish4(a, L.has_gate != 0, gl, sv);
}

// Expert-parallel shard (mode 1), one 128-column tile, tokens CB_TOK g ..: make ybuf the shard's exact contribution
// to the slot sum -- zeros in every slot this shard does not own (other shards' experts, invalid ids), and the
// shared expert's output in rows M * topk + t when this shard computes it (zeros otherwise). The routed slots of
// local experts were written by the down-projection epilogues.
__device__ void shard_tile(const Params& p, const Layout& L, const int16_t* sids, int c, int g, int ctid) {
    const int H = p.H, topk = p.topk;
    const int t = CB_TOK * g + (ctid >> 5), n = 128 * c + 4 * (ctid & 31);
    if (t >= p.M) return;
    const uint2 zero = make_uint2(0u, 0u);
    uint2 sv = zero;
    if (L.has_shw) sv = __ldcg(reinterpret_cast<const uint2*>(p.sbuf + (size_t)t * H + n));
    else if (p.shared != nullptr) sv = __ldcg(reinterpret_cast<const uint2*>(p.shared + (size_t)t * H + n));
    for (int kp = 0; kp < topk; ++kp) {
        const int s = t * topk + kp;
        const int e = sids[s];
        if (e < 0 || e < p.elo || e >= p.ehi) *reinterpret_cast<uint2*>(p.ybuf + (size_t)s * H + n) = zero;
    }
    *reinterpret_cast<uint2*>(p.ybuf + (size_t)(p.M * topk + t) * H + n) = sv;
}

// ------------------------------------------------------------------------------------------------ fused router
// logits[t, e] = bf16(x[t] . w[e]) for this CTA's router rows (already requested into rrows), a grid barrier, then
// the top-k of every token into rids / rtw (serve/qwenfast/qf_router.cu). Up to TOPK_ALL_MAX tokens every CTA
// selects every token itself (at most one token per warp), so the plan needs no ids from memory; above that, CTA c
// selects token c (and c + grid ...) into the caller's ids / weights outputs, a second grid barrier follows, and every
// CTA reads them back. Not inlined: it runs once per launch, and as a separate function its registers do not compete
// with the pipelines' loops.
// This CTA's router rows [r0, r0 + nrows) times every token, with the standalone router's arithmetic (router.cu):
// the 16 warps split the hidden dimension into 32-k blocks (BPW consecutive blocks per warp, BPW the power of two the
// standalone router picks for H); per token tile of 8 a warp runs two m16n8k16 mmas per block (this CTA's rows as the
// A operand: rows g < nrows, the others zero; the tokens' x from L2 as B); the per-warp fp32 partials are summed in
// warp order through red (shared memory). The x of TB token tiles is requested before the first of their mmas.
template <int BPW>
__device__ __forceinline__ void router_logits(const Params& p, float* red, const uint8_t* rrows, int r0, int nrows) {
    constexpr int TB = 16 / BPW < 8 ? 16 / BPW : 8;
    static_assert(MOE_THREADS / 32 == 16 && 16 * RPC_MAX * QF_MAX_TOKENS * 4 <= VP_BYTES, "router partials");
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t4 = lane & 3;
    const int M = p.M, nblk = p.H / 32, b0 = warp * BPW;
    const int ntile = (M + 7) >> 3, rp = ntile * 8;
    const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
    const uint4* wrow = reinterpret_cast<const uint4*>(rrows) + (size_t)g * (p.H / 8) + t4;
    for (int nt0 = 0; nt0 < ntile; nt0 += TB) {
        uint4 xv[TB][BPW];
#pragma unroll
        for (int tb = 0; tb < TB; ++tb) {
            const int tok = (nt0 + tb) * 8 + g;
            const uint4* xr = reinterpret_cast<const uint4*>(p.x + (size_t)(tok < M ? tok : 0) * p.H) + t4;
#pragma unroll
            for (int i = 0; i < BPW; ++i) xv[tb][i] = (tok < M && b0 + i < nblk) ? __ldcg(xr + 4 * (b0 + i)) : zero;
        }
#pragma unroll
        for (int tb = 0; tb < TB; ++tb) {
            const int nt = nt0 + tb;
            if (nt >= ntile) break;
            float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int i = 0; i < BPW; ++i) {
                if (b0 + i < nblk) {
                    const uint4 wa = g < nrows ? wrow[4 * (b0 + i)] : zero;
                    qf::mma_bf16(d, wa.x, 0u, wa.y, 0u, xv[tb][i].x, xv[tb][i].y);
                    qf::mma_bf16(d, wa.z, 0u, wa.w, 0u, xv[tb][i].z, xv[tb][i].w);
                }
            }
            if (g < nrows) {
                red[(warp * RPC_MAX + g) * rp + nt * 8 + 2 * t4] = d[0];
                red[(warp * RPC_MAX + g) * rp + nt * 8 + 2 * t4 + 1] = d[1];
            }
        }
    }
    __syncthreads();
    for (int idx = tid; idx < nrows * M; idx += MOE_THREADS) {
        const int r = idx % nrows, t = idx / nrows;
        float sum = 0.f;
#pragma unroll
        for (int ww = 0; ww < 16; ++ww) sum += red[(ww * RPC_MAX + r) * rp + t];
        p.logits[(size_t)t * p.E + r0 + r] = __float2bfloat16(sum);
    }
}

constexpr int TOPK_ALL_MAX = 16;
__device__ __noinline__ void fused_router(const Params& p, uint8_t* smem, const uint8_t* rrows, int r0, int nrows,
                                          int* rids, float* rtw) {
    const int tid = threadIdx.x, warp = tid >> 5;
    const int M = p.M, E = p.E, topk = p.topk;
    uint32_t* ctrl = p.ctrl;
    qf::cp_async_wait_all();
    __syncthreads();
    // logits with the standalone router's arithmetic (router.cu), so that both routers give the same bits
    const int bpw = (p.H / 32 + 15) / 16;
    float* red = reinterpret_cast<float*>(smem + 2 * VP_BYTES);   // pipeline 2's ring, idle until the plan is done
    if (bpw <= 1) router_logits<1>(p, red, rrows, r0, nrows);
    else if (bpw <= 2) router_logits<2>(p, red, rrows, r0, nrows);
    else if (bpw <= 4) router_logits<4>(p, red, rrows, r0, nrows);
    else router_logits<8>(p, red, rrows, r0, nrows);
    grid_barrier(ctrl, C_RBAR);
    if (M <= TOPK_ALL_MAX) {
        for (int t = warp; t < M; t += MOE_THREADS / 32)
            qf::topk_row_any(p.logits + (size_t)t * E, E, topk, p.renorm, rtw + t * topk, rids + t * topk);
    } else {
        for (int t = (int)blockIdx.x + (int)gridDim.x * warp; t < M; t += (int)gridDim.x * (MOE_THREADS / 32))
            qf::topk_row_any(p.logits + (size_t)t * E, E, topk, p.renorm, p.tw_out + t * topk, p.ids_out + t * topk);
        grid_barrier(ctrl, C_TBAR);
        for (int s = tid; s < M * topk; s += MOE_THREADS) {
            rids[s] = __ldcg(p.ids_out + s);
            rtw[s] = __ldcg(p.tw_out + s);
        }
    }
    __syncthreads();
}

// FMT 0: int4 experts (code - 8, one bf16 scale per 128 k, applied to each stage's fp32 partial). FMT 1: NVFP4 experts
// (e2m1 codes with one E4M3 scale per 16 k, folded into the dequantised weights; the per-expert global multiplier
// is gs13 / gs2, as for int4).
template <int FMT>
__global__ void __launch_bounds__(MOE_THREADS, 1) moe_persistent_kernel(const __grid_constant__ Params p) {
    extern __shared__ __align__(128) uint8_t smem[];
    if (p.dbg != nullptr && threadIdx.x == 0 && blockIdx.x < QF_MOE_DBG_NUMEL / 32)   // timeline: CTA entry
        p.dbg[blockIdx.x * 32 + 31] = (long long)((qf::globaltimer() << 12) | (uint64_t)DBG_ENTRY);
    uint8_t* plan = smem + OFF_PLAN;
    int16_t* ulist = reinterpret_cast<int16_t*>(plan + PLAN_ULIST);
    int16_t* gpre = reinterpret_cast<int16_t*>(plan + PLAN_GPRE);
    int16_t* toff = reinterpret_cast<int16_t*>(plan + PLAN_TOFF);
    int16_t* tlist = reinterpret_cast<int16_t*>(plan + PLAN_TLIST);
    int16_t* sids = reinterpret_cast<int16_t*>(plan + PLAN_SIDS);
    int16_t* dupn = reinterpret_cast<int16_t*>(plan + PLAN_DUPN);
    float* tws = reinterpret_cast<float*>(plan + PLAN_TW);
    int16_t* qgu = reinterpret_cast<int16_t*>(plan + PLAN_QGU);
    int16_t* ttok = reinterpret_cast<int16_t*>(plan + PLAN_TTOK);
    int* misc = reinterpret_cast<int*>(plan + PLAN_MISC);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int M = p.M, E = p.E, topk = p.topk, nslots = M * topk;
    uint32_t* ctrl = p.ctrl;

    // this warp's pipeline block (the agent warp uses all of them)
    const int vp = warp < AGENT_WARP ? warp / VP_WARPS : 0;
    const int vw = warp - vp * VP_WARPS;   // role within the pipeline: 0..3 consumers, VP_PRODUCER, VP_MMA
    uint8_t* vb = smem + vp * VP_BYTES;
    uint8_t* ring = vb + VO_RING;
    uint64_t* full = reinterpret_cast<uint64_t*>(vb + VO_BAR);
    uint64_t* empty = full + NST;
    uint64_t* efull = empty + NST;
    uint64_t* eempty = efull + NEPI;
    StageDesc* desc = reinterpret_cast<StageDesc*>(vb + VO_DESC);
    EpiRec* epi = reinterpret_cast<EpiRec*>(vb + VO_EPI);

    if (tid == 0) {
        for (int v = 0; v < NVP; ++v) {
            uint64_t* f = reinterpret_cast<uint64_t*>(smem + v * VP_BYTES + VO_BAR);
            for (int i = 0; i < NST; ++i) {
                qf::mbar_init(f + i, 1);             // full
                qf::mbar_init(f + NST + i, NCW);     // empty
            }
            for (int i = 0; i < NEPI; ++i) {
                qf::mbar_init(f + 2 * NST + i, NCW);          // efull
                qf::mbar_init(f + 2 * NST + NEPI + i, 1);     // eempty
            }
        }
        qf::mbar_fence_init();
        misc[MISC_DBGN] = 0;
    }
    // fused router: this CTA's router rows (load-time constants) are requested before the wait on the previous
    // kernel; CTA c owns rows [c rpc, c rpc + rpc)
    const bool fused = p.rw != nullptr;
    const int rpc = fused ? (E + (int)gridDim.x - 1) / (int)gridDim.x : 0;
    const int r0 = (int)blockIdx.x * rpc;
    const int nrows = fused ? max(0, min(E, r0 + rpc) - r0) : 0;
    uint8_t* rrows = smem + VP_BYTES;
    if (nrows > 0) {
        const int chunks = nrows * (p.H / 8);
        const char* src = reinterpret_cast<const char*>(p.rw + (size_t)r0 * p.H);
        for (int c = tid; c < chunks; c += MOE_THREADS) qf::cp_async16(rrows + 16 * c, src + 16 * c, 16u);
    }
    // the plan's expert bitmasks live in shared scratch only: cleared before the wait on the previous kernel
    {
        uint64_t* mask = reinterpret_cast<uint64_t*>(smem + SCR_MASK);
        for (int e = tid; e < E; e += MOE_THREADS) mask[e] = 0ull;
        if (tid == 0) misc[MISC_DUPS] = 0;
    }
    __syncthreads();
    // Everything below reads data of the previous kernel (topk ids, x) or the control block it may re-arm.
    qf::pdl_wait();
    // each producer claims its first item now: the atomic's round trip overlaps the routing plan
    int first_item = 0;
    if (warp < AGENT_WARP && vw == VP_PRODUCER && lane == 0) first_item = (int)atomicAdd(ctrl + C_QUEUE, 1u);
    int* rids = reinterpret_cast<int*>(smem + SCR_RIDS);
    float* rtw = reinterpret_cast<float*>(smem + SCR_RTW);
    if (fused && p.xsrc != nullptr) {
        // the layer input is in pinned host memory: each CTA copies its slice into the device copy p.x (one PCIe
        // round trip), then a grid barrier; every later read of x goes to the device copy
        const int nch = M * p.H / 8;
        const int per = (nch + (int)gridDim.x - 1) / (int)gridDim.x;
        const int c1 = min(nch, ((int)blockIdx.x + 1) * per);
        const uint4* src = reinterpret_cast<const uint4*>(p.xsrc);
        uint4* dst = reinterpret_cast<uint4*>(const_cast<__nv_bfloat16*>(p.x));
        for (int c = (int)blockIdx.x * per + tid; c < c1; c += MOE_THREADS) __stcg(dst + c, __ldcv(src + c));
        grid_barrier(ctrl, C_XBAR);
    }
    if (fused) fused_router(p, smem, rrows, r0, nrows, rids, rtw);

    // ------------------------------------------------------------------ routing plan (all threads)
    {
        uint64_t* mask = reinterpret_cast<uint64_t*>(smem + SCR_MASK);
        int16_t* exf = reinterpret_cast<int16_t*>(smem + SCR_EXF);
        int16_t* exc = exf + QF_MAX_EXPERTS;
        int16_t* exg = exc + QF_MAX_EXPERTS;
        int16_t* toffe = reinterpret_cast<int16_t*>(smem + SCR_TOFFE);
        int* chunk = reinterpret_cast<int*>(smem + SCR_CHUNK);
        bool bad = false, dup = false;
        for (int s = tid; s < nslots; s += MOE_THREADS) {
            const int e = fused ? rids[s] : p.ids[s];
            const float twv = fused ? rtw[s] : p.tw[s];
            tws[s] = bf16r(twv);   // the down epilogues read the slot weights from here, not from L2
            if (fused && blockIdx.x == 0 && M <= TOPK_ALL_MAX) {   // the fused router's outputs for the caller
                p.ids_out[s] = e;
                p.tw_out[s] = twv;
            }
            if (e < 0 || e >= E) {
                bad = true;
                sids[s] = -1;
                continue;
            }
            sids[s] = (int16_t)e;
            if (e < p.elo || e >= p.ehi) continue;
            const unsigned long long bit = 1ull << (s / topk);
            // a token that names one expert in two slots (never from the router; possible through the op's API)
            dup |= (atomicOr(reinterpret_cast<unsigned long long*>(mask + e), bit) & bit) != 0ull;
        }
        if (bad) set_err(ctrl, QF_MOE_ERR_BAD_EXPERT);
        if (dup) misc[MISC_DUPS] = 1;
        __syncthreads();
        const int nch = (E + 31) >> 5;
        for (int c = warp; c < nch; c += MOE_THREADS / 32) {
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
                const int ng = (__popcll(mask[e]) + TG - 1) / TG;
                for (int q = 0; q < ng; ++q) qgu[gpre[u] + q] = (int16_t)u;
            }
        }
        if (tid == 0) {
            toff[misc[MISC_U]] = (int16_t)misc[MISC_NTOK];
            gpre[misc[MISC_U]] = (int16_t)misc[MISC_GT];
            make_layout(*reinterpret_cast<Layout*>(plan + PLAN_LAYOUT), p, M, misc[MISC_U], misc[MISC_GT],
                        (int)gridDim.x);
        }
        __syncthreads();
        const bool any_dup = misc[MISC_DUPS] != 0;
        for (int s = tid; s < nslots; s += MOE_THREADS) {
            const int e = sids[s];
            dupn[s] = -1;
            if (e < 0 || e < p.elo || e >= p.ehi) continue;
            const int t = s / topk, kp = s - t * topk;
            bool first = true;
            if (any_dup) {
                for (int k2 = 0; k2 < kp; ++k2) first &= sids[t * topk + k2] != e;
                for (int k2 = topk - 1; k2 > kp; --k2)   // the next slot of this token routed to the same expert
                    if (sids[t * topk + k2] == e) dupn[s] = (int16_t)(t * topk + k2);
            }
            if (first) {
                const int j = __popcll(mask[e] & ((1ull << t) - 1ull));
                tlist[toffe[e] + j] = (int16_t)s;
                ttok[toffe[e] + j] = (int16_t)t;
            }
        }
        __syncthreads();
    }
    qf::pdl_launch_dependents();

    const Layout& L = *reinterpret_cast<const Layout*>(plan + PLAN_LAYOUT);


    if (warp == AGENT_WARP) {
        if (lane == 0) {
            // ========================================================== signal agent (one thread, all pipelines)
            // Consumer warps arrive on efull[slot] of their pipeline after their item's global stores; this thread
            // makes those stores visible at gpu scope (fence) and publishes the item's counter increment. It polls
            // the pipelines' rings without blocking (a suspended wait on one ring would hold up the others).
            // per pipeline v, bits 4v .. 4v + 2: the next record slot, bit 4v + 3: its phase
            static_assert(NEPI == 8 && NVP <= 8, "agent ring state packing");
            uint32_t estate = 0u;
            uint32_t alive = (1u << NVP) - 1u;
            long long idle_since = clock64();
            const long long idle_limit = (long long)(2 * PIPE_WAIT_NS);
            while (alive != 0u) {
                bool any = false;
#pragma unroll
                for (int v = 0; v < NVP; ++v) {
                    if (!(alive & (1u << v))) continue;
                    const int es = (int)((estate >> (4 * v)) & 7u);
                    const uint32_t eph = (estate >> (4 * v + 3)) & 1u;
                    uint8_t* vbv = smem + v * VP_BYTES;
                    uint64_t* ef = reinterpret_cast<uint64_t*>(vbv + VO_BAR) + 2 * NST;
                    if (!qf::mbar_test_wait(ef + es, eph)) continue;
                    const EpiRec r = reinterpret_cast<const EpiRec*>(vbv + VO_EPI)[es];
                    if (r.idx == -2) {   // this pipeline's consumers stopped
                        alive &= ~(1u << v);
                    } else {
                        if (r.idx >= 0) {
                            __threadfence();
                            atomicAdd(ctrl + r.idx, (uint32_t)r.add);
                        }
                        qf::mbar_arrive(ef + NEPI + es);
                        // slot + 1; from slot 7 the carry flips the phase bit (and stays inside the 4-bit field)
                        const uint32_t f = (((estate >> (4 * v)) & 0xFu) + 1u) & 0xFu;
                        estate = (estate & ~(0xFu << (4 * v))) | (f << (4 * v));
                    }
                    any = true;
                }
                if (any) {
                    idle_since = clock64();
                } else {
                    if (clock64() - idle_since > idle_limit) {
                        set_err(ctrl, QF_MOE_ERR_PIPELINE);
                        break;
                    }
                    __nanosleep(64);
                }
            }
        }
        __syncwarp();
    } else if (vw == VP_PRODUCER) {
        if (lane == 0) {
            // ========================================================== producer (one thread)
            const uint64_t pol = qf::policy_evict_first();
            // the copy engine reads x (possibly staged by this launch's own threads) and, later, rows other CTAs wrote:
            // order this thread's view of them (acquired at the barriers and counters) before its copies
            qf::fence_proxy_async();
            int st = 0;
            uint32_t ph = 0;
            // diagnostic mode 2: CTA 0's first producer waits, before its first item, for a dependency that never
            // arrives; the bounded wait runs out, records QF_MOE_ERR_TIMEOUT and the launch drains
            bool never = p.mode == 2 && blockIdx.x == 0 && vp == 0;
            // An item decoded from its queue index: the stage descriptor (written with the item's first stage; the
            // consumers read it once), the weight / scale sources (advanced by a constant per stage), bytes per
            // stage, and the counter that must be acquired before the first stage is marked full (its inputs).
            struct Work {
                StageDesc d;
                const uint8_t* wsrc;
                const uint16_t* ssrc;
                uint32_t bytes, dep_target;
                int dep_idx;               // -1: no input to acquire, or acquired while the item was decoded
                uint32_t rows[TG / 2];     // routed item: its token rows (x row / hbuf slot), two per word; entries
                                           // from ntok on repeat the last row (the tail of a 4-row gather)
            };
            // Decoding is plan arithmetic only (no waits): it runs one item ahead, while the current item's later
            // stages wait for ring slots, so that an item boundary costs the ring no more than a stage does.
            auto decode = [&](int claim) {
                Work w;
                int kind = K_STOP, u = 0, tile = 0, tg = 0, split = 0, nk = 1, ntok = 0, e = 0;
                const int item = L.base + claim;
                if (claim >= L.nq) {
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
                    // gate_up: (tile, k half) pairs, the two halves of a tile next to each other in the queue
                    // token group q (all groups of all routed experts, expert-major), then its R tiles
                    const int R = down ? L.R2 : L.R1 * L.g1s;
                    const int q = j / R;
                    const int th = j - q * R;
                    u = qgu[q];
                    tg = q - gpre[u];
                    tile = down ? th : th >> (L.g1s - 1);
                    split = down ? 0 : th & (L.g1s - 1);
                    kind = down ? K_G2 : K_G1;
                    e = ulist[u];
                    nk = ((down ? p.I : p.H) + W4_KC - 1) / W4_KC >> (down ? 0 : L.g1s - 1);
                    const int tb = toff[u] + TG * tg;
                    ntok = min(TG, toff[u + 1] - tb);
                    const int16_t* tl = (down ? tlist : ttok) + tb;
                    const int npad = ntok >= GATHER_MIN ? (ntok + 3) & ~3 : ntok;
#pragma unroll
                    for (int n = 0; n < TG; n += 2) {
                        if (n >= npad) break;
                        const uint32_t r0 = (uint16_t)tl[min(n, ntok - 1)], r1 = (uint16_t)tl[min(n + 1, ntok - 1)];
                        w.rows[n / 2] = r0 | (r1 << 16);
                    }
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
                    const int j = item - L.b_cb;   // (column tile, group of CB_TOK tokens), tile-major
                    tile = j / L.ngc;
                    tg = j - tile * L.ngc;
                }
                StageDesc& d = w.d;
                d.kind = (int16_t)kind; d.u = (int16_t)u; d.tile = (int16_t)tile; d.tg = (int16_t)tg;
                d.split = (int16_t)split; d.kidx = 0; d.nk = (int16_t)nk; d.ntok = (int16_t)ntok;
                w.wsrc = nullptr;
                w.ssrc = nullptr;
                w.bytes = 0;
                w.dep_idx = -1;
                w.dep_target = 0;
                if (kind == K_G1 || kind == K_G2) {
                    const bool down = kind == K_G2;
                    const int K = down ? p.I : p.H;
                    const int N = down ? p.H : 2 * p.I;
                    d.kc = (int16_t)W4_KC;
                    w.wsrc = (down ? p.w2 : p.w13) + (size_t)(e - p.wofs) * ((size_t)N * K / 2) +
                             (size_t)tile * (128 * (size_t)K / 2) + (size_t)split * nk * STAGE_W;
                    if constexpr (FMT == 0) {
                        w.bytes = STAGE_W + STAGE_S;
                        w.ssrc = (down ? p.s2 : p.s13) + (size_t)(e - p.wofs) * ((size_t)N * K / 128) + (size_t)tile * K +
                                 (size_t)split * nk * W4_KC;
                    } else {
                        // the item's E4M3 scales (1 KB per stage, contiguous) into L2; the consumers load them
                        w.bytes = STAGE_W;
                        qf::prefetch_l2((down ? p.f2 : p.f13) + (size_t)(e - p.wofs) * ((size_t)N * K / 16) +
                                            (size_t)tile * (8 * (size_t)K) + (size_t)split * nk * 1024,
                                        (uint32_t)nk * 1024u);
                    }
                    // (phase 2: the gate_up items completed in the previous launch)
                    if (down && p.phase != 2) {
                        w.dep_idx = C_DONE + u;
                        w.dep_target = (uint32_t)(L.R1 * (gpre[u + 1] - gpre[u]));
                    }
                } else if (kind == K_S1 || kind == K_S2) {
                    const bool down = kind == K_S2;
                    const int K = down ? p.Is : p.H;
                    const int k0 = down ? 0 : split * (p.H / NSPLIT);
                    d.kc = (int16_t)BF_KC;
                    w.bytes = STAGE_W;
                    w.wsrc = (down ? p.shw2 : p.shw13) + (size_t)tile * (128 * (size_t)K * 2) + (size_t)(k0 / BF_KC) * STAGE_W;
                    if (down) { w.dep_idx = C_SDONE + tg; w.dep_target = (uint32_t)L.Rs1; }
                } else {
                    d.kc = 0;
                }
                if (w.bytes != 0) {
                    if (kind == K_S1 || kind == K_S2) w.bytes += (uint32_t)(p.tok_box * BF_KC * 2);
                    else w.bytes += (uint32_t)((ntok >= GATHER_MIN ? (ntok + 3) / 4 * 4 : ntok) * W4_KC * 2);
                }
                return w;
            };
            // the first item was claimed before the plan; the second is claimed now (claims run two items ahead)
            int next = first_item < L.nq ? (int)atomicAdd(ctrl + C_QUEUE, 1u) : L.nq;
            uint32_t herr = 0u;
            Work cur = decode(first_item);
            for (;;) {
                if (never) {
                    never = false;
                    wait_counter(ctrl, C_NEVER, 1u);
                }
                const StageDesc& d = cur.d;
                const int kind = d.kind;
                // dependencies of items without copies are resolved before their (empty) stage is published
                if (kind == K_S1F) wait_counter(ctrl, C_SPLIT + d.tile * L.ngs + d.tg, (uint32_t)NSPLIT);
                if (kind == K_CB) {
                    wait_counter(ctrl, C_CNT + d.tile, L.tile_target);
                    if (L.has_gate && p.phase != 2) wait_counter(ctrl, C_GLF, 1u);   // phase 2: gl is given
                }
                // the k-slice of the item's token rows rides in every stage (token block at STAGE_TOK): the shared
                // expert's consecutive rows as one tensor copy (rows beyond M read zeros), a routed expert's rows one
                // by one (row stride BROW_W4) or, from GATHER_MIN rows, in 4-row gathers (stride BROW_G4; a partial
                // last group repeats its last row). Rows beyond the item's tokens hold stale data: the mma columns
                // they feed are never read.
                const int ntok = d.ntok;
                const bool g4 = (kind == K_G1 || kind == K_G2) && ntok >= GATHER_MIN;
                auto copy_tokens = [&](uint8_t* sb, int kidx) {
                    uint8_t* tb = sb + STAGE_TOK;
                    if (kind == K_S1) {
                        qf::tma_tile_2d(tb, &p.xt, d.split * (p.H / NSPLIT) + kidx * BF_KC, TG * d.tg, full + st);
                    } else if (kind == K_S2) {
                        qf::tma_tile_2d(tb, &p.ht, kidx * BF_KC, TG * d.tg, full + st);
                    } else {
                        const int x0 = (kind == K_G1 ? d.split * (p.H / G1_SPLIT) : 0) + kidx * W4_KC;
                        if (!g4) {   // one or two rows
                            const __nv_bfloat16* base = kind == K_G1 ? p.x : p.hbuf;
                            const size_t ld = kind == K_G1 ? (size_t)p.H : (size_t)p.I;
                            qf::bulk_g2s(tb, base + (size_t)(cur.rows[0] & 0xFFFFu) * ld + x0, W4_KC * 2, full + st);
                            if (ntok > 1)
                                qf::bulk_g2s(tb + BROW_W4, base + (size_t)(cur.rows[0] >> 16) * ld + x0, W4_KC * 2,
                                             full + st);
                        } else {
                            const void* map = kind == K_G1 ? static_cast<const void*>(&p.xg) : static_cast<const void*>(&p.hg);
#pragma unroll
                            for (int n0 = 0; n0 < TG; n0 += 4) {
                                if (n0 >= ntok) break;
                                const uint32_t a = cur.rows[n0 / 2], b = cur.rows[n0 / 2 + 1];
                                qf::tma_gather4(tb + n0 * BROW_G4, map, x0, (int)(a & 0xFFFFu), (int)(a >> 16),
                                                (int)(b & 0xFFFFu), (int)(b >> 16), full + st);
                            }
                        }
                    }
                };
                Work nxt;
                const int nk = d.nk;
                for (int kidx = 0; kidx < nk; ++kidx) {
                    if (!qf::mbar_wait(empty + st, ph ^ 1u, PIPE_WAIT_NS)) set_err(ctrl, QF_MOE_ERR_PIPELINE);
                    uint8_t* sb = ring + st * STAGE_BYTES;
                    if (kidx == 0) desc[st] = d;
                    if (cur.bytes == 0) {
                        qf::mbar_arrive(full + st);
                    } else if (kidx == 0 && cur.dep_idx >= 0) {
                        // weights first; the token rows (the item's inputs, written by other CTAs) are copied, and the
                        // stage is marked full (arrive), only after the inputs are acquired; the proxy fence orders
                        // the copy engine's reads of global memory after that acquire
                        qf::mbar_expect_tx(full + st, cur.bytes);
                        qf::bulk_g2s_hint(sb, cur.wsrc, STAGE_W, full + st, pol);
                        if (cur.ssrc != nullptr) qf::bulk_g2s_hint(sb + STAGE_W, cur.ssrc, STAGE_S, full + st, pol);
                        wait_counter(ctrl, cur.dep_idx, cur.dep_target);
                        qf::fence_proxy_async_global();
                        copy_tokens(sb, kidx);
                        qf::mbar_arrive(full + st);
                    } else {
                        qf::mbar_arrive_expect_tx(full + st, cur.bytes);
                        qf::bulk_g2s_hint(sb, cur.wsrc, STAGE_W, full + st, pol);
                        if (cur.ssrc != nullptr) qf::bulk_g2s_hint(sb + STAGE_W, cur.ssrc, STAGE_S, full + st, pol);
                        copy_tokens(sb, kidx);
                    }
                    cur.wsrc += STAGE_W;
                    if (cur.ssrc != nullptr) cur.ssrc += W4_KC;
                    if (++st == NST) { st = 0; ph ^= 1u; }
                    if (kidx == 0 && kind != K_STOP) {
                        // look ahead: claim the item after the next one and decode the next one; if its input is
                        // complete already, acquire it now (then the proxy fence orders every later copy of this
                        // thread after it). After a hard error anywhere (read one item ahead) the next item is the
                        // stop.
                        const int item = (herr & HARD_ERR) ? L.nq : next;
                        herr = qf::ld_volatile(ctrl + C_ERR);
                        if (item < L.nq) next = (int)atomicAdd(ctrl + C_QUEUE, 1u);
                        nxt = decode(item);
                        if (nxt.dep_idx >= 0 && qf::ld_acquire(ctrl + nxt.dep_idx) >= nxt.dep_target) {
                            nxt.dep_idx = -1;
                            qf::fence_proxy_async_global();
                        }
                    }
                }
                if (kind == K_STOP) break;
                cur = nxt;
            }
        }
        __syncwarp();
    } else {
        // ============================================================== consumers (4 warps per pipeline)
        // Warp rw owns the m16 tiles 2 rw, 2 rw + 1 of every 128-row stage; acc[2 m + n][i] = row 16 (2 rw + m) + g +
        // 8 (i / 2) of the item's tile, token 8 n + 2 t4 + (i % 2) (see stage_w4).
        const int rw = vw;                    // 0..3: consumer warp within the pipeline
        const int ctid = rw * 32 + lane;      // 0..127
        const int g = lane >> 2, t4 = lane & 3;
        int st = 0, es = 0;
        uint32_t ph = 0, eph = 0;
        float acc[4][4];
        // optional timeline: (globaltimer << 12) | tag in the CTA's first 31 entries, tag = event | pipeline << 5;
        // events: 1..7 an item of that kind starts (its first stage is in the ring), 16 + kind its stages are done,
        // DBG_CONSUMERS the pipeline's consumers start (routing plan built), DBG_STOP they stop
        auto stamp = [&](int tag) {
            if (p.dbg != nullptr && ctid == 0 && blockIdx.x < QF_MOE_DBG_NUMEL / 32) {
                const int i = atomicAdd(&misc[MISC_DBGN], 1);
                if (i < 31)
                    p.dbg[blockIdx.x * 32 + i] = (long long)((qf::globaltimer() << 12) | (uint64_t)(tag | (vp << 5)));
            }
        };
        stamp(DBG_CONSUMERS);
        // hand one completion record to the agent (record written by thread 0; every consumer warp arrives)
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
        // the ring slot of a consumed stage goes back to the producer (each warp arrives once it read its part)
        auto release = [&](int slot) {
            __syncwarp();
            if (lane == 0) qf::mbar_arrive(empty + slot);
        };
        auto pipelined = [](int kind) { return kind == K_G1 || kind == K_G2 || kind == K_S1 || kind == K_S2; };
        for (;;) {
            // the item's first stage: every consumer thread of the pipeline takes the same decision (a wait that
            // ran out in one thread ends the pipeline in all of them)
            const bool got = qf::mbar_wait(full + st, ph, PIPE_WAIT_NS);
            if (!qf::named_bar_and(1 + vp, CONS_THREADS, got)) {
                set_err(ctrl, QF_MOE_ERR_PIPELINE);
                signal(-2, 0);
                break;
            }
            const StageDesc d = desc[st];
            if (d.kind == K_STOP) {
                stamp(DBG_STOP);
                signal(-2, 0);
                break;
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
            stamp(d.kind);
            const bool w4 = d.kind == K_G1 || d.kind == K_G2;
            if (pipelined(d.kind)) {
                // ---------------------------------------------------------------- pipelined item: nk stages
                // each warp runs through the stages on its own (a stage arrives whole: weights, scales, token rows)
                const int nk = d.nk;
                const bool two = d.ntok > 8;
                const int brow = d.ntok >= GATHER_MIN ? BROW_G4 : BROW_W4;   // the producer's choice for int4 stages
                bool ok = true;
                // NVFP4: this lane's E4M3 scales of the item's stages (1 KB per stage), one stage loaded ahead
                const uint8_t* fsrc = nullptr;
                uint2 scl = make_uint2(0u, 0u);
                if constexpr (FMT == 1) {
                    if (w4) {
                        const bool down = d.kind == K_G2;
                        const int K = down ? p.I : p.H, N = down ? p.H : 2 * p.I;
                        fsrc = (down ? p.f2 : p.f13) + (size_t)(ulist[d.u] - p.wofs) * ((size_t)N * K / 16) +
                               (size_t)d.tile * (8 * (size_t)K) + (size_t)d.split * d.nk * 1024 + ctid * 8;
                        scl = __ldg(reinterpret_cast<const uint2*>(fsrc));
                    }
                }
                for (int kidx = 0;;) {
                    const uint8_t* sb = ring + st * STAGE_BYTES;
                    const uint8_t* bb = sb + STAGE_TOK;
                    float dd[4][4];
                    if (w4) {
                        if constexpr (FMT == 0) {
                            // the group-128 scales of rows (g, g + 8) of tiles 2 rw, 2 rw + 1
                            const uint2 sc = *reinterpret_cast<const uint2*>(sb + STAGE_W + (rw * 8 + g) * 8);
                            // one code path per token-tile count (the second tile's work only when it exists)
                            auto run = [&](auto two_c) {
                                constexpr bool T2 = decltype(two_c)::value;
                                stage_w4<0, T2>(sb, bb, brow, rw, lane, sc, dd);
                                release(st);
                                const float sr[4] = {bf16_lo(sc.x), bf16_hi(sc.x), bf16_lo(sc.y), bf16_hi(sc.y)};
#pragma unroll
                                for (int j = 0; j < 4; ++j) {
                                    if (!T2 && (j & 1)) continue;
                                    const float s0 = sr[2 * (j >> 1)], s1 = sr[2 * (j >> 1) + 1];
                                    acc[j][0] = fmaf(dd[j][0], s0, acc[j][0]);
                                    acc[j][1] = fmaf(dd[j][1], s0, acc[j][1]);
                                    acc[j][2] = fmaf(dd[j][2], s1, acc[j][2]);
                                    acc[j][3] = fmaf(dd[j][3], s1, acc[j][3]);
                                }
                            };
                            if (two) run(std::true_type{});
                            else run(std::false_type{});
                        } else {
                            if (two) stage_w4<1, true>(sb, bb, brow, rw, lane, scl, dd);
                            else stage_w4<1, false>(sb, bb, brow, rw, lane, scl, dd);
                            release(st);
                            if (kidx + 1 < nk) scl = __ldg(reinterpret_cast<const uint2*>(fsrc + (size_t)(kidx + 1) * 1024));
#pragma unroll
                            for (int j = 0; j < 4; ++j)
#pragma unroll
                                for (int i = 0; i < 4; ++i) acc[j][i] += dd[j][i];
                        }
                    } else {
                        if (two) stage_bf16<true>(sb, bb, rw, lane, dd);
                        else stage_bf16<false>(sb, bb, rw, lane, dd);
                        release(st);
#pragma unroll
                        for (int j = 0; j < 4; ++j)
#pragma unroll
                            for (int i = 0; i < 4; ++i) acc[j][i] += dd[j][i];
                    }
                    if (++st == NST) { st = 0; ph ^= 1u; }
                    if (++kidx == nk) break;
                    if (!qf::mbar_wait(full + st, ph, PIPE_WAIT_NS)) {
                        ok = false;
                        break;
                    }
                }
                // the pipeline's consumer warps agree on the item's outcome before its epilogue
                if (!qf::named_bar_and(1 + vp, CONS_THREADS, ok)) {
                    set_err(ctrl, QF_MOE_ERR_PIPELINE);
                    signal(-2, 0);
                    break;
                }
                stamp(16 + d.kind);
            } else {
                release(st);
                if (++st == NST) { st = 0; ph ^= 1u; }
            }

            // ------------------------------------------------------------ epilogues (item complete)
            // acc[2 m + n][i]: row 16 (2 rw + m) + g + 8 (i / 2) of the tile, token 8 n + 2 t4 + (i % 2); split
            // partials are exchanged in this thread order (16 floats per thread, ctid-major)
            if (d.kind == K_GL) {
                for (int tok = rw; tok < M; tok += NCW) {
                    const float a = gate_logit(p.x + (size_t)tok * p.H, p.wgate, p.H, lane);
                    if (lane == 0) p.gl[tok] = a;
                }
                signal(C_GLF, 1);
            } else if (d.kind == K_G1 || d.kind == K_S1F) {
                if (d.kind == K_G1 && L.g1s > 1) {
                    // one k half of the tile: publish this half's partials, count it; the half counted second
                    // adds the other half's partials (a + b: the same bits whichever half comes second) and runs
                    // the SwiGLU epilogue. The counter is left at zero for the next launch.
                    const int unit = (gpre[d.u] + d.tg) * L.R1 + d.tile;
                    uint32_t* cnt = reinterpret_cast<uint32_t*>(p.pbuf) + unit;
                    float* parts = p.pbuf + L.g1_part_off + (size_t)unit * G1_SPLIT * 2048;
                    float* mine = parts + (size_t)d.split * 2048 + ctid * 16;
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        __stcg(reinterpret_cast<float4*>(mine + 4 * j), make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]));
                    __threadfence();
                    qf::named_bar(1 + vp, CONS_THREADS);
                    volatile int* gflag = reinterpret_cast<volatile int*>(vb + VO_FLAG);
                    if (ctid == 0) {
                        const bool last = atomicAdd(cnt, 1u) == (uint32_t)(L.g1s - 1);
                        if (last) {
                            __threadfence();
                            *cnt = 0u;
                        }
                        *gflag = last ? 1 : 0;
                    }
                    qf::named_bar(1 + vp, CONS_THREADS);
                    const bool last = *gflag != 0;
                    qf::named_bar(1 + vp, CONS_THREADS);   // every thread has read the flag before its next use
                    if (!last) continue;
#pragma unroll
                    for (int sp = 0; sp < G1_SPLIT; ++sp) {
                        if (sp == d.split || sp >= L.g1s) continue;
                        const float* other = parts + (size_t)sp * 2048 + ctid * 16;
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const float4 q = __ldcg(reinterpret_cast<const float4*>(other + 4 * j));
                            acc[j][0] += q.x; acc[j][1] += q.y; acc[j][2] += q.z; acc[j][3] += q.w;
                        }
                    }
                }
                if (d.kind == K_S1F) {
                    const float* pb = p.pbuf + L.sh_off + (size_t)((d.tile * L.ngs + d.tg) * NSPLIT) * 2048 + ctid * 16;
#pragma unroll
                    for (int sp = 0; sp < NSPLIT; ++sp) {   // fixed split order: the sum does not depend on timing
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const float4 q = __ldcg(reinterpret_cast<const float4*>(pb + (size_t)sp * 2048 + 4 * j));
                            acc[j][0] += q.x; acc[j][1] += q.y; acc[j][2] += q.z; acc[j][3] += q.w;
                        }
                    }
                }
                // fragment row g is gate row j = 64 tile + 8 (2 rw + m) + g, row g + 8 its up row: elements (0, 1)
                // and (2, 3) of acc[2 m + n] are (gate, up) of tokens 8 n + 2 t4 and + 1
                // the destination rows of the lane's four tokens (j = 2 n + h: token 8 n + 2 t4 + h; -1: none), loaded
                // before the math (independent shared-memory loads): hbuf by slot for a routed expert, the shared
                // expert's h by token. The shared expert has no global multiplier (gs = 1: bf16r(bf16r(g) * 1) is
                // bf16r(g)).
                const bool routed = d.kind == K_G1;
                float gs = 1.f;
                int tbase = 0;
                if (routed) {
                    const int e = ulist[d.u];
                    gs = p.gs13 ? bf16_bits(p.gs13[e - p.wofs]) : 1.f;
                    tbase = toff[d.u] + TG * d.tg;
                }
                int row[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int tok = 8 * (j >> 1) + 2 * t4 + (j & 1);
                    row[j] = tok >= d.ntok ? -1 : (routed ? tlist[tbase + tok] : TG * d.tg + tok);
                }
                __nv_bfloat16* const dst = routed ? p.hbuf : p.hsh;
                const int ldd = routed ? p.I : p.Is;
#pragma unroll
                for (int m = 0; m < 2; ++m) {
                    const int col = 64 * d.tile + 8 * (2 * rw + m) + g;
#pragma unroll
                    for (int n = 0; n < (d.ntok > 8 ? 2 : 1); ++n)   // the second token tile only when it has tokens
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const int r = row[2 * n + h];
                            if (r < 0) continue;
                            const float g0 = acc[2 * m + n][h], u0 = acc[2 * m + n][2 + h];
                            const float gv = bf16r(bf16r(g0) * gs), uv = bf16r(bf16r(u0) * gs);
                            dst[(size_t)r * ldd + col] = __float2bfloat16(gv / (1.f + __expf(-gv)) * uv);
                        }
                }
                signal(d.kind == K_G1 ? C_DONE + d.u : C_SDONE + d.tg, 1);
            } else if (d.kind == K_S1) {
                float* pb = p.pbuf + L.sh_off + (size_t)((d.tile * L.ngs + d.tg) * NSPLIT + d.split) * 2048 + ctid * 16;
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    __stcg(reinterpret_cast<float4*>(pb + 4 * j), make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]));
                signal(C_SPLIT + d.tile * L.ngs + d.tg, 1);
            } else if (d.kind == K_G2) {
                const int u = d.u, e = ulist[u];
                const float g2 = p.gs2 ? bf16_bits(p.gs2[e - p.wofs]) : 1.f;
                const int tbase = toff[u] + TG * d.tg;
                // the first slot of each of the lane's four tokens routed to e (j = 2 n + h: token 8 n + 2 t4 + h;
                // -1: none) and its weight, loaded before any store (independent shared-memory loads)
                int sl[4];
                float wt[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int tok = 8 * (j >> 1) + 2 * t4 + (j & 1);
                    sl[j] = tok < d.ntok ? tlist[tbase + tok] : -1;
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) wt[j] = sl[j] >= 0 ? bf16r(g2 * tws[sl[j]]) : 0.f;
#pragma unroll
                for (int m = 0; m < 2; ++m)
#pragma unroll
                    for (int n = 0; n < (d.ntok > 8 ? 2 : 1); ++n)   // the second token tile only when it has tokens
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int j = 2 * n + (i & 1);
                            if (sl[j] < 0) continue;
                            const int n0 = 128 * d.tile + 16 * (2 * rw + m) + g + 8 * (i >> 1);
                            p.ybuf[(size_t)sl[j] * p.H + n0] = __float2bfloat16(bf16r(acc[2 * m + n][i]) * wt[j]);
                        }
                if (misc[MISC_DUPS] != 0) {
                    // a token that names e in more than one slot (possible only through the op's API): the same
                    // row, weighted by each later slot's weight, into that slot
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        if (sl[j] < 0) continue;
                        for (int s = dupn[sl[j]]; s >= 0; s = dupn[s]) {
                            const float w = bf16r(g2 * tws[s]);
#pragma unroll
                            for (int m = 0; m < 2; ++m)
#pragma unroll
                                for (int i = (j & 1); i < 4; i += 2) {
                                    const int n0 = 128 * d.tile + 16 * (2 * rw + m) + g + 8 * (i >> 1);
                                    p.ybuf[(size_t)s * p.H + n0] = __float2bfloat16(bf16r(acc[2 * m + (j >> 1)][i]) * w);
                                }
                        }
                    }
                }
                signal(C_CNT + d.tile, 1);
            } else if (d.kind == K_S2) {
#pragma unroll
                for (int m = 0; m < 2; ++m)
#pragma unroll
                    for (int n = 0; n < (d.ntok > 8 ? 2 : 1); ++n)   // the second token tile only when it has tokens
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int tok = 8 * n + 2 * t4 + (i & 1);
                            if (tok >= d.ntok) continue;
                            const int n0 = 128 * d.tile + 16 * (2 * rw + m) + g + 8 * (i >> 1);
                            p.sbuf[(size_t)(TG * d.tg + tok) * p.H + n0] = __float2bfloat16(acc[2 * m + n][i]);
                        }
                signal(C_CNT + d.tile, 1);
            } else if (d.kind == K_CB) {
                // the producer acquired every producer of this tile (and the gate logits) before publishing it
                if (p.mode != 1) combine_tile(p, L, sids, d.tile, d.tg, ctid);
                else shard_tile(p, L, sids, d.tile, d.tg, ctid);
                signal(-1, 0);
            }
        }
    }

    // ------------------------------------------------------------------ exit: the last CTA re-arms ctrl
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        misc[MISC_FLAG] = atomicAdd(ctrl + C_EXIT, 1u) == gridDim.x - 1;
    }
    __syncwarp();
    __syncthreads();
    if (misc[MISC_FLAG]) {
        __threadfence();
        for (int i = tid; i < QF_MOE_CTRL_MIRROR; i += MOE_THREADS)
            if (i != C_ERR) ctrl[i] = 0u;
        if (tid == 0) {   // the sticky error word, copied to the caller's host-mapped mirror word (if any)
            const uint32_t err = qf::ld_volatile(ctrl + C_ERR);
            const uint64_t mirror = (uint64_t)ctrl[QF_MOE_CTRL_MIRROR] | ((uint64_t)ctrl[QF_MOE_CTRL_MIRROR + 1] << 32);
            if (err != 0u && mirror != 0ull) {
                *reinterpret_cast<volatile uint32_t*>(mirror) = err;
                __threadfence_system();
            }
        }
    }
}

// ------------------------------------------------------------------------------------------ weight repacking
// Kernel layouts (one expert matrix [N, K]; qwenfast_b200/formats.py computes the same maps with torch):
//   128-row tiles; inside a tile, m16 tile m holds rows 16 m .. 16 m + 15 (plain), or for gate_up ("gated") gate rows
//   64 r + 8 m + g at fragment rows g = 0..7 and the matching up rows N/2 + 64 r + 8 m + g at fragment rows 8 + g.
//   int4 stage (128 k = one scale group, 8 KB): [m16 tile m (8)][64-k half h (2)][lane (32)][step s (4)] words; the
//   word of lane (g, t4) holds rows A = 16 m + g and B = A + 8 at k = 128 st + 64 h + 16 t4 + 4 s + (0..3), nibbles
//   0, 4, 2, 6 = A's k+0, k+1, k+2, k+3 and 1, 5, 3, 7 = B's (so pair j = nibbles (j, j + 4) is A register j of the
//   mma step). Scales per stage: [consumer warp w (4)][g (8)][c (4)] bf16, row 16 (2 w + c / 2) + g + 8 (c % 2).
//   bf16 stage (32 k, 8 KB): [m16 tile m (8)][step s (2)][lane (32)][8 elements], element 2 w + h of lane (g, t4) =
//   row 16 m + g + 8 (w % 2), k = 32 st + 8 t4 + 4 s + 2 (w / 2) + h.
__device__ __forceinline__ int kernel_row_to_src(int pos, int N, int gated) {
    if (!gated) return pos;
    const int r = pos >> 7, rho = pos & 127;
    const int j = 64 * r + 8 * (rho >> 4) + (rho & 7);
    return (rho & 8) ? N / 2 + j : j;
}

// word o of an expert's int4 kernel-layout matrix -> its two source rows and the first of its four k
__device__ __forceinline__ void w4_word_src(long long o, int N, int K, int gated, int& ra, int& rb, int& k0) {
    const long long per_tile = 128LL * K / 8;
    const int r = (int)(o / per_tile);
    const int ot = (int)(o - r * per_tile);
    const int st = ot >> 11, os = ot & 2047;
    const int s = os & 3, lane = (os >> 2) & 31, h = (os >> 7) & 1, m = os >> 8;
    k0 = 128 * st + 64 * h + 16 * (lane & 3) + 4 * s;
    ra = kernel_row_to_src(128 * r + 16 * m + (lane >> 2), N, gated);
    rb = kernel_row_to_src(128 * r + 16 * m + (lane >> 2) + 8, N, gated);
}

__device__ __forceinline__ void w4_scale_src(long long o, int N, int K, int gated, int& row, int& grp) {
    const int r = (int)(o / K);
    const int ot = (int)(o - (long long)r * K);
    grp = ot >> 7;
    const int e = ot & 127, w = e >> 5, g = (e >> 2) & 7, c = e & 3;
    row = kernel_row_to_src(128 * r + 16 * (2 * w + (c >> 1)) + g + 8 * (c & 1), N, gated);
}

// four codes (k+0..k+3, low nibble first) of rows A and B -> the kernel word, and back
__device__ __forceinline__ uint32_t w4_spread(uint32_t a, uint32_t b) {
    const int pos[4] = {0, 4, 2, 6};   // nibble of k+j
    uint32_t o = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) o |= (((a >> (4 * j)) & 0xFu) << (4 * pos[j])) | (((b >> (4 * j)) & 0xFu) << (4 * pos[j] + 4));
    return o;
}
__device__ __forceinline__ uint32_t w4_gather(uint32_t w, int rowb) {
    const int pos[4] = {0, 4, 2, 6};
    uint32_t o = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) o |= ((w >> (4 * pos[j] + 4 * rowb)) & 0xFu) << (4 * j);
    return o;
}

__global__ void w4_repack_kernel(const uint32_t* __restrict__ src, const uint16_t* __restrict__ ssrc,
                                 uint32_t* __restrict__ dst, uint16_t* __restrict__ sdst, int E, int N, int K,
                                 int gated, int unpack) {
    const long long words = (long long)N * K / 8, ents = (long long)N * K / 128;
    const long long total = (long long)E * words;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const long long e = i / words, o = i - e * words;
        int ra, rb, k0;
        w4_word_src(o, N, K, gated, ra, rb, k0);
        // the canonical half-words (four codes each) of rows A and B at k0
        const long long ha = (e * words + (long long)ra * (K / 8) + k0 / 8) * 2 + ((k0 >> 2) & 1);
        const long long hb = (e * words + (long long)rb * (K / 8) + k0 / 8) * 2 + ((k0 >> 2) & 1);
        if (!unpack) {
            const uint16_t* h = reinterpret_cast<const uint16_t*>(src);
            dst[i] = w4_spread(h[ha], h[hb]);
        } else {
            uint16_t* h = reinterpret_cast<uint16_t*>(dst);
            h[ha] = (uint16_t)w4_gather(src[i], 0);
            h[hb] = (uint16_t)w4_gather(src[i], 1);
        }
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
        const int st = ot >> 12, os = ot & 4095;
        const int el = os & 7, lane = (os >> 3) & 31, s = (os >> 8) & 1, m = os >> 9;
        const int w = el >> 1, h = el & 1;
        const int k = 32 * st + 8 * (lane & 3) + 4 * s + 2 * (w >> 1) + h;
        const int row = kernel_row_to_src(128 * r + 16 * m + (lane >> 2) + 8 * (w & 1), N, gated);
        const long long si = (long long)row * K + k;
        if (!unpack) dst[o] = src[si];
        else dst[si] = src[o];
    }
}

// Expert-parallel finish, one CTA per token: ybuf = the shards' slot buffers summed (each slot has exactly one
// owner, so the sum is exact), laid out as in mode 1; out = the mode-0 combine of it, bit for bit (same gate logit
// and combine arithmetic; the zero slots of other shards add exactly nothing).
constexpr int COMBINE_THREADS = 256;
__global__ void __launch_bounds__(COMBINE_THREADS) moe_combine_kernel(const __nv_bfloat16* __restrict__ ybuf,
                                                                      const __nv_bfloat16* __restrict__ x,
                                                                      const __nv_bfloat16* __restrict__ wgate,
                                                                      bool has_shared, __nv_bfloat16* __restrict__ out,
                                                                      int M, int H, int topk) {
    __shared__ float s_gl;
    const int t = blockIdx.x, tid = threadIdx.x;
    qf::pdl_wait();
    if (has_shared && tid < 32) {
        const float a = gate_logit(x + (size_t)t * H, wgate, H, tid);
        if (tid == 0) s_gl = a;
    }
    __syncthreads();
    qf::pdl_launch_dependents();
    const float gl = has_shared ? s_gl : 0.f;
    for (int n = 8 * tid; n < H; n += 8 * COMBINE_THREADS) {
        float a[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) a[j] = 0.f;
        for (int k0 = 0; k0 < topk; k0 += 8) {   // eight slots' loads in flight, sums in top-k order
            uint4 v[8];
#pragma unroll
            for (int b = 0; b < 8; ++b)
                if (k0 + b < topk) v[b] = __ldcg(reinterpret_cast<const uint4*>(ybuf + (size_t)(t * topk + k0 + b) * H + n));
#pragma unroll
            for (int b = 0; b < 8; ++b)
                if (k0 + b < topk) add8(a, v[b]);
        }
        const uint4 sv = has_shared ? __ldcg(reinterpret_cast<const uint4*>(ybuf + (size_t)(M * topk + t) * H + n))
                                    : make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(out + (size_t)t * H + n) = finish8(a, has_shared, gl, sv);
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
    if (pbuf_numel) {
        // the zero-kept gate_up k-half counters (sized for QF_MAX_TOKENS: their place does not depend on M), the
        // shared expert's split-K partials, the gate_up k-half partials (at most M * topk token groups of routed
        // experts, 2I / 128 tiles each). Everything after the counters grows with M, so a workspace sized for the
        // largest M serves every smaller M.
        const int64_t cnt = ((int64_t)QF_MAX_TOKENS * topk * (2 * I / 128) + 3) & ~(int64_t)3;
        const int64_t sh = Is > 0 ? (int64_t)(2 * Is / 128) * ngs * NSPLIT * 2048 : 0;
        const int64_t units = (int64_t)M * topk * (2 * I / 128);
        *pbuf_numel = cnt + sh + units * G1_SPLIT * 2048;
    }
    if (shbuf_bytes) *shbuf_bytes = Is > 0 ? (int64_t)M * (Is + H) * 2 : 0;
    return QF_OK;
}

namespace {
struct FusedRouter {   // the router inputs and outputs of qf_moe_layer_decode
    const void* w;
    int renorm;
    void* logits;
    void* x_stage;   // device copy of x when x is in pinned host memory, or nullptr
};

int moe_launch(const void* x, const int32_t* topk_ids, const float* topk_w, const int32_t* w13, const void* s13,
               const void* gs13, const int32_t* w2, const void* s2, const void* gs2, const void* w_gate,
               const void* shared, const void* sh_w13, const void* sh_w2, void* hbuf, int64_t hbuf_bytes, void* ybuf,
               int64_t ybuf_bytes, float* gl, int64_t gl_numel, int32_t* ctrl, int64_t ctrl_numel, float* pbuf,
               int64_t pbuf_numel, void* shbuf, int64_t shbuf_bytes, void* out, int M, int H, int I, int E, int topk,
               int Is, int phase, int mode, int expert_lo, int expert_hi, int64_t* dbg, int pdl, qf_stream_t stream,
               const FusedRouter* fr, int fmt = 0) {
    QF_REQUIRE(x && topk_ids && topk_w && w13 && s13 && w2 && s2 && hbuf && ybuf && gl && ctrl && out,
               "a16_moe_decode: null pointer argument");
    QF_REQUIRE(phase >= 1 && phase <= 4, "a16_moe_decode: phase must be 1, 2, 3 or 4, got %d", phase);
    QF_REQUIRE(mode == 0 || mode == 1 || mode == 2,
               "a16_moe_decode: mode must be 0 (full layer), 1 (expert-parallel shard) or 2 (diagnostic), got %d",
               mode);
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
    if (phase <= 2) {   // the reference's split phases: gate_up (1) and down + combine (2) as separate launches
        QF_REQUIRE(!has_shw, "a16_moe_decode: shared-expert weights need the whole layer (phase 3 or 4), got phase %d",
                   phase);
        QF_REQUIRE(mode == 0 && fr == nullptr, "a16_moe_decode: phases 1 and 2 run the full layer without the router");
    }
    int64_t need_h, need_y, need_gl, need_ctrl, need_p, need_sh;
    qf_a16_moe_workspace(M, H, I, topk, has_shw ? Is : 0, &need_h, &need_y, &need_gl, &need_ctrl, &need_p, &need_sh);
    QF_REQUIRE(hbuf_bytes >= need_h && ybuf_bytes >= need_y && gl_numel >= need_gl && ctrl_numel >= need_ctrl,
               "a16_moe_decode: scratch too small (need hbuf %lld B, ybuf %lld B, gl %lld, ctrl %lld)", (long long)need_h,
               (long long)need_y, (long long)need_gl, (long long)need_ctrl);
    QF_REQUIRE(pbuf && pbuf_numel >= need_p && (!has_shw || shbuf_bytes >= need_sh),
               "a16_moe_decode: pbuf / shared scratch too small (need pbuf %lld, shbuf %lld B)", (long long)need_p,
               (long long)need_sh);
    const void* al[] = {x, w13, s13, w2, s2, hbuf, ybuf, out, w_gate, shared, sh_w13, sh_w2, pbuf, shbuf};
    for (const void* a : al) QF_REQUIRE(a == nullptr || qf::aligned(a, 16), "a16_moe_decode: every tensor must be 16-byte aligned");

    int dev = 0;
    cudaError_t ce = cudaGetDevice(&dev);
    if (ce != cudaSuccess) return qf::cuda_status(ce, "a16_moe_decode: cudaGetDevice");
    const int sms = qf::sm_count(dev);
    QF_REQUIRE(sms > 0, "a16_moe_decode: cannot query the SM count");
    if (fr != nullptr) {
        QF_REQUIRE(fr->w && fr->logits, "moe_layer_decode: null router weight or logits");
        QF_REQUIRE(qf::aligned(fr->w, 16), "moe_layer_decode: the router weight must be 16-byte aligned");
        QF_REQUIRE(H % 256 == 0 && H <= 4096, "moe_layer_decode: H must be a multiple of 256 <= 4096, got %d", H);
        const int rpc = (E + sms - 1) / sms;
        QF_REQUIRE(rpc <= RPC_MAX && (int64_t)rpc * H * 2 <= RROWS_BYTES,
                   "moe_layer_decode: %d router rows per CTA of %d do not fit (E %d, H %d)", rpc, sms, E, H);
        QF_REQUIRE(fr->x_stage == nullptr || qf::aligned(fr->x_stage, 16),
                   "moe_layer_decode: x_stage must be 16-byte aligned");
    }
    if (fmt == 1) {
        QF_REQUIRE(I % 128 == 0 && H % 128 == 0, "a16_moe_decode_nvfp4: H and I must be multiples of 128");
    }
    void (*kern)(Params) = fmt == 1 ? moe_persistent_kernel<1> : moe_persistent_kernel<0>;
    ce = qf::ensure_smem_attr(reinterpret_cast<const void*>(kern), MOE_SMEM);
    if (ce != cudaSuccess) return qf::cuda_status(ce, "a16_moe_decode: cudaFuncSetAttribute");
    static bool carveout_set[2][64] = {{false}};
    if (dev >= 64 || !carveout_set[fmt][dev]) {
        // the CTA needs the largest shared-memory carveout; without the hint the driver may pick a smaller one
        ce = cudaFuncSetAttribute(reinterpret_cast<const void*>(kern), cudaFuncAttributePreferredSharedMemoryCarveout,
                                  (int)cudaSharedmemCarveoutMaxShared);
        if (ce != cudaSuccess) return qf::cuda_status(ce, "a16_moe_decode: cudaFuncSetAttribute (carveout)");
        if (dev < 64) carveout_set[fmt][dev] = true;
    }
    // Grid: one CTA per SM (three pipelines each; the shared memory of one CTA fills the SM). The item queue
    // needs no co-residency (an item only waits for items claimed before it, by pipelines that are already running),
    // but the fused router's grid barriers (its logits; x copied from host memory) need every CTA resident at once:
    // that launch is cooperative, so the runtime either co-schedules the whole grid or refuses it (then this entry
    // returns QF_ERR_UNSUPPORTED and the caller takes the two-launch path: router_topk, then a16_moe_decode).

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
    p.phase = phase <= 2 ? phase : 0;
    p.wofs = mode == 1 ? expert_lo : 0;
    p.f13 = p.f2 = nullptr;
    if (fmt == 1) {   // s13 / s2 are the E4M3 group-16 scales
        p.f13 = static_cast<const uint8_t*>(s13);
        p.f2 = static_cast<const uint8_t*>(s2);
        p.s13 = p.s2 = nullptr;
    }
    p.rw = fr ? static_cast<const __nv_bfloat16*>(fr->w) : nullptr;
    p.logits = fr ? static_cast<__nv_bfloat16*>(fr->logits) : nullptr;
    p.ids_out = fr ? const_cast<int*>(topk_ids) : nullptr;
    p.tw_out = fr ? const_cast<float*>(topk_w) : nullptr;
    p.renorm = fr ? (fr->renorm != 0) : 0;
    p.xsrc = nullptr;
    if (fr && fr->x_stage) {   // x is pinned host memory (read by the kernel through its mapping); x_stage its copy
        p.xsrc = p.x;
        p.x = static_cast<const __nv_bfloat16*>(fr->x_stage);
    }
    // tensor maps of the token-row sources (the copy engine's view of x, hbuf and the shared expert's h)
    {
        qf::EncodeTiled enc = nullptr;
        ce = qf::encode_tiled_fn(&enc);
        if (ce != cudaSuccess) return qf::cuda_status(ce, "a16_moe_decode: cuTensorMapEncodeTiled entry point");
        auto encode2d = [&](CUtensorMap* m, const void* base, int rows, int cols, int box_cols, int box_rows) {
            const cuuint64_t gdim[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
            const cuuint64_t gstride[1] = {(cuuint64_t)cols * 2};
            const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
            const cuuint32_t estr[2] = {1, 1};
            return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), gdim, gstride, box, estr,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        };
        p.tok_box = M < TG ? M : TG;
        CUresult cr = encode2d(&p.xt, p.x, M, H, BF_KC, p.tok_box);
        if (cr == CUDA_SUCCESS) cr = encode2d(&p.xg, p.x, M, H, W4_KC, 1);
        if (cr == CUDA_SUCCESS) cr = encode2d(&p.hg, p.hbuf, M * topk, I, W4_KC, 1);
        if (cr == CUDA_SUCCESS && has_shw) cr = encode2d(&p.ht, p.hsh, M, Is, BF_KC, p.tok_box);
        else if (!has_shw) p.ht = p.xt;   // no shared-expert down items read it
        QF_REQUIRE(cr == CUDA_SUCCESS, "a16_moe_decode: cuTensorMapEncodeTiled failed (%d)", (int)cr);
    }
    if (fr != nullptr) {
        ce = qf::launch_coop(kern, dim3(sms * CTAS_PER_SM), dim3(MOE_THREADS), MOE_SMEM,
                             reinterpret_cast<cudaStream_t>(stream), pdl != 0, p);
        if (ce == cudaErrorCooperativeLaunchTooLarge) {
            (void)cudaGetLastError();
            qf::set_error("moe_layer_decode: the %d CTAs of the fused layer-step cannot all be resident (grid barriers); "
                          "use router_topk + a16_moe_decode", sms * CTAS_PER_SM);
            return QF_ERR_UNSUPPORTED;
        }
        return qf::cuda_status(ce, "moe_layer_decode: launch");
    }
    ce = qf::launch_ex(kern, dim3(sms * CTAS_PER_SM), dim3(MOE_THREADS), MOE_SMEM,
                       reinterpret_cast<cudaStream_t>(stream), pdl != 0, p);
    return qf::cuda_status(ce, "a16_moe_decode: launch");
}
}  // namespace

extern "C" int qf_a16_moe_decode(const void* x, const int32_t* topk_ids, const float* topk_w, const int32_t* w13,
                                 const void* s13, const void* gs13, const int32_t* w2, const void* s2, const void* gs2,
                                 const void* w_gate, const void* shared, const void* sh_w13, const void* sh_w2,
                                 void* hbuf, int64_t hbuf_bytes, void* ybuf, int64_t ybuf_bytes, float* gl,
                                 int64_t gl_numel, int32_t* ctrl, int64_t ctrl_numel, float* pbuf, int64_t pbuf_numel,
                                 void* shbuf, int64_t shbuf_bytes, void* out, int M, int H, int I, int E, int topk,
                                 int Is, int phase, int mode, int expert_lo, int expert_hi, int64_t* dbg, int pdl,
                                 qf_stream_t stream) {
    return moe_launch(x, topk_ids, topk_w, w13, s13, gs13, w2, s2, gs2, w_gate, shared, sh_w13, sh_w2, hbuf,
                      hbuf_bytes, ybuf, ybuf_bytes, gl, gl_numel, ctrl, ctrl_numel, pbuf, pbuf_numel, shbuf,
                      shbuf_bytes, out, M, H, I, E, topk, Is, phase, mode, expert_lo, expert_hi, dbg, pdl, stream,
                      nullptr);
}

extern "C" int qf_a16_moe_decode_nvfp4(const void* x, const int32_t* topk_ids, const float* topk_w,
                                       const int32_t* w13, const void* f13, const void* gs13, const int32_t* w2,
                                       const void* f2, const void* gs2, const void* w_gate, const void* shared,
                                       const void* sh_w13, const void* sh_w2, void* hbuf, int64_t hbuf_bytes, void* ybuf,
                                       int64_t ybuf_bytes, float* gl, int64_t gl_numel, int32_t* ctrl,
                                       int64_t ctrl_numel, float* pbuf, int64_t pbuf_numel, void* shbuf,
                                       int64_t shbuf_bytes, void* out, int M, int H, int I, int E, int topk, int Is,
                                       int phase, int mode, int expert_lo, int expert_hi, int64_t* dbg, int pdl,
                                       qf_stream_t stream) {
    return moe_launch(x, topk_ids, topk_w, w13, f13, gs13, w2, f2, gs2, w_gate, shared, sh_w13, sh_w2, hbuf,
                      hbuf_bytes, ybuf, ybuf_bytes, gl, gl_numel, ctrl, ctrl_numel, pbuf, pbuf_numel, shbuf,
                      shbuf_bytes, out, M, H, I, E, topk, Is, phase, mode, expert_lo, expert_hi, dbg, pdl, stream,
                      nullptr, 1);
}

extern "C" int qf_moe_layer_decode(const void* x, void* x_stage, const void* router_w, int renormalize, float* topk_w,
                                   int32_t* topk_ids, void* logits, const int32_t* w13, const void* s13,
                                   const void* gs13, const int32_t* w2, const void* s2, const void* gs2,
                                   const void* w_gate, const void* shared, const void* sh_w13, const void* sh_w2,
                                   void* hbuf, int64_t hbuf_bytes, void* ybuf, int64_t ybuf_bytes, float* gl,
                                   int64_t gl_numel, int32_t* ctrl, int64_t ctrl_numel, float* pbuf,
                                   int64_t pbuf_numel, void* shbuf, int64_t shbuf_bytes, void* out, int M, int H,
                                   int I, int E, int topk, int Is, int mode, int expert_lo, int expert_hi,
                                   int64_t* dbg, int pdl, qf_stream_t stream) {
    const FusedRouter fr{router_w, renormalize, logits, x_stage};
    return moe_launch(x, topk_ids, topk_w, w13, s13, gs13, w2, s2, gs2, w_gate, shared, sh_w13, sh_w2, hbuf,
                      hbuf_bytes, ybuf, ybuf_bytes, gl, gl_numel, ctrl, ctrl_numel, pbuf, pbuf_numel, shbuf,
                      shbuf_bytes, out, M, H, I, E, topk, Is, 4, mode, expert_lo, expert_hi, dbg, pdl, stream, &fr);
}

extern "C" int qf_moe_layer_decode_nvfp4(const void* x, void* x_stage, const void* router_w, int renormalize,
                                         float* topk_w, int32_t* topk_ids, void* logits, const int32_t* w13,
                                         const void* f13, const void* gs13, const int32_t* w2, const void* f2,
                                         const void* gs2, const void* w_gate, const void* shared, const void* sh_w13,
                                         const void* sh_w2, void* hbuf, int64_t hbuf_bytes, void* ybuf,
                                         int64_t ybuf_bytes, float* gl, int64_t gl_numel, int32_t* ctrl,
                                         int64_t ctrl_numel, float* pbuf, int64_t pbuf_numel, void* shbuf,
                                         int64_t shbuf_bytes, void* out, int M, int H, int I, int E, int topk, int Is,
                                         int mode, int expert_lo, int expert_hi, int64_t* dbg, int pdl,
                                         qf_stream_t stream) {
    const FusedRouter fr{router_w, renormalize, logits, x_stage};
    return moe_launch(x, topk_ids, topk_w, w13, f13, gs13, w2, f2, gs2, w_gate, shared, sh_w13, sh_w2, hbuf,
                      hbuf_bytes, ybuf, ybuf_bytes, gl, gl_numel, ctrl, ctrl_numel, pbuf, pbuf_numel, shbuf,
                      shbuf_bytes, out, M, H, I, E, topk, Is, 4, mode, expert_lo, expert_hi, dbg, pdl, stream, &fr, 1);
}

extern "C" int qf_moe_combine(const void* ybuf, const void* x, const void* w_gate, int has_shared, void* out, int M,
                              int H, int topk, int pdl, qf_stream_t stream) {
    QF_REQUIRE(ybuf && x && out, "moe_combine: null pointer argument");
    QF_REQUIRE(!has_shared || w_gate, "moe_combine: a shared term needs w_gate");
    QF_REQUIRE(M >= 1 && M <= QF_MAX_TOKENS, "moe_combine: M must be in [1, %d], got %d", QF_MAX_TOKENS, M);
    QF_REQUIRE(H >= 128 && H % 128 == 0 && H <= 8192, "moe_combine: H must be a multiple of 128 in [128, 8192], got %d", H);
    QF_REQUIRE(topk >= 1 && topk <= QF_MAX_TOPK, "moe_combine: topk must be in [1, %d], got %d", QF_MAX_TOPK, topk);
    QF_REQUIRE(qf::aligned(ybuf, 16) && qf::aligned(x, 16) && qf::aligned(out, 16) && (!w_gate || qf::aligned(w_gate, 16)),
               "moe_combine: ybuf, x, w_gate and out need 16-byte alignment");
    const cudaError_t e = qf::launch_ex(moe_combine_kernel, dim3(M), dim3(COMBINE_THREADS), 0,
                                        reinterpret_cast<cudaStream_t>(stream), pdl != 0,
                                        static_cast<const __nv_bfloat16*>(ybuf), static_cast<const __nv_bfloat16*>(x),
                                        static_cast<const __nv_bfloat16*>(w_gate), has_shared != 0,
                                        static_cast<__nv_bfloat16*>(out), M, H, topk);
    return qf::cuda_status(e, "moe_combine: launch");
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
    QF_REQUIRE(N >= 128 && N % 128 == 0 && K >= 32 && K % 32 == 0, "bf16_repack: need N %% 128 == 0 and K %% 32 == 0");
    bf16_repack_kernel<<<repack_grid((long long)N * K), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t*>(w), static_cast<uint16_t*>(wk), N, K, gated, 0);
    return qf::cuda_status(cudaGetLastError(), "bf16_repack: launch");
}

extern "C" int qf_bf16_unpack(const void* wk, void* w, int N, int K, int gated, qf_stream_t stream) {
    QF_REQUIRE(w && wk, "bf16_unpack: null pointer argument");
    QF_REQUIRE(N >= 128 && N % 128 == 0 && K >= 32 && K % 32 == 0, "bf16_unpack: need N %% 128 == 0 and K %% 32 == 0");
    bf16_repack_kernel<<<repack_grid((long long)N * K), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t*>(wk), static_cast<uint16_t*>(w), N, K, gated, 1);
    return qf::cuda_status(cudaGetLastError(), "bf16_unpack: launch");
}
