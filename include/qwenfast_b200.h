/*
 * qwenfast_b200 -- C ABI of the sm_100a decode-path kernels (router top-k, W4A16 routed-expert MoE with shared
 * expert and combine, INT8 dense GEMMs).
 *
 * Conventions
 *   - Every pointer is a device pointer unless stated otherwise; nothing here allocates device memory or
 *     synchronises the stream. Work is enqueued on `stream` (a cudaStream_t).
 *   - bf16 tensors are passed as `void*` (IEEE bfloat16, row-major, contiguous unless a leading dimension is given).
 *   - Every entry point returns QF_OK (0) or a negative QF_ERR_* code; qf_last_error() then describes the failure
 *     (thread-local text). Argument checks happen on the host before anything is enqueued.
 *   - `pdl != 0` launches with programmatic stream serialization so the kernel can start while the previous kernel
 *     in the stream drains; every kernel waits (griddepcontrol.wait) before it touches data that kernel produced.
 *   - Kernels that wait on other CTAs bound each wait; a wait that runs out records a code in the kernel's control
 *     block instead of hanging (see QF_MOE_CTRL_ERR).
 */
#ifndef QWENFAST_B200_H
#define QWENFAST_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* qf_stream_t; /* identical to cudaStream_t */

enum {
    QF_OK = 0,
    QF_ERR_INVALID_ARGUMENT = -1, /* shape, dtype, alignment or size check failed */
    QF_ERR_CUDA = -2,             /* a CUDA runtime call failed */
    QF_ERR_UNSUPPORTED = -3       /* valid request this build does not implement */
};

/* Limits of this build. */
#define QF_MAX_TOKENS 64   /* decode/verify rows per call (M) */
#define QF_MAX_TOPK 16
#define QF_MAX_EXPERTS 1024

/* MoE control block: int32[QF_MOE_CTRL_WORDS], zeroed once by the caller, re-armed by the kernel itself.
 * Word QF_MOE_CTRL_ERR is sticky: non-zero after a launch means a bounded wait ran out or a routed expert id was out
 * of range (QF_MOE_ERR_* bits). After a TIMEOUT or PIPELINE error the caller must zero the control block (except
 * the mirror words below) AND the pbuf workspace again before the next launch: pbuf holds counters that an
 * interrupted launch leaves behind. BAD_EXPERT leaves the workspace consistent.
 * Words QF_MOE_CTRL_MIRROR, +1: optional 64-bit device-visible address (low word first) of a uint32 in mapped pinned
 * host memory; when it is non-zero, every launch that ends with a non-zero (sticky, so accumulated) error word stores
 * the word there, so a host can poll for kernel errors without synchronising. The kernel's re-arm keeps these two
 * words. */
#define QF_MOE_CTRL_WORDS 2048
#define QF_MOE_CTRL_ERR 3
#define QF_MOE_CTRL_MIRROR 2046
/* Size of the optional MoE timeline buffer (int64 entries). */
#define QF_MOE_DBG_NUMEL (32 * 512)
#define QF_MOE_ERR_TIMEOUT 0x1
#define QF_MOE_ERR_BAD_EXPERT 0x2
#define QF_MOE_ERR_PIPELINE 0x4

const char* qf_last_error(void);
int qf_version(void);

/* ------------------------------------------------------------------------------------------------------------
 * Router: logits = bf16(x . w^T) (fp32 accumulation), fp32 softmax over the logits, top-k by logit value with the
 * lower expert id winning ties (NaN ranks as -1e30, -0 equals +0), weights renormalised over the selection when
 * `renormalize` (unless their sum is not positive).
 * Replaces `router_topk` (serve/qwenfast/qf_router.cu:164-193, binding serve/qwenfast/qf_bind.cpp:14-15,121-123).
 *   x bf16 [rows, hidden]; w bf16 [experts, hidden]; outputs topk_weights fp32 [rows, topk],
 *   topk_ids int32 [rows, topk], logits bf16 [rows, experts];
 *   scratch fp32 >= rows*experts; counter int32[1] zeroed once (re-armed by the kernel).
 * rows 1..QF_MAX_TOKENS, hidden % 256 == 0 (<= 4096), experts % 16 == 0 (<= QF_MAX_EXPERTS), topk 1..16.
 * ------------------------------------------------------------------------------------------------------------ */
int qf_router_topk(const void* x, const void* w, int rows, int hidden, int experts, int topk, int renormalize,
                   float* topk_weights, int32_t* topk_ids, void* logits, float* scratch, int64_t scratch_numel,
                   int32_t* counter, int pdl, qf_stream_t stream);

/* Same router, for callers that cannot allocate device memory (no counterpart in the reference). Hosts such as an
 * inference engine's plugin enqueue, whose device memory is fixed at start-up, or a launcher running during CUDA-graph
 * capture cannot hand over scratch tensors: this variant keeps the fp32 logit scratch and the ticket counter in a
 * static device array of the library (rows * experts <= 64 * 1024, i.e. 256 KB per GPU, held until exit) and calls no
 * allocator. The first call in a CUDA context (the device's primary context, or one the host made current) resolves
 * that array's address in that context -- make it before any stream capture; a later call in another context (after
 * cudaDeviceReset, say) resolves it again. Each call checks its arguments before enqueueing anything, then clears the
 * counter on `stream`; calls that may overlap on the GPU share the array and race. */
int qf_router_topk_noalloc(const void* x, const void* w, int rows, int hidden, int experts, int topk, int renormalize,
                           float* topk_weights, int32_t* topk_ids, void* logits, int pdl, qf_stream_t stream);

/* ------------------------------------------------------------------------------------------------------------
 * Routed experts (W4A16) + shared expert + combine, one persistent launch.
 * Replaces `a16_moe_decode` (serve/qwenfast/qf_a16moe.cu:852-922, binding serve/qwenfast/qf_bind.cpp:90-97,142);
 * same argument roles, with the synthetic configurations' int4 format instead of NVFP4:
 *   x bf16 [M, H]; topk_ids int32 [M, topk]; topk_w fp32 [M, topk];
 *   w13 / s13: gate_up experts, int4 (code - 8) and bf16 group-128 scales in the kernel layout made by
 *              qf_w4_repack(gated = 1) from [E, 2I, H/8] int32 / [E, 2I, H/128] bf16;
 *   w2 / s2:   down experts in the kernel layout made by qf_w4_repack(gated = 0) from [E, H, I/8] / [E, H, I/128];
 *   gs13, gs2: bf16 [E] per-expert global scales or NULL (= 1);
 *   w_gate:    bf16 [H] shared-expert gate vector (required when a shared term is present);
 *   shared:    bf16 [M, H] precomputed shared-expert output, or NULL;
 *   sh_w13, sh_w2: bf16 shared expert weights (gate_up [2*Is, H] and down [H, Is]) in the kernel layout made by
 *              qf_bf16_repack (gated = 1 / 0), or NULL; Is = their intermediate size (0 when absent);
 *   scratch (caller-owned, sizes from qf_a16_moe_workspace): hbuf, ybuf, gl, ctrl (zeroed once), pbuf (required;
 *              zeroed once: it holds counters the kernel re-arms), shbuf; scratch sized for some M serves every
 *              smaller M of the same layer shape (the re-armed counters sit at places that do not depend on M);
 *   out bf16 [M, H].
 * out[t] = bf16(sigmoid(x[t].w_gate) * shared[t] + bf16(sum over top-k positions, in order, of
 *          bf16(bf16(expert_out) * bf16(gs2 * bf16(topk_w)))))  -- the reference's rounding points.
 * phase: 3 or 4: the whole layer in one launch. 1 and 2: the reference's split phases (qf_a16moe.cu:889, 915) as
 *   two launches of the same kernel over one workspace -- 1 computes the gate logits into gl and every routed
 *   slot's bf16(SwiGLU(gate_up)) into hbuf, 2 the down projections, the weighting and the combine (with `shared`)
 *   into out from hbuf and gl; phase 1 then phase 2 give the same bits as phase 4. Not with sh_w13 / sh_w2 (as in
 *   the reference, in-kernel shared-expert weights need the whole layer), mode 0 only.
 * mode 0: full layer. mode 1: expert-parallel shard -- only experts in [expert_lo, expert_hi) are computed; their
 *   weighted slot outputs go to ybuf [M, topk + 1, H] with every other slot zero, slot `topk` holding the shared
 *   expert output when this shard computes it; qf_moe_combine then finishes the layer (after the caller has summed
 *   ybuf over the shards). mode 2: diagnostic of the failure path -- the full layer, except that one producer first
 *   waits for a control word that nothing increments: the bounded wait runs out (about one second), the launch
 *   drains and leaves QF_MOE_ERR_TIMEOUT in ctrl[QF_MOE_CTRL_ERR] (its outputs are then undefined).
 * dbg: optional int64 [QF_MOE_DBG_NUMEL] timeline, or NULL: 32 entries per CTA (CTAs beyond the first
 *   QF_MOE_DBG_NUMEL / 32 record nothing), each (globaltimer ns << 12) | tag as a 64-bit pattern; entry 31 is the
 *   CTA's entry (tag 0xFFF), entries 0..30 in order of recording: tag bits 0-4 the event (1..7 an item of that kind
 *   starts -- GL, S1, G1, S1F, S2, G2, CB --, 16 + kind its stages are done, 30 the pipeline's consumers start, 31
 *   they stop), bits 5-6 the pipeline.
 * ------------------------------------------------------------------------------------------------------------ */
int qf_a16_moe_workspace(int M, int H, int I, int topk, int Is, int64_t* hbuf_bytes, int64_t* ybuf_bytes,
                         int64_t* gl_numel, int64_t* ctrl_numel, int64_t* pbuf_numel, int64_t* shbuf_bytes);

int qf_a16_moe_decode(const void* x, const int32_t* topk_ids, const float* topk_w, const int32_t* w13,
                      const void* s13, const void* gs13, const int32_t* w2, const void* s2, const void* gs2,
                      const void* w_gate, const void* shared, const void* sh_w13, const void* sh_w2, void* hbuf,
                      int64_t hbuf_bytes, void* ybuf, int64_t ybuf_bytes, float* gl, int64_t gl_numel, int32_t* ctrl,
                      int64_t ctrl_numel, float* pbuf, int64_t pbuf_numel, void* shbuf, int64_t shbuf_bytes,
                      void* out, int M, int H, int I, int E, int topk, int Is, int phase, int mode, int expert_lo,
                      int expert_hi, int64_t* dbg, int pdl, qf_stream_t stream);

/* The same layer on NVFP4 experts -- the reference's own expert format (qf_a16moe.cu:43-57 dequantisation,
 * serve/qwenfast/test_a16moe.py:134-137): e2m1 codes with one E4M3 scale per 16 k and a per-expert global value.
 *   w13 / w2: the codes (canonical uint8 [E, N, K/2], even k in the low nibble, read as int32 [E, N, K/8]) in the
 *             int4 kernel layout (qf_w4_repack on those words, or qwenfast_b200.formats.repack_nvfp4);
 *   f13 / f2: the E4M3 scales (canonical [E, N, K/16]) in the scale layout of formats.repack_nvfp4: per 128-row tile
 *             and 128-k stage, [kernel row (128)][8 groups];
 *   gs13 / gs2: bf16 [E] per-expert multipliers (the reference's 1 / global scale), or NULL (= 1).
 * The group scales are folded into the dequantised bf16 weights (e2m1 x E4M3 is exact in bf16); the rounding
 * points, the shared expert, the combine and every other argument are those of qf_a16_moe_decode. H, I % 128 == 0. */
int qf_a16_moe_decode_nvfp4(const void* x, const int32_t* topk_ids, const float* topk_w, const int32_t* w13,
                            const void* f13, const void* gs13, const int32_t* w2, const void* f2, const void* gs2,
                            const void* w_gate, const void* shared, const void* sh_w13, const void* sh_w2, void* hbuf,
                            int64_t hbuf_bytes, void* ybuf, int64_t ybuf_bytes, float* gl, int64_t gl_numel,
                            int32_t* ctrl, int64_t ctrl_numel, float* pbuf, int64_t pbuf_numel, void* shbuf,
                            int64_t shbuf_bytes, void* out, int M, int H, int I, int E, int topk, int Is, int phase,
                            int mode, int expert_lo, int expert_hi, int64_t* dbg, int pdl, qf_stream_t stream);

/* One decode MoE layer-step with the router inside the same launch (no counterpart in the reference, whose `dual`
 * path -- serve/overlays/sglang/srt/qwenfast.py:1177-1201 -- calls router_topk and then a16_moe_decode; this entry
 * gives the caller the outputs of both): every CTA computes bf16 logits of E / SMs router rows, a grid barrier on
 * ctrl follows, then every CTA runs the router's softmax / top-k / renormalise (the routine of qf_router_topk) on
 * all rows and the layer continues as qf_a16_moe_decode (phase 4). router_w bf16 [E, H] (H % 256 == 0, <= 4096,
 * 16-byte aligned); outputs topk_w fp32 [M, topk], topk_ids int32 [M, topk], logits bf16 [M, E]. The logits are
 * fp32 dot products in this kernel's own order, rounded to bf16 (within one bf16 ulp of qf_router_topk's); ids and
 * weights follow from them exactly as in qf_router_topk. Other arguments as qf_a16_moe_decode; ctrl also holds the
 * barrier's counter (re-armed by the kernel). All CTAs of the launch (one per SM) must be resident at once for the grid
 * barriers: the launch is cooperative, so the runtime co-schedules the grid or refuses it -- this entry then returns
 * QF_ERR_UNSUPPORTED and the caller takes the two-launch path (qf_router_topk, then qf_a16_moe_decode). The
 * barrier's wait is still bounded (~1 s), after which the sticky error word is set and the items stop.
 * x_stage: NULL (x is device memory), or a device buffer bf16 [M, H], 16-byte aligned: then x is pinned host memory
 *   (page-locked, mapped into the device's address space, as cudaHostAlloc gives under unified addressing) that the
 *   kernel itself copies into x_stage (each CTA a slice, then a second grid barrier) instead of a copy-engine transfer;
 *   out may likewise be pinned host memory (the combine writes it directly). */
int qf_moe_layer_decode(const void* x, void* x_stage, const void* router_w, int renormalize, float* topk_w, int32_t* topk_ids,
                        void* logits, const int32_t* w13, const void* s13, const void* gs13, const int32_t* w2,
                        const void* s2, const void* gs2, const void* w_gate, const void* shared, const void* sh_w13,
                        const void* sh_w2, void* hbuf, int64_t hbuf_bytes, void* ybuf, int64_t ybuf_bytes, float* gl,
                        int64_t gl_numel, int32_t* ctrl, int64_t ctrl_numel, float* pbuf, int64_t pbuf_numel,
                        void* shbuf, int64_t shbuf_bytes, void* out, int M, int H, int I, int E, int topk, int Is,
                        int mode, int expert_lo, int expert_hi, int64_t* dbg, int pdl, qf_stream_t stream);

/* qf_moe_layer_decode on NVFP4 experts: the router inside the launch, then the layer of qf_a16_moe_decode_nvfp4
 * (f13 / f2 the E4M3 group-16 scales in the kernel layout, gs13 / gs2 the per-expert multipliers); every other
 * argument as qf_moe_layer_decode. */
int qf_moe_layer_decode_nvfp4(const void* x, void* x_stage, const void* router_w, int renormalize, float* topk_w,
                              int32_t* topk_ids, void* logits, const int32_t* w13, const void* f13, const void* gs13,
                              const int32_t* w2, const void* f2, const void* gs2, const void* w_gate,
                              const void* shared, const void* sh_w13, const void* sh_w2, void* hbuf,
                              int64_t hbuf_bytes, void* ybuf, int64_t ybuf_bytes, float* gl, int64_t gl_numel,
                              int32_t* ctrl, int64_t ctrl_numel, float* pbuf, int64_t pbuf_numel, void* shbuf,
                              int64_t shbuf_bytes, void* out, int M, int H, int I, int E, int topk, int Is, int mode,
                              int expert_lo, int expert_hi, int64_t* dbg, int pdl, qf_stream_t stream);

/* Expert-parallel finish: out = the mode-0 combine of a ybuf [M, topk + 1, H] summed over the shards.
 * gl fp32 [M] is recomputed from x and w_gate when w_gate is given (has_shared != 0). */
int qf_moe_combine(const void* ybuf, const void* x, const void* w_gate, int has_shared, void* out, int M, int H,
                   int topk, int pdl, qf_stream_t stream);

/* Offline weight preparation (load time). Canonical int4 experts -> kernel layout, and back (exact).
 *   qweight int32 [E, N, K/8] (eight codes per word, lowest k in the low nibble), scales bf16 [E, N, K/128]
 *   -> wk int32 [E, N*K/8], sk bf16 [E, N*K/128]. gated = 1 for gate_up (N = 2I rows: gate then up), else 0.
 *   N % 128 == 0 and K % 128 == 0. */
int qf_w4_repack(const int32_t* qweight, const void* scales, int32_t* wk, void* sk, int E, int N, int K, int gated,
                 qf_stream_t stream);
int qf_w4_unpack(const int32_t* wk, const void* sk, int32_t* qweight, void* scales, int E, int N, int K, int gated,
                 qf_stream_t stream);
/* bf16 [N, K] -> kernel layout [N*K] (and back). N % 128 == 0, K % 64 == 0. */
int qf_bf16_repack(const void* w, void* wk, int N, int K, int gated, qf_stream_t stream);
int qf_bf16_unpack(const void* wk, void* w, int N, int K, int gated, qf_stream_t stream);

/* ------------------------------------------------------------------------------------------------------------
 * W8A16 group-scaled INT8 GEMM: y[M, N] = x[M, K] @ (q * s)^T, fp32 accumulation, bf16 out (tcgen05 tensor cores).
 * Replaces `w8g_gemm` (serve/qwenfast/qf_w8g.cu:303-336, binding serve/qwenfast/qf_bind.cpp:42,133);
 *   x bf16 [M, K] row stride ldx (ldx % 8 == 0, 16-byte aligned); q int8 [N, K] canonical row-major (16-byte
 *   aligned); s bf16 [N, K/group]; y bf16 [M, N] row stride ldy. M 1..QF_MAX_TOKENS, N >= 8 and N % 8 == 0 (a last
 *   tile of 128 rows past N computes zeros there), K % 64 == 0, group 128 or 64. Every product is exact (int8 weights and tokens scaled by a power of two as fp16) and the sums
 *   are fp32; the result does not depend on timing.
 *   fix: caller-owned float buffer of qf_w8g_fixup_elems(N) elements, zero-filled before its first use; every call
 *   leaves its counters zero again (after a non-zero qf_w8g_take_status, zero it again). Calls that may run
 *   concurrently need their own. The launch is cooperative (every CTA resident), with programmatic dependent launch
 *   when pdl != 0.
 *   rpw: the reference's path bits (qf_w8g.cu:315-318). 0x100 forces the tensor-memory (tcgen05) kernel, 0x200
 *   forbids it: the register-fragment kernel runs, or the call fails with QF_ERR_UNSUPPORTED when that kernel does
 *   not take the shape (M <= 16, K % 128 == 0 and a one-wave split); both bits together are invalid. Without them
 *   the register-fragment kernel takes the decode shapes it supports and the tensor-memory kernel the rest. The low
 *   byte (the reference's rows per warp of its CUDA-core kernel) has no counterpart and is ignored.
 * ------------------------------------------------------------------------------------------------------------ */
int qf_w8g_gemm(const void* x, int64_t ldx, const int8_t* q, const void* s, void* y, int64_t ldy, int M, int N,
                int K, int group, int rpw, float* fix, int64_t fix_elems, int pdl, qf_stream_t stream);
/* Elements (float) of the W8A16 fixup buffer for an N-row weight on the current device. */
int qf_w8g_fixup_elems(int N, int64_t* elems);
/* Sticky device status of the W8A16 kernel since the last call (synchronises the device, then clears it): 0 = every
 * bounded wait completed; bit 0 = a weight-ring wait ran out, bit 1 = a unit (operand / accumulator) wait, bit 2 =
 * the final tensor-core wait, bit 3 = the wait for the other runs of a split tile (the outputs are then undefined). */
int qf_w8g_take_status(uint32_t* status);
/* w bf16 [rows, K] = bf16(q * s). Replaces `w8g_unpack` (serve/qwenfast/qf_w8g.cu:338-351). */
int qf_w8g_unpack(const int8_t* q, const void* s, void* w, int64_t rows, int K, int group, qf_stream_t stream);

/* ------------------------------------------------------------------------------------------------------------
 * W8A8 INT8 GEMM (no counterpart kernel in the reference; the dense projections of the synthetic config 3):
 *   sx[t] = absmax(x[t]) / 127 (1 for an all-zero row); xq = rint(x / sx) clamped to [-127, 127];
 *   acc = sum_k xq * q (exact int32 on tcgen05 tensor cores); y = bf16((float(acc) * sx[t]) * sw[n]).
 *   x bf16 [M, K] (row stride ldx); q int8: the weight [N, K] in the kernel layout of qf_w8_repack; sw fp32 [N];
 *   y bf16 [M, N] (row stride ldy). Scratch, written: xq int8 [16 * K] = the quantised activations packed as the
 *   tensor-core operand (element (t, k) at (k / 16) * 256 + t * 16 + k % 16; rows t >= M zero), sx fp32 [M].
 *   acc: int32 split-K fixup buffer of qf_w8a8_fixup_elems(N) elements; zero-filled before its first use, every
 *   call leaves it zero-filled again (after a non-zero qf_w8a8_take_status, zero it again). One buffer per
 *   stream: calls that may run concurrently need their own. acc_out: optional int32 [M, N] copy of the exact
 *   accumulators (NULL to skip). M 1..16, N % 128 == 0, K % 128 == 0 (<= 16384).
 *   q is load-time data: the kernel requests weight tiles before griddepcontrol.wait, so q must not be written
 *   by the kernel directly before it in the stream (synchronise after qf_w8_repack). Two launches: the
 *   quantisation kernel, then the GEMM under programmatic dependent launch.
 * ------------------------------------------------------------------------------------------------------------ */
int qf_w8a8_gemm(const void* x, int64_t ldx, const int8_t* q, const float* sw, void* y, int64_t ldy, int M, int N,
                 int K, int8_t* xq, float* sx, int32_t* acc, int32_t* acc_out, int pdl, qf_stream_t stream);
/* W8A8 weight layout (load time): canonical q int8 [N, K] row-major -> qk, contiguous 16 KB tiles
 * [N/128][K/128][128 rows][128 bytes] with each row's 16-byte k chunk c stored at position c ^ (row % 8) (the
 * K-major 128-byte-swizzle operand layout of the tensor cores). qf_w8_unpack is the exact inverse.
 * (No counterpart in the reference.) N % 128 == 0, K % 128 == 0. */
/* Sticky device status of the W8A8 kernel since the last call (synchronises the device, then clears it):
 * 0 = every bounded wait completed; bit 0 = a weight-ring wait ran out, bit 1 = a segment
 * (accumulator) wait ran out, bit 2 = the final tensor-core wait ran out, bit 3 = the wait for the other runs of a
 * split weight tile ran out (the affected outputs and the fixup buffer are undefined). */
int qf_w8a8_take_status(uint32_t* status);
/* Elements (int32) of the W8A8 split-K fixup buffer for an N-row weight. */
int qf_w8a8_fixup_elems(int N, int64_t* elems);
int qf_w8_repack(const int8_t* q, int8_t* qk, int N, int K, qf_stream_t stream);
int qf_w8_unpack(const int8_t* qk, int8_t* q, int N, int K, qf_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* QWENFAST_B200_H */
