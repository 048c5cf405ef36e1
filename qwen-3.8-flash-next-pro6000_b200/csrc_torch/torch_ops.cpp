// torch.ops.qwenfast_b200.*: the decode-path kernels registered as torch custom operators (TORCH_LIBRARY), over the
// C ABI of libqwenfast_b200.so (include/qwenfast_b200.h). Names and argument roles follow the reference extension's
// binding (serve/qwenfast/qf_bind.cpp:14-15 router_topk, :42-43 w8g_gemm / w8g_unpack, :90-97 a16_moe_decode); the
// reference registers them with pybind11, here they are dispatcher operators with CUDA and Meta kernels, so that
// torch.compile / dynamo can trace through them (the Meta kernels give the output shapes without running anything).
// Every CUDA kernel launches on the current stream of the tensors' device; bad arguments raise c10::Error (the
// reference's TORCH_CHECK), the library's own checks raise with its message. No CPU path.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <map>
#include <mutex>
#include <tuple>

#include "qwenfast_b200.h"

namespace {

using at::Tensor;

void check_status(int status, const char* what) {
    TORCH_CHECK(status == QF_OK, what, ": ", qf_last_error());
}

qf_stream_t stream_of(const Tensor& t) {
    return reinterpret_cast<qf_stream_t>(at::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

const void* ptr_or_null(const Tensor& t) { return t.defined() && t.numel() > 0 ? t.data_ptr() : nullptr; }
void* mut_ptr_or_null(const Tensor& t) { return t.defined() && t.numel() > 0 ? t.data_ptr() : nullptr; }
bool present(const Tensor& t) { return t.defined() && t.numel() > 0; }

// zero-filled scratch kept per (device, stream, tag, size) -- the split-K fixup buffers whose counters the kernels
// leave at zero after every call; created on first use (make that first call before any CUDA-graph capture)
Tensor zero_kept(const Tensor& like, int64_t tag, int64_t n, at::ScalarType dt) {
    static std::mutex mu;
    static std::map<std::tuple<int, void*, int64_t, int64_t>, Tensor> cache;
    const int dev = like.device().index();
    void* st = at::cuda::getCurrentCUDAStream(dev).stream();
    std::lock_guard<std::mutex> lock(mu);
    auto key = std::make_tuple(dev, st, tag, n);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    Tensor t = at::zeros({n}, like.options().dtype(dt));
    cache.emplace(key, t);
    return t;
}

// ------------------------------------------------------------------------------------------------------ router
std::tuple<Tensor, Tensor, Tensor> router_topk_cuda(const Tensor& x, const Tensor& w, int64_t topk, bool renormalize,
                                                    Tensor scratch, Tensor counter, bool pdl) {
    TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.is_contiguous(),
                "router_topk: x must be contiguous bf16 [rows, H] on CUDA");
    TORCH_CHECK(w.scalar_type() == at::kBFloat16 && w.dim() == 2 && w.size(1) == x.size(1) && w.is_contiguous() &&
                    w.device() == x.device(),
                "router_topk: w must be contiguous bf16 [E, H] on x's device");
    TORCH_CHECK(scratch.scalar_type() == at::kFloat && scratch.device() == x.device(), "router_topk: scratch fp32");
    TORCH_CHECK(counter.scalar_type() == at::kInt && counter.numel() >= 1 && counter.device() == x.device(),
                "router_topk: counter int32 [>=1]");
    const c10::cuda::CUDAGuard guard(x.device());
    const int64_t rows = x.size(0), H = x.size(1), E = w.size(0);
    Tensor weights = at::empty({rows, topk}, x.options().dtype(at::kFloat));
    Tensor ids = at::empty({rows, topk}, x.options().dtype(at::kInt));
    Tensor logits = at::empty({rows, E}, x.options());
    check_status(qf_router_topk(x.data_ptr(), w.data_ptr(), (int)rows, (int)H, (int)E, (int)topk, renormalize ? 1 : 0,
                                weights.data_ptr<float>(), ids.data_ptr<int32_t>(), logits.data_ptr(),
                                scratch.data_ptr<float>(), scratch.numel(), counter.data_ptr<int32_t>(), pdl ? 1 : 0,
                                stream_of(x)),
                 "router_topk");
    return {weights, ids, logits};
}

std::tuple<Tensor, Tensor, Tensor> router_topk_meta(const Tensor& x, const Tensor& w, int64_t topk, bool, Tensor,
                                                    Tensor, bool) {
    return {at::empty({x.size(0), topk}, x.options().dtype(at::kFloat)),
            at::empty({x.size(0), topk}, x.options().dtype(at::kInt)), at::empty({x.size(0), w.size(0)}, x.options())};
}

// ------------------------------------------------------------------------------------------------------ MoE
// Routed experts (kernel-layout int4 weights) + shared expert + combine; `out` is written in place (the reference's
// pybind function returns that same tensor; a schema without an aliased return lets torch.compile functionalize the
// call). Empty tensors mean "absent", as in the reference. The shared expert is given as bf16 kernel-layout weights
// (shq1 / shq2, shs1 / shs2 empty) or as a precomputed `shared`; the reference's INT8 shared weights go through
// qwenfast_b200.ops.shared_w8_as_bf16 once (the Python op does that conversion and caches it).
void a16_moe_decode_fmt(int fmt, const Tensor& x, const Tensor& topk_ids, const Tensor& topk_w, const Tensor& w13,
                        const Tensor& s13, const Tensor& gs13, const Tensor& w2, const Tensor& s2, const Tensor& gs2,
                        const Tensor& w_gate, const Tensor& shared, Tensor hbuf, Tensor ybuf, Tensor gl,
                        Tensor counters, Tensor out, int64_t phase, Tensor dbg, Tensor pbuf, const Tensor& shq1,
                        const Tensor& shs1, const Tensor& shq2, const Tensor& shs2, Tensor shbuf) {
    TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.is_contiguous(),
                "a16_moe_decode: x must be contiguous bf16 [M, H] on CUDA");
    TORCH_CHECK(topk_ids.scalar_type() == at::kInt && topk_ids.dim() == 2 && topk_ids.size(0) == x.size(0) &&
                    topk_ids.is_contiguous(),
                "a16_moe_decode: topk_ids must be contiguous int32 [M, topk]");
    TORCH_CHECK(topk_w.scalar_type() == at::kFloat && topk_w.sizes() == topk_ids.sizes() && topk_w.is_contiguous(),
                "a16_moe_decode: topk_w must be contiguous fp32 [M, topk]");
    TORCH_CHECK(w13.scalar_type() == at::kInt && w2.scalar_type() == at::kInt && w13.dim() == 2 && w2.dim() == 2,
                "a16_moe_decode: w13 / w2 must be int32 kernel-layout [E, *] tensors");
    TORCH_CHECK(fmt == 0 ? s13.scalar_type() == at::kBFloat16 && s2.scalar_type() == at::kBFloat16
                         : s13.scalar_type() == at::kByte && s2.scalar_type() == at::kByte,
                "a16_moe_decode: s13 / s2 must be bf16 group-128 scales (int4 experts) or uint8 E4M3 group-16 scales "
                "(NVFP4 experts) in the kernel layout");
    TORCH_CHECK(!present(shs1) && !present(shs2),
                "a16_moe_decode: INT8 shared-expert weights need a one-time conversion "
                "(qwenfast_b200.ops.shared_w8_as_bf16); pass the bf16 kernel-layout weights as shq1 / shq2");
    TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.sizes() == x.sizes() && out.is_contiguous(),
                "a16_moe_decode: out must be bf16 [M, H]");
    const c10::cuda::CUDAGuard guard(x.device());
    const int64_t M = x.size(0), H = x.size(1), E = w13.size(0), topk = topk_ids.size(1);
    const int64_t I = (w2.size(1) * 8) / H;
    const bool has_shw = present(shq1);
    const int64_t Is = has_shw ? shq2.numel() / H : 0;
    auto entry = fmt == 0 ? &qf_a16_moe_decode : &qf_a16_moe_decode_nvfp4;
    check_status(entry(x.data_ptr(), topk_ids.data_ptr<int32_t>(), topk_w.data_ptr<float>(),
                                   w13.data_ptr<int32_t>(), s13.data_ptr(), ptr_or_null(gs13), w2.data_ptr<int32_t>(),
                                   s2.data_ptr(), ptr_or_null(gs2), ptr_or_null(w_gate), ptr_or_null(shared),
                                   has_shw ? shq1.data_ptr() : nullptr, has_shw ? shq2.data_ptr() : nullptr,
                                   hbuf.data_ptr(), hbuf.numel() * hbuf.element_size(), ybuf.data_ptr(),
                                   ybuf.numel() * ybuf.element_size(), gl.data_ptr<float>(), gl.numel(),
                                   counters.data_ptr<int32_t>(), counters.numel(),
                                   static_cast<float*>(mut_ptr_or_null(pbuf)), present(pbuf) ? pbuf.numel() : 0,
                                   mut_ptr_or_null(shbuf), present(shbuf) ? shbuf.numel() * shbuf.element_size() : 0,
                                   out.data_ptr(), (int)M, (int)H, (int)I, (int)E, (int)topk, (int)Is, (int)phase, 0, 0,
                                   (int)E, static_cast<int64_t*>(mut_ptr_or_null(dbg)), 1, stream_of(x)),
                 fmt == 0 ? "a16_moe_decode" : "a16_moe_decode_nvfp4");
}

#define QF_A16_ARGS                                                                                                  \
    const Tensor &x, const Tensor &topk_ids, const Tensor &topk_w, const Tensor &w13, const Tensor &s13,             \
        const Tensor &gs13, const Tensor &w2, const Tensor &s2, const Tensor &gs2, const Tensor &w_gate,             \
        const Tensor &shared, Tensor hbuf, Tensor ybuf, Tensor gl, Tensor counters, Tensor out, int64_t phase,        \
        Tensor dbg, Tensor pbuf, const Tensor &shq1, const Tensor &shs1, const Tensor &shq2, const Tensor &shs2,     \
        Tensor shbuf
#define QF_A16_PASS \
    x, topk_ids, topk_w, w13, s13, gs13, w2, s2, gs2, w_gate, shared, hbuf, ybuf, gl, counters, out, phase, dbg, pbuf, \
        shq1, shs1, shq2, shs2, shbuf
void a16_moe_decode_cuda(QF_A16_ARGS) { a16_moe_decode_fmt(0, QF_A16_PASS); }
void a16_moe_decode_nvfp4_cuda(QF_A16_ARGS) { a16_moe_decode_fmt(1, QF_A16_PASS); }

void a16_moe_decode_meta(const Tensor&, const Tensor&, const Tensor&, const Tensor&, const Tensor&, const Tensor&,
                         const Tensor&, const Tensor&, const Tensor&, const Tensor&, const Tensor&, Tensor, Tensor, Tensor,
                         Tensor, Tensor, int64_t, Tensor, Tensor, const Tensor&, const Tensor&, const Tensor&,
                         const Tensor&, Tensor) {}

// The layer-step with the router inside the launch (qf_moe_layer_decode): writes out, returns the routing.
std::tuple<Tensor, Tensor, Tensor> moe_layer_decode_cuda(const Tensor& x, const Tensor& router_w, bool renormalize,
                                                         const Tensor& w13, const Tensor& s13, const Tensor& gs13,
                                                         const Tensor& w2, const Tensor& s2, const Tensor& gs2,
                                                         const Tensor& w_gate, const Tensor& shared,
                                                         const Tensor& sh_w13, const Tensor& sh_w2, int64_t topk,
                                                         Tensor hbuf, Tensor ybuf, Tensor gl, Tensor ctrl, Tensor pbuf,
                                                         Tensor shbuf, Tensor out) {
    TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.is_contiguous(),
                "moe_layer_decode: x must be contiguous bf16 [M, H] on CUDA");
    TORCH_CHECK(router_w.scalar_type() == at::kBFloat16 && router_w.dim() == 2 && router_w.size(1) == x.size(1),
                "moe_layer_decode: router_w must be bf16 [E, H]");
    TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.sizes() == x.sizes() && out.is_contiguous(),
                "moe_layer_decode: out must be bf16 [M, H]");
    const c10::cuda::CUDAGuard guard(x.device());
    const int64_t M = x.size(0), H = x.size(1), E = router_w.size(0);
    const int64_t I = (w2.size(1) * 8) / H;
    const bool has_shw = present(sh_w13);
    const int64_t Is = has_shw ? sh_w2.numel() / H : 0;
    Tensor tw = at::empty({M, topk}, x.options().dtype(at::kFloat));
    Tensor ids = at::empty({M, topk}, x.options().dtype(at::kInt));
    Tensor logits = at::empty({M, E}, x.options());
    check_status(qf_moe_layer_decode(x.data_ptr(), nullptr, router_w.data_ptr(), renormalize ? 1 : 0,
                                     tw.data_ptr<float>(), ids.data_ptr<int32_t>(), logits.data_ptr(),
                                     w13.data_ptr<int32_t>(), s13.data_ptr(), ptr_or_null(gs13), w2.data_ptr<int32_t>(),
                                     s2.data_ptr(), ptr_or_null(gs2), ptr_or_null(w_gate), ptr_or_null(shared),
                                     has_shw ? sh_w13.data_ptr() : nullptr, has_shw ? sh_w2.data_ptr() : nullptr,
                                     hbuf.data_ptr(), hbuf.numel() * hbuf.element_size(), ybuf.data_ptr(),
                                     ybuf.numel() * ybuf.element_size(), gl.data_ptr<float>(), gl.numel(),
                                     ctrl.data_ptr<int32_t>(), ctrl.numel(), pbuf.data_ptr<float>(), pbuf.numel(),
                                     mut_ptr_or_null(shbuf), present(shbuf) ? shbuf.numel() * shbuf.element_size() : 0,
                                     out.data_ptr(), (int)M, (int)H, (int)I, (int)E, (int)topk, (int)Is, 0, 0, (int)E,
                                     nullptr, 1, stream_of(x)),
                 "moe_layer_decode");
    return {tw, ids, logits};
}

std::tuple<Tensor, Tensor, Tensor> moe_layer_decode_meta(const Tensor& x, const Tensor& router_w, bool, const Tensor&,
                                                         const Tensor&, const Tensor&, const Tensor&, const Tensor&,
                                                         const Tensor&, const Tensor&, const Tensor&, const Tensor&,
                                                         const Tensor&, int64_t topk, Tensor, Tensor, Tensor, Tensor,
                                                         Tensor, Tensor, Tensor) {
    return {at::empty({x.size(0), topk}, x.options().dtype(at::kFloat)),
            at::empty({x.size(0), topk}, x.options().dtype(at::kInt)),
            at::empty({x.size(0), router_w.size(0)}, x.options())};
}

// ------------------------------------------------------------------------------------------------------ INT8
Tensor w8g_gemm_cuda(const Tensor& x, const Tensor& q, const Tensor& s, int64_t rpw) {
    TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1,
                "w8g_gemm: x must be bf16 [M, K] with unit column stride on CUDA");
    TORCH_CHECK(q.scalar_type() == at::kChar && q.dim() == 2 && q.is_contiguous() && q.size(1) == x.size(1),
                "w8g_gemm: q must be contiguous int8 [N, K]");
    TORCH_CHECK(s.scalar_type() == at::kBFloat16 && s.dim() == 2 && s.size(0) == q.size(0) && s.is_contiguous() &&
                    q.size(1) % s.size(1) == 0,
                "w8g_gemm: s must be bf16 [N, K / group]");
    const c10::cuda::CUDAGuard guard(x.device());
    const int64_t M = x.size(0), K = x.size(1), N = q.size(0);
    int64_t fe = 0;
    check_status(qf_w8g_fixup_elems((int)N, &fe), "w8g_gemm");
    Tensor fix = zero_kept(x, 1, fe, at::kFloat);
    Tensor y = at::empty({M, N}, x.options());
    check_status(qf_w8g_gemm(x.data_ptr(), x.stride(0), q.data_ptr<int8_t>(), s.data_ptr(), y.data_ptr(), N, (int)M,
                             (int)N, (int)K, (int)(K / s.size(1)), (int)rpw, fix.data_ptr<float>(), fix.numel(), 0,
                             stream_of(x)),
                 "w8g_gemm");
    return y;
}

Tensor w8g_gemm_meta(const Tensor& x, const Tensor& q, const Tensor&, int64_t) {
    return at::empty({x.size(0), q.size(0)}, x.options());
}

void w8g_unpack_cuda(const Tensor& q, const Tensor& s, Tensor w) {
    TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kChar && q.dim() == 2 && q.is_contiguous(),
                "w8g_unpack: q must be contiguous int8 [rows, K] on CUDA");
    TORCH_CHECK(s.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && w.sizes() == q.sizes() &&
                    w.is_contiguous() && s.is_contiguous() && q.size(1) % s.size(1) == 0,
                "w8g_unpack: s bf16 [rows, K / group], w bf16 [rows, K]");
    const c10::cuda::CUDAGuard guard(q.device());
    check_status(qf_w8g_unpack(q.data_ptr<int8_t>(), s.data_ptr(), w.data_ptr(), q.size(0), (int)q.size(1),
                               (int)(q.size(1) / s.size(1)), stream_of(q)),
                 "w8g_unpack");
}

void w8g_unpack_meta(const Tensor&, const Tensor&, Tensor) {}

// W8A8 (no counterpart in the reference): q in the kernel layout of qf_w8_repack, sw fp32 [N]; y bf16 [M, N].
Tensor w8a8_gemm_cuda(const Tensor& x, const Tensor& q, const Tensor& sw) {
    TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1,
                "w8a8_gemm: x must be bf16 [M, K] with unit column stride on CUDA");
    TORCH_CHECK(q.scalar_type() == at::kChar && q.dim() == 2 && q.is_contiguous() && q.size(1) == x.size(1),
                "w8a8_gemm: q must be int8 [N, K] (kernel layout)");
    TORCH_CHECK(sw.scalar_type() == at::kFloat && sw.numel() == q.size(0), "w8a8_gemm: sw must be fp32 [N]");
    const c10::cuda::CUDAGuard guard(x.device());
    const int64_t M = x.size(0), K = x.size(1), N = q.size(0);
    int64_t fe = 0;
    check_status(qf_w8a8_fixup_elems((int)N, &fe), "w8a8_gemm");
    Tensor fix = zero_kept(x, 2, fe, at::kInt);
    Tensor xq = at::empty({16 * K}, x.options().dtype(at::kChar));
    Tensor sx = at::empty({M}, x.options().dtype(at::kFloat));
    Tensor y = at::empty({M, N}, x.options());
    check_status(qf_w8a8_gemm(x.data_ptr(), x.stride(0), q.data_ptr<int8_t>(), sw.data_ptr<float>(), y.data_ptr(), N,
                              (int)M, (int)N, (int)K, xq.data_ptr<int8_t>(), sx.data_ptr<float>(),
                              fix.data_ptr<int32_t>(), nullptr, 1, stream_of(x)),
                 "w8a8_gemm");
    return y;
}

Tensor w8a8_gemm_meta(const Tensor& x, const Tensor& q, const Tensor&) {
    return at::empty({x.size(0), q.size(0)}, x.options());
}

}  // namespace

TORCH_LIBRARY(qwenfast_b200, m) {
    m.def("router_topk(Tensor x, Tensor w, int topk, bool renormalize, Tensor(a!) scratch, Tensor(b!) counter, "
          "bool pdl=True) -> (Tensor, Tensor, Tensor)");
    m.def("a16_moe_decode(Tensor x, Tensor topk_ids, Tensor topk_w, Tensor w13, Tensor s13, Tensor gs13, Tensor w2, "
          "Tensor s2, Tensor gs2, Tensor w_gate, Tensor shared, Tensor(a!) hbuf, Tensor(b!) ybuf, Tensor(c!) gl, "
          "Tensor(d!) counters, Tensor(e!) out, int phase, Tensor(f!) dbg, Tensor(g!) pbuf, Tensor shq1, Tensor shs1, "
          "Tensor shq2, Tensor shs2, Tensor(h!) shbuf) -> ()");
    m.def("a16_moe_decode_nvfp4(Tensor x, Tensor topk_ids, Tensor topk_w, Tensor w13, Tensor s13, Tensor gs13, "
          "Tensor w2, Tensor s2, Tensor gs2, Tensor w_gate, Tensor shared, Tensor(a!) hbuf, Tensor(b!) ybuf, "
          "Tensor(c!) gl, Tensor(d!) counters, Tensor(e!) out, int phase, Tensor(f!) dbg, Tensor(g!) pbuf, Tensor shq1, "
          "Tensor shs1, Tensor shq2, Tensor shs2, Tensor(h!) shbuf) -> ()");
    m.def("moe_layer_decode(Tensor x, Tensor router_w, bool renormalize, Tensor w13, Tensor s13, Tensor gs13, "
          "Tensor w2, Tensor s2, Tensor gs2, Tensor w_gate, Tensor shared, Tensor sh_w13, Tensor sh_w2, int topk, "
          "Tensor(a!) hbuf, Tensor(b!) ybuf, Tensor(c!) gl, Tensor(d!) ctrl, Tensor(e!) pbuf, Tensor(f!) shbuf, "
          "Tensor(g!) out) -> (Tensor, Tensor, Tensor)");
    m.def("w8g_gemm(Tensor x, Tensor q, Tensor s, int rpw=0) -> Tensor");
    m.def("w8g_unpack(Tensor q, Tensor s, Tensor(a!) w) -> ()");
    m.def("w8a8_gemm(Tensor x, Tensor q, Tensor sw) -> Tensor");
}

TORCH_LIBRARY_IMPL(qwenfast_b200, CUDA, m) {
    m.impl("router_topk", &router_topk_cuda);
    m.impl("a16_moe_decode", &a16_moe_decode_cuda);
    m.impl("a16_moe_decode_nvfp4", &a16_moe_decode_nvfp4_cuda);
    m.impl("moe_layer_decode", &moe_layer_decode_cuda);
    m.impl("w8g_gemm", &w8g_gemm_cuda);
    m.impl("w8g_unpack", &w8g_unpack_cuda);
    m.impl("w8a8_gemm", &w8a8_gemm_cuda);
}

TORCH_LIBRARY_IMPL(qwenfast_b200, Meta, m) {
    m.impl("router_topk", &router_topk_meta);
    m.impl("a16_moe_decode", &a16_moe_decode_meta);
    m.impl("a16_moe_decode_nvfp4", &a16_moe_decode_meta);
    m.impl("moe_layer_decode", &moe_layer_decode_meta);
    m.impl("w8g_gemm", &w8g_gemm_meta);
    m.impl("w8g_unpack", &w8g_unpack_meta);
    m.impl("w8a8_gemm", &w8a8_gemm_meta);
}
