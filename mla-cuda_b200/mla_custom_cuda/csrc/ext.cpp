// mla_custom_cuda._C — the C++ torch extension of the drop-in module, built by
// mla-cuda_b200/setup.py like the reference's extension (setup.py:20-26). It
// binds the reference's two functions, q_absorbed and mla_attention
// (mla_kernels.cu:1688-1692), with the same positional signatures, return
// types and errors (TORCH_CHECK -> RuntimeError), plus their precision / causal
// variants, and runs them through the C ABI of libmla_b200.so
// (include/mla_b200.h). Outputs and workspaces come from torch's caching
// allocator on the inputs' device; all work goes on torch's current stream
// (mla_kernels.cu:664-667, :1528-1549).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <vector>

#include "mla_b200.h"

namespace {

mla_dtype_t dtype_code(const at::Tensor& t) {
    switch (t.scalar_type()) {
        case at::kFloat: return MLA_DTYPE_F32;
        case at::kDouble: return MLA_DTYPE_F64;
        case at::kHalf: return MLA_DTYPE_F16;
        case at::kBFloat16: return MLA_DTYPE_BF16;
        default: TORCH_CHECK(false, "mla_custom_cuda: unsupported dtype ", t.scalar_type());
    }
    return MLA_DTYPE_F32;
}

mla_precision_t precision_code(const std::string& p) {
    if (p == "exact") return MLA_PREC_EXACT;
    if (p == "tensor") return MLA_PREC_TENSOR;
    TORCH_CHECK(false, "mla_custom_cuda: precision must be 'exact' or 'tensor', got ", p);
    return MLA_PREC_EXACT;
}

void check_status(mla_status_t st, const char* what) {
    TORCH_CHECK(st == MLA_OK, what, ": ", mla_status_string(st), ": ", mla_last_error_message());
}

void check_operands(const std::vector<std::pair<const char*, const at::Tensor*>>& ts) {
    const at::Tensor& first = *ts.front().second;
    for (const auto& nt : ts) {
        const at::Tensor& t = *nt.second;
        TORCH_CHECK(t.is_cuda(), nt.first, " must be a CUDA tensor (there is no CPU path)");
        TORCH_CHECK(t.scalar_type() == first.scalar_type(), nt.first, " has dtype ", t.scalar_type(), ", expected ",
                    first.scalar_type());
        TORCH_CHECK(t.device() == first.device(), nt.first, " is on ", t.device(), ", expected ", first.device());
    }
}

std::vector<at::Tensor> ext_q_absorbed_ex(at::Tensor x, at::Tensor W_q_a, at::Tensor q_norm_w, at::Tensor W_q_b,
                                      at::Tensor W_uk, at::Tensor positions, int64_t nope_dim, int64_t rope_dim,
                                      double eps, const std::string& precision) {
    check_operands({{"x", &x}, {"W_q_a", &W_q_a}, {"q_norm_w", &q_norm_w}, {"W_q_b", &W_q_b}, {"W_uk", &W_uk}});
    TORCH_CHECK(x.dim() == 3, "x must be [B, Sq, hidden]");
    TORCH_CHECK(W_q_a.dim() == 2 && W_q_a.size(0) == x.size(2), "W_q_a must be [hidden, q_lora]");
    TORCH_CHECK(W_uk.dim() == 3 && W_uk.size(1) == nope_dim, "W_uk must be [H, nope_dim, kv_rank]");
    const int64_t B = x.size(0), Sq = x.size(1), hidden = x.size(2), q_lora = W_q_a.size(1);
    const int64_t H = W_uk.size(0), R = W_uk.size(2);
    TORCH_CHECK(W_q_b.dim() == 2 && W_q_b.size(0) == q_lora && W_q_b.size(1) == H * (nope_dim + rope_dim),
                "W_q_b must be [q_lora, H*(nope+rope)]");
    TORCH_CHECK(q_norm_w.dim() == 1 && q_norm_w.size(0) == q_lora, "q_norm_w must be a 1-D tensor of length q_lora");
    TORCH_CHECK(positions.dim() == 1 && positions.size(0) == Sq, "positions must be a 1-D tensor of length Sq");
    TORCH_CHECK(!positions.is_floating_point() && !positions.is_complex(), "positions must be an integer tensor");
    const c10::cuda::CUDAGuard guard(x.device());
    auto xc = x.contiguous(), Wa = W_q_a.contiguous(), g = q_norm_w.contiguous(), Wb = W_q_b.contiguous(),
         Wk = W_uk.contiguous();
    auto pos = positions.to(x.device(), at::kLong).contiguous();
    auto qa = at::empty({B, Sq, H, R}, x.options());
    auto qr = at::empty({B, Sq, H, rope_dim}, x.options());
    const mla_dtype_t dt = dtype_code(x);
    const mla_precision_t pc = precision_code(precision);
    size_t nbytes = 0;
    check_status(mla_q_absorbed_workspace_size(dt, pc, B, Sq, hidden, q_lora, H, nope_dim, rope_dim, R, &nbytes),
                 "q_absorbed");
    auto ws = at::empty({int64_t(nbytes > 0 ? nbytes : 1)}, x.options().dtype(at::kByte));
    check_status(mla_q_absorbed(dt, pc, xc.data_ptr(), Wa.data_ptr(), g.data_ptr(), Wb.data_ptr(), Wk.data_ptr(),
                                pos.data_ptr<int64_t>(), B, Sq, hidden, q_lora, H, nope_dim, rope_dim, R, eps,
                                qa.data_ptr(), qr.data_ptr(), ws.data_ptr(), size_t(ws.numel()),
                                at::cuda::getCurrentCUDAStream().stream()),
                 "q_absorbed");
    return {qa, qr};
}

at::Tensor ext_mla_attention_ex(at::Tensor q_absorbed, at::Tensor q_rope, at::Tensor c_kv, at::Tensor pe_cache,
                            at::Tensor W_uv, double scale, bool causal, const std::string& precision) {
    check_operands({{"q_absorbed", &q_absorbed}, {"q_rope", &q_rope}, {"c_kv", &c_kv}, {"pe_cache", &pe_cache},
                    {"W_uv", &W_uv}});
    TORCH_CHECK(q_absorbed.dim() == 4, "q_absorbed must be [B, Sq, H, kv_rank]");
    const int64_t B = q_absorbed.size(0), Sq = q_absorbed.size(1), H = q_absorbed.size(2), R = q_absorbed.size(3);
    TORCH_CHECK(q_rope.dim() == 4 && q_rope.size(0) == B && q_rope.size(1) == Sq && q_rope.size(2) == H,
                "q_rope must be [B, Sq, H, rope]");
    const int64_t D = q_rope.size(3);
    TORCH_CHECK(c_kv.dim() == 3 && c_kv.size(0) == B && c_kv.size(2) == R, "c_kv must be [B, Sk, kv_rank]");
    const int64_t Sk = c_kv.size(1);
    TORCH_CHECK(pe_cache.dim() == 3 && pe_cache.size(0) == B && pe_cache.size(1) == Sk && pe_cache.size(2) == D,
                "pe_cache must be [B, Sk, rope]");
    TORCH_CHECK(W_uv.dim() == 3 && W_uv.size(0) == H && W_uv.size(2) == R, "W_uv must be [H, v_dim, kv_rank]");
    const int64_t V = W_uv.size(1);
    const c10::cuda::CUDAGuard guard(q_absorbed.device());
    auto qa = q_absorbed.contiguous(), qr = q_rope.contiguous(), ck = c_kv.contiguous(), pe = pe_cache.contiguous(),
         wv = W_uv.contiguous();
    auto out = at::empty({B, Sq, H, V}, q_absorbed.options());
    const mla_dtype_t dt = dtype_code(q_absorbed);
    const mla_precision_t pc = precision_code(precision);
    size_t nbytes = 0;
    check_status(mla_attention_workspace_size(dt, pc, B, Sq, Sk, H, R, D, V, causal ? 1 : 0, &nbytes),
                 "mla_attention");
    auto ws = at::empty({int64_t(nbytes > 0 ? nbytes : 1)}, q_absorbed.options().dtype(at::kByte));
    check_status(mla_attention(dt, pc, qa.data_ptr(), qr.data_ptr(), ck.data_ptr(), pe.data_ptr(), wv.data_ptr(), B,
                               Sq, Sk, H, R, D, V, scale, causal ? 1 : 0, out.data_ptr(), ws.data_ptr(),
                               size_t(ws.numel()), at::cuda::getCurrentCUDAStream().stream()),
                 "mla_attention");
    return out;
}

// The reference's bindings (mla_kernels.cu:1688-1692): exact precision, no mask.
std::vector<at::Tensor> ext_q_absorbed(at::Tensor x, at::Tensor W_q_a, at::Tensor q_norm_w, at::Tensor W_q_b,
                                   at::Tensor W_uk, at::Tensor positions, int64_t nope_dim, int64_t rope_dim,
                                   double eps) {
    return ext_q_absorbed_ex(x, W_q_a, q_norm_w, W_q_b, W_uk, positions, nope_dim, rope_dim, eps, "exact");
}

at::Tensor ext_mla_attention(at::Tensor q_absorbed, at::Tensor q_rope, at::Tensor c_kv, at::Tensor pe_cache,
                             at::Tensor W_uv, double scale) {
    return ext_mla_attention_ex(q_absorbed, q_rope, c_kv, pe_cache, W_uv, scale, false, "exact");
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.doc() = "B200-native absorbed MLA (C++ extension over libmla_b200)";
    m.def("q_absorbed", &ext_q_absorbed, "Q path: x -> [q_absorbed, q_rope] (exact precision)");
    m.def("mla_attention", &ext_mla_attention, "absorbed MLA attention (exact precision, no mask)");
    m.def("q_absorbed_ex", &ext_q_absorbed_ex, "q_absorbed with a precision");
    m.def("mla_attention_ex", &ext_mla_attention_ex, "mla_attention with a causal flag and a precision");
    m.def("abi_version", &mla_abi_version);
}
