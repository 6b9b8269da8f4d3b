// C-ABI entry points (include/mla_b200.h): argument validation, dtype and
// precision dispatch, workspace sizing and error reporting. The validation
// mirrors the reference's TORCH_CHECKs (mla_kernels.cu:627-635) and adds the
// checks the reference's attention launcher leaves out (mla_kernels.cu:1487-1491
// performs none).
#include "qprep.cuh"
#include "tc.cuh"
#include "lse_combine.cuh"

#include <cstdarg>
#include <cstdio>
#include <cstring>

namespace mla {

namespace {
thread_local char g_last_error[512] = "";
}

mla_status_t set_error(mla_status_t st, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return st;
}

mla_status_t check_launch(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return set_error(MLA_ERR_CUDA, "MLA: launch of %s failed: %s", what, cudaGetErrorString(e));
    return MLA_OK;
}

int sm_count() {
    constexpr int kMaxDev = 64;
    static int cached[kMaxDev] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return 148;
    if (cached[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}

bool pdl_enabled() {
    static const bool on = [] {
        const char* e = getenv("MLA_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

namespace {

mla_status_t validate_q(mla_dtype_t dtype, mla_precision_t prec, int64_t batch, int64_t sq, int64_t hidden,
                        int64_t q_lora, int64_t heads, int64_t nope, int64_t rope, int64_t kv_rank) {
    if (dtype < MLA_DTYPE_F32 || dtype > MLA_DTYPE_BF16)
        return set_error(MLA_ERR_UNSUPPORTED, "MLA: unknown dtype %d", int(dtype));
    if (prec != MLA_PREC_EXACT && prec != MLA_PREC_TENSOR)
        return set_error(MLA_ERR_UNSUPPORTED, "MLA: unknown precision %d", int(prec));
    if (batch < 0 || sq < 0 || hidden <= 0 || q_lora <= 0 || heads <= 0 || nope <= 0 || rope < 0 || kv_rank <= 0)
        return set_error(MLA_ERR_INVALID_ARGUMENT,
                         "MLA q_absorbed: sizes must be positive (batch=%lld sq=%lld hidden=%lld q_lora=%lld "
                         "heads=%lld nope=%lld rope=%lld kv_rank=%lld)",
                         (long long)batch, (long long)sq, (long long)hidden, (long long)q_lora, (long long)heads,
                         (long long)nope, (long long)rope, (long long)kv_rank);
    if (rope % 2 != 0 || rope / 2 > kMaxRopePairs)
        return set_error(MLA_ERR_INVALID_ARGUMENT, "MLA q_absorbed: rope_dim must be even and <= %d (got %lld)",
                         2 * kMaxRopePairs, (long long)rope);
    return MLA_OK;
}

mla_status_t validate_a(mla_dtype_t dtype, mla_precision_t prec, int64_t batch, int64_t sq, int64_t sk,
                        int64_t heads, int64_t kv_rank, int64_t rope, int64_t v_dim, int causal) {
    if (dtype < MLA_DTYPE_F32 || dtype > MLA_DTYPE_BF16)
        return set_error(MLA_ERR_UNSUPPORTED, "MLA: unknown dtype %d", int(dtype));
    if (prec != MLA_PREC_EXACT && prec != MLA_PREC_TENSOR)
        return set_error(MLA_ERR_UNSUPPORTED, "MLA: unknown precision %d", int(prec));
    if (batch < 0 || sq < 0 || sk < 0 || heads <= 0 || kv_rank <= 0 || rope < 0 || v_dim <= 0)
        return set_error(MLA_ERR_INVALID_ARGUMENT,
                         "MLA mla_attention: invalid sizes (batch=%lld sq=%lld sk=%lld heads=%lld kv_rank=%lld "
                         "rope=%lld v_dim=%lld)",
                         (long long)batch, (long long)sq, (long long)sk, (long long)heads, (long long)kv_rank,
                         (long long)rope, (long long)v_dim);
    if (causal && sk < sq)
        return set_error(MLA_ERR_INVALID_ARGUMENT, "MLA mla_attention: causal masking needs sk >= sq (sk=%lld sq=%lld)",
                         (long long)sk, (long long)sq);
    if (batch > 65535)
        return set_error(MLA_ERR_UNSUPPORTED, "MLA mla_attention: batch > 65535 is not supported (got %lld)",
                         (long long)batch);
    return MLA_OK;
}

template <typename F>
auto dispatch(mla_dtype_t dt, F&& f) {
    switch (dt) {
        case MLA_DTYPE_F64: return f(double{});
        case MLA_DTYPE_F16: return f(__half{});
        case MLA_DTYPE_BF16: return f(__nv_bfloat16{});
        default: return f(float{});
    }
}

// Tensor precision, and exact precision for 16-bit storage (tcgen05 kind::f16
// products are exact in fp32; the kernel's exact variant keeps scores and
// probabilities fp32-class), run the tensor-core attention where it covers the shape.
bool exact16(mla_dtype_t dt, mla_precision_t prec) {
    return prec == MLA_PREC_EXACT && (dt == MLA_DTYPE_BF16 || dt == MLA_DTYPE_F16);
}
bool use_tc_attention(mla_dtype_t dt, mla_precision_t prec, const AArgs& a) {
    return ((prec == MLA_PREC_TENSOR && dt != MLA_DTYPE_F64) || exact16(dt, prec)) && tc_attention_supported(a);
}

}  // namespace
}  // namespace mla

using namespace mla;

extern "C" {

int mla_abi_version(void) { return MLA_B200_ABI_VERSION; }

const char* mla_status_string(mla_status_t s) {
    switch (s) {
        case MLA_OK: return "ok";
        case MLA_ERR_INVALID_ARGUMENT: return "invalid argument";
        case MLA_ERR_UNSUPPORTED: return "unsupported";
        case MLA_ERR_WORKSPACE: return "workspace too small";
        case MLA_ERR_CUDA: return "CUDA error";
        case MLA_ERR_DEVICE: return "device-side failure";
    }
    return "unknown status";
}

const char* mla_last_error_message(void) { return g_last_error; }

mla_status_t mla_q_absorbed_workspace_size(mla_dtype_t dtype, mla_precision_t precision, int64_t batch, int64_t sq,
                                           int64_t hidden, int64_t q_lora, int64_t heads, int64_t nope, int64_t rope,
                                           int64_t kv_rank, size_t* bytes) {
    MLA_TRY(validate_q(dtype, precision, batch, sq, hidden, q_lora, heads, nope, rope, kv_rank));
    if (!bytes) return set_error(MLA_ERR_INVALID_ARGUMENT, "MLA: bytes must not be NULL");
    QArgs a{};
    a.batch = batch; a.sq = sq; a.hidden = hidden; a.q_lora = q_lora;
    a.heads = heads; a.nope = nope; a.rope = rope; a.kv_rank = kv_rank;
    *bytes = dispatch(dtype, [&](auto t) {
        using T = decltype(t);
        return (precision == MLA_PREC_TENSOR && qprep_tensor_supported<T>(a)) ? qprep_tensor_workspace<T>(a)
                                                                               : qprep_exact_workspace<T>(a);
    });
    return MLA_OK;
}

mla_status_t mla_q_absorbed(mla_dtype_t dtype, mla_precision_t precision, const void* x, const void* W_q_a,
                            const void* q_norm_w, const void* W_q_b, const void* W_uk, const int64_t* positions,
                            int64_t batch, int64_t sq, int64_t hidden, int64_t q_lora, int64_t heads, int64_t nope,
                            int64_t rope, int64_t kv_rank, double eps, void* q_absorbed, void* q_rope,
                            void* workspace, size_t workspace_bytes, void* stream) {
    MLA_TRY(validate_q(dtype, precision, batch, sq, hidden, q_lora, heads, nope, rope, kv_rank));
    if (batch * sq == 0) return MLA_OK;
    if (!x || !W_q_a || !q_norm_w || !W_q_b || !W_uk || !positions || !q_absorbed || (rope > 0 && !q_rope))
        return set_error(MLA_ERR_INVALID_ARGUMENT, "MLA q_absorbed: null operand pointer");
    QArgs a{x, W_q_a, q_norm_w, W_q_b, W_uk, positions, batch, sq, hidden, q_lora, heads, nope, rope, kv_rank,
            eps, q_absorbed, q_rope, workspace, workspace_bytes};
    const bool tc = dispatch(dtype, [&](auto t) {
        return precision == MLA_PREC_TENSOR && qprep_tensor_supported<decltype(t)>(a);
    });
    const size_t need = dispatch(dtype, [&](auto t) {
        return tc ? qprep_tensor_workspace<decltype(t)>(a) : qprep_exact_workspace<decltype(t)>(a);
    });
    if (need > 0 && (!workspace || workspace_bytes < need))
        return set_error(MLA_ERR_WORKSPACE, "MLA q_absorbed: workspace of %zu bytes needed, %zu given", need,
                         workspace ? workspace_bytes : size_t(0));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (tc) return dispatch(dtype, [&](auto t) { return qprep_tensor<decltype(t)>(a, st); });
    return dispatch(dtype, [&](auto t) { return qprep_exact<decltype(t)>(a, st); });
}

mla_status_t mla_pack_q_weights_size(mla_dtype_t dtype, int64_t hidden, int64_t q_lora, int64_t heads, int64_t nope,
                                    int64_t rope, int64_t kv_rank, size_t* bytes) {
    MLA_TRY(validate_q(dtype, MLA_PREC_TENSOR, 1, 1, hidden, q_lora, heads, nope, rope, kv_rank));
    if (dtype != MLA_DTYPE_F32)
        return set_error(MLA_ERR_UNSUPPORTED, "MLA: weight packing is for fp32 storage (16-bit weights are used as is)");
    if (!bytes) return set_error(MLA_ERR_INVALID_ARGUMENT, "MLA: bytes must not be NULL");
    *bytes = pack_q_weights_bytes(hidden, q_lora, heads, nope, rope, kv_rank);
    return MLA_OK;
}

mla_status_t mla_pack_q_weights(mla_dtype_t dtype, const void* W_q_a, const void* W_q_b, const void* W_uk,
                                int64_t hidden, int64_t q_lora, int64_t heads, int64_t nope, int64_t rope,
                                int64_t kv_rank, void* packed, size_t packed_bytes, void* stream) {
    size_t need = 0;
    MLA_TRY(mla_pack_q_weights_size(dtype, hidden, q_lora, heads, nope, rope, kv_rank, &need));
    if (!W_q_a || !W_q_b || !W_uk || !packed)
        return set_error(MLA_ERR_INVALID_ARGUMENT, "MLA pack_q_weights: null pointer");
    if (packed_bytes < need)
        return set_error(MLA_ERR_WORKSPACE, "MLA pack_q_weights: %zu bytes needed, %zu given", need, packed_bytes);
    if (hidden * q_lora % 4 != 0 || q_lora * heads * (nope + rope) % 4 != 0 || heads * nope * kv_rank % 4 != 0)
        return set_error(MLA_ERR_UNSUPPORTED, "MLA pack_q_weights: weight sizes must be multiples of 4");
    return pack_q_weights(static_cast<const float*>(W_q_a), static_cast<const float*>(W_q_b),
                          static_cast<const float*>(W_uk), hidden, q_lora, heads, nope, rope, kv_rank, packed,
                          static_cast<cudaStream_t>(stream));
}

mla_status_t mla_q_absorbed_packed_workspace_size(mla_dtype_t dtype, int64_t batch, int64_t sq, int64_t hidden,
                                                  int64_t q_lora, int64_t heads, int64_t nope, int64_t rope,
                                                  int64_t kv_rank, size_t* bytes) {
    MLA_TRY(validate_q(dtype, MLA_PREC_TENSOR, batch, sq, hidden, q_lora, heads, nope, rope, kv_rank));
    if (dtype != MLA_DTYPE_F32) return set_error(MLA_ERR_UNSUPPORTED, "MLA: packed Q-prep is for fp32 storage");
    if (!bytes) return set_error(MLA_ERR_INVALID_ARGUMENT, "MLA: bytes must not be NULL");
    QArgs a{};
    a.batch = batch; a.sq = sq; a.hidden = hidden; a.q_lora = q_lora;
    a.heads = heads; a.nope = nope; a.rope = rope; a.kv_rank = kv_rank;
    *bytes = (batch * sq == 0) ? 0 : qprep_packed_workspace(a);
    return MLA_OK;
}

mla_status_t mla_q_absorbed_packed(mla_dtype_t dtype, const void* x, const void* packed, const void* q_norm_w,
                                   const int64_t* positions, int64_t batch, int64_t sq, int64_t hidden,
                                   int64_t q_lora, int64_t heads, int64_t nope, int64_t rope, int64_t kv_rank,
                                   double eps, void* q_absorbed, void* q_rope, void* workspace,
                                   size_t workspace_bytes, void* stream) {
    size_t need = 0;
    MLA_TRY(mla_q_absorbed_packed_workspace_size(dtype, batch, sq, hidden, q_lora, heads, nope, rope, kv_rank, &need));
    if (batch * sq == 0) return MLA_OK;
    if (!x || !packed || !q_norm_w || !positions || !q_absorbed || !q_rope)
        return set_error(MLA_ERR_INVALID_ARGUMENT, "MLA q_absorbed_packed: null operand pointer");
    QArgs a{x, nullptr, q_norm_w, nullptr, nullptr, positions, batch, sq, hidden, q_lora, heads, nope, rope, kv_rank,
            eps, q_absorbed, q_rope, workspace, workspace_bytes};
    if (!qprep_packed_supported(a))
        return set_error(MLA_ERR_UNSUPPORTED, "MLA q_absorbed_packed: shape not covered (needs q_lora, heads*(nope+rope), "
                                              "kv_rank multiples of 32, hidden and nope multiples of 8, q_lora <= 4096)");
    if (!workspace || workspace_bytes < need)
        return set_error(MLA_ERR_WORKSPACE, "MLA q_absorbed_packed: workspace of %zu bytes needed, %zu given", need,
                         workspace ? workspace_bytes : size_t(0));
    return qprep_packed(a, packed, static_cast<cudaStream_t>(stream));
}

mla_status_t mla_attention_workspace_size(mla_dtype_t dtype, mla_precision_t precision, int64_t batch, int64_t sq,
                                          int64_t sk, int64_t heads, int64_t kv_rank, int64_t rope, int64_t v_dim,
                                          int causal, size_t* bytes) {
    MLA_TRY(validate_a(dtype, precision, batch, sq, sk, heads, kv_rank, rope, v_dim, causal));
    if (!bytes) return set_error(MLA_ERR_INVALID_ARGUMENT, "MLA: bytes must not be NULL");
    AArgs a{};
    a.batch = batch; a.sq = sq; a.sk = sk; a.heads = heads; a.kv_rank = kv_rank; a.rope = rope; a.v_dim = v_dim;
    a.causal = causal;
    if (use_tc_attention(dtype, precision, a))
        *bytes = dispatch(dtype, [&](auto t) { return tc_attention_workspace<decltype(t)>(a); });
    else
        *bytes = dispatch(dtype, [&](auto t) { return attn_exact_workspace<decltype(t)>(a); });
    return MLA_OK;
}

}  // extern "C"

static mla_status_t attention_impl(mla_dtype_t dtype, mla_precision_t precision, const void* q_absorbed, const void* q_rope,
                           const void* c_kv, const void* pe_cache, const void* W_uv, int64_t batch, int64_t sq,
                           int64_t sk, int64_t heads, int64_t kv_rank, int64_t rope, int64_t v_dim, double scale,
                           int causal, void* out, float* lse, void* workspace, size_t workspace_bytes, void* stream,
                           const void* W_uv_bf16 = nullptr) {
    MLA_TRY(validate_a(dtype, precision, batch, sq, sk, heads, kv_rank, rope, v_dim, causal));
    if (batch * sq == 0) return MLA_OK;
    if (!out || !W_uv || !q_absorbed) return set_error(MLA_ERR_INVALID_ARGUMENT, "MLA mla_attention: null pointer");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (sk == 0) {
        // Softmax over no keys: the reference's einsums reduce over an empty axis.
        const size_t esz = dtype == MLA_DTYPE_F64 ? 8 : dtype == MLA_DTYPE_F32 ? 4 : 2;
        if (cudaMemsetAsync(out, 0, size_t(batch * sq * heads * v_dim) * esz, st) != cudaSuccess)
            return set_error(MLA_ERR_CUDA, "MLA mla_attention: memset failed");
        if (lse) return fill_neg_inf(lse, batch * sq * heads, st);   // an empty shard weighs nothing
        return MLA_OK;
    }
    if (!c_kv || (rope > 0 && (!q_rope || !pe_cache)))
        return set_error(MLA_ERR_INVALID_ARGUMENT, "MLA mla_attention: null operand pointer");
    if (scale == 0.0) return set_error(MLA_ERR_INVALID_ARGUMENT, "MLA mla_attention: scale must be non-zero");
    AArgs a{q_absorbed, q_rope, c_kv, pe_cache, W_uv, batch, sq, sk, heads, kv_rank, rope, v_dim,
            scale, causal, out, workspace, workspace_bytes, lse};
    a.W_uv_bf16 = W_uv_bf16;
    const bool tc = use_tc_attention(dtype, precision, a);
    const size_t need = tc ? dispatch(dtype, [&](auto t) { return tc_attention_workspace<decltype(t)>(a); })
                           : dispatch(dtype, [&](auto t) { return attn_exact_workspace<decltype(t)>(a); });
    if (need > 0 && (!workspace || workspace_bytes < need))
        return set_error(MLA_ERR_WORKSPACE, "MLA mla_attention: workspace of %zu bytes needed, %zu given", need,
                         workspace ? workspace_bytes : size_t(0));
    if (tc) return dispatch(dtype, [&](auto t) { return tc_attention<decltype(t)>(a, st, exact16(dtype, precision)); });
    return dispatch(dtype, [&](auto t) { return attn_exact<decltype(t)>(a, st); });
}

extern "C" {

mla_status_t mla_attention(mla_dtype_t dtype, mla_precision_t precision, const void* q_absorbed, const void* q_rope,
                           const void* c_kv, const void* pe_cache, const void* W_uv, int64_t batch, int64_t sq,
                           int64_t sk, int64_t heads, int64_t kv_rank, int64_t rope, int64_t v_dim, double scale,
                           int causal, void* out, void* workspace, size_t workspace_bytes, void* stream) {
    return attention_impl(dtype, precision, q_absorbed, q_rope, c_kv, pe_cache, W_uv, batch, sq, sk, heads, kv_rank,
                          rope, v_dim, scale, causal, out, nullptr, workspace, workspace_bytes, stream);
}

mla_status_t mla_pack_uv_weights_size(mla_dtype_t dtype, int64_t heads, int64_t v_dim, int64_t kv_rank, size_t* bytes) {
    if (dtype != MLA_DTYPE_F32)
        return set_error(MLA_ERR_UNSUPPORTED, "MLA: W_uv packing is for fp32 storage (16-bit weights are used as is)");
    if (!bytes) return set_error(MLA_ERR_INVALID_ARGUMENT, "MLA: bytes must not be NULL");
    if (heads <= 0 || v_dim <= 0 || kv_rank <= 0)
        return set_error(MLA_ERR_INVALID_ARGUMENT, "MLA pack_uv_weights: sizes must be positive");
    *bytes = size_t(heads * v_dim * kv_rank) * 2;
    return MLA_OK;
}

mla_status_t mla_pack_uv_weights(mla_dtype_t dtype, const void* W_uv, int64_t heads, int64_t v_dim, int64_t kv_rank,
                                 void* packed, size_t packed_bytes, void* stream) {
    size_t need = 0;
    MLA_TRY(mla_pack_uv_weights_size(dtype, heads, v_dim, kv_rank, &need));
    if (!W_uv || !packed) return set_error(MLA_ERR_INVALID_ARGUMENT, "MLA pack_uv_weights: null pointer");
    if (packed_bytes < need)
        return set_error(MLA_ERR_WORKSPACE, "MLA pack_uv_weights: %zu bytes needed, %zu given", need, packed_bytes);
    if ((heads * v_dim * kv_rank) % 4 != 0 || reinterpret_cast<uintptr_t>(W_uv) % 16 != 0 ||
        reinterpret_cast<uintptr_t>(packed) % 16 != 0)
        return set_error(MLA_ERR_UNSUPPORTED, "MLA pack_uv_weights: needs a multiple of 4 elements, 16-byte aligned");
    return cast_to_bf16(static_cast<const float*>(W_uv), static_cast<__nv_bfloat16*>(packed), heads * v_dim * kv_rank,
                        static_cast<cudaStream_t>(stream));
}

mla_status_t mla_attention_packed_uv(mla_dtype_t dtype, const void* q_absorbed, const void* q_rope, const void* c_kv,
                                     const void* pe_cache, const void* W_uv_packed, int64_t batch, int64_t sq,
                                     int64_t sk, int64_t heads, int64_t kv_rank, int64_t rope, int64_t v_dim,
                                     double scale, int causal, void* out, void* workspace, size_t workspace_bytes,
                                     void* stream) {
    if (dtype != MLA_DTYPE_F32)
        return set_error(MLA_ERR_UNSUPPORTED, "MLA mla_attention_packed_uv: fp32 storage only");
    AArgs a{};
    a.batch = batch; a.sq = sq; a.sk = sk; a.heads = heads; a.kv_rank = kv_rank; a.rope = rope; a.v_dim = v_dim;
    a.causal = causal;
    if (batch * sq > 0 && sk > 0 && (!tc_attention_supported(a) || v_dim % 32 != 0))
        return set_error(MLA_ERR_UNSUPPORTED, "MLA mla_attention_packed_uv: shape not covered by the tensor-core "
                                              "attention (heads 128, kv_rank 512, rope 64, v_dim a multiple of 32)");
    if (!W_uv_packed) return set_error(MLA_ERR_INVALID_ARGUMENT, "MLA mla_attention_packed_uv: null W_uv_packed");
    return attention_impl(dtype, MLA_PREC_TENSOR, q_absorbed, q_rope, c_kv, pe_cache, W_uv_packed, batch, sq, sk,
                          heads, kv_rank, rope, v_dim, scale, causal, out, nullptr, workspace, workspace_bytes, stream,
                          W_uv_packed);
}

mla_status_t mla_attention_partial(mla_dtype_t dtype, mla_precision_t precision, const void* q_absorbed,
                                   const void* q_rope, const void* c_kv, const void* pe_cache, const void* W_uv,
                                   int64_t batch, int64_t sq, int64_t sk, int64_t heads, int64_t kv_rank, int64_t rope,
                                   int64_t v_dim, double scale, void* out, float* lse, void* workspace,
                                   size_t workspace_bytes, void* stream) {
    if (!lse) return set_error(MLA_ERR_INVALID_ARGUMENT, "MLA mla_attention_partial: lse must not be NULL");
    return attention_impl(dtype, precision, q_absorbed, q_rope, c_kv, pe_cache, W_uv, batch, sq, sk, heads, kv_rank,
                          rope, v_dim, scale, 0, out, lse, workspace, workspace_bytes, stream);
}

mla_status_t mla_lse_combine(mla_dtype_t dtype, int64_t parts, int64_t rows, int64_t v_dim, const void* outs,
                             const float* lses, void* out, float* lse_out, void* stream) {
    if (dtype < MLA_DTYPE_F32 || dtype > MLA_DTYPE_BF16)
        return set_error(MLA_ERR_UNSUPPORTED, "MLA: unknown dtype %d", int(dtype));
    if (parts <= 0 || rows < 0 || v_dim <= 0)
        return set_error(MLA_ERR_INVALID_ARGUMENT, "MLA mla_lse_combine: invalid sizes (parts=%lld rows=%lld v=%lld)",
                         (long long)parts, (long long)rows, (long long)v_dim);
    if (rows == 0) return MLA_OK;
    if (!outs || !lses || !out) return set_error(MLA_ERR_INVALID_ARGUMENT, "MLA mla_lse_combine: null pointer");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    return dispatch(dtype, [&](auto t) {
        return lse_combine<decltype(t)>(parts, rows, v_dim, outs, lses, out, lse_out, st);
    });
}

}  // extern "C"
