// Argument bundles and entry points of the Q-prep and attention stages, shared
// by the C-ABI layer (abi.cu) and the kernels.
#pragma once

#include "common.cuh"

namespace mla {

constexpr int kMaxRopePairs = 128;   // rope <= 256

struct QArgs {
    const void* x; const void* W_q_a; const void* q_norm_w; const void* W_q_b; const void* W_uk;
    const int64_t* positions;
    int64_t batch, sq, hidden, q_lora, heads, nope, rope, kv_rank;
    double eps;
    void* q_absorbed; void* q_rope;
    void* workspace; size_t workspace_bytes;
};

struct AArgs {
    const void* q_absorbed; const void* q_rope; const void* c_kv; const void* pe_cache; const void* W_uv;
    int64_t batch, sq, sk, heads, kv_rank, rope, v_dim;
    double scale;
    int causal;
    void* out;
    void* workspace; size_t workspace_bytes;
    float* lse;   // optional [B*Sq*H]: natural-log sum of exp(score) per row (partial attention)
    const void* W_uv_bf16;   // optional (fp32 storage, tensor precision): bf16 W_uv; bf16 context for 3d
};

// fp32 -> bf16 copy of n elements (n a multiple of 4), 16-byte aligned buffers
mla_status_t cast_to_bf16(const float* src, __nv_bfloat16* dst, int64_t n, cudaStream_t st);

template <typename T> size_t qprep_exact_workspace(const QArgs& a);
template <typename T> mla_status_t qprep_exact(const QArgs& a, cudaStream_t st);

template <typename T> bool qprep_tensor_supported(const QArgs& a);
template <typename T> size_t qprep_tensor_workspace(const QArgs& a);
template <typename T> mla_status_t qprep_tensor(const QArgs& a, cudaStream_t st);

// fp32 storage, tensor precision, with bf16 weights packed once (qprep_exact.cu)
bool qprep_packed_supported(const QArgs& a);
size_t pack_q_weights_bytes(int64_t hidden, int64_t q_lora, int64_t heads, int64_t nope, int64_t rope, int64_t kv_rank);
mla_status_t pack_q_weights(const float* W_q_a, const float* W_q_b, const float* W_uk, int64_t hidden, int64_t q_lora,
                            int64_t heads, int64_t nope, int64_t rope, int64_t kv_rank, void* packed, cudaStream_t st);
size_t qprep_packed_workspace(const QArgs& a);
mla_status_t qprep_packed(const QArgs& a, const void* packed, cudaStream_t st);

// KV-cache write (kv_write.cu)
bool kv_write_supported(mla_dtype_t dt, int64_t hidden, int64_t kv_rank, int64_t rope);

template <typename T> size_t attn_exact_workspace(const AArgs& a);
template <typename T> mla_status_t attn_exact(const AArgs& a, cudaStream_t st);

}  // namespace mla
