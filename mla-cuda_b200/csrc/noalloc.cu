// Allocation-free variant of the tensor-core attention entry point.
//
// Some callers cannot allocate device memory at call time: an inference server
// that has handed the whole GPU to its own memory pool, or code running where
// cudaMalloc is not allowed to be called. For them this file keeps the
// attention's workspace in one fixed device array, reserved when the library is
// loaded on a device and held until the process exits, and passes it to the
// ordinary tensor-core attention path (mla_attention with MLA_PREC_TENSOR).
//
// Nothing here calls cudaMalloc, cudaFree or any allocating routine.
#include "tc.cuh"

#include <mutex>

namespace {

// Maximum workspace of one call: 96 MiB, enough for B*Sq up to 128 decode rows
// at Sk = 4989 on a 148-SM B200.
constexpr size_t kNoAllocScratchBytes = size_t(96) << 20;

// The shared scratch. Host code must not pass this name to a kernel: on the
// host it is only a stand-in for the device symbol. Its device address is
// looked up below with cudaGetSymbolAddress, per device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mu;

// Device address of the scratch on the current device; looked up on the first
// call made on that device.
mla_status_t scratch_address(void** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return mla::set_error(MLA_ERR_CUDA, "MLA no-alloc attention: no usable current device");
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return mla::set_error(MLA_ERR_CUDA, "MLA no-alloc attention: cudaGetSymbolAddress failed: %s",
                                  cudaGetErrorString(e));
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return MLA_OK;
}

}  // namespace

extern "C" {

MLA_API mla_status_t mla_attention_noalloc(
    mla_dtype_t dtype, const void* q_absorbed, const void* q_rope, const void* c_kv, const void* pe_cache,
    const void* W_uv, int64_t batch, int64_t sq, int64_t sk, int64_t heads, int64_t kv_rank, int64_t rope,
    int64_t v_dim, double scale, int causal, void* out, void* stream)
{
    if (dtype == MLA_DTYPE_F64)
        return mla::set_error(MLA_ERR_UNSUPPORTED, "MLA no-alloc attention: fp64 has no tensor-core path");
    mla::AArgs a{};
    a.batch = batch; a.sq = sq; a.sk = sk; a.heads = heads; a.kv_rank = kv_rank; a.rope = rope; a.v_dim = v_dim;
    a.causal = causal;
    if (batch * sq > 0 && sk > 0 && !mla::tc_attention_supported(a))
        return mla::set_error(MLA_ERR_UNSUPPORTED,
                              "MLA no-alloc attention: shape not covered by the tensor-core kernel "
                              "(needs heads=128, kv_rank=512, rope=64 and batch*sk < 2^31)");
    size_t need = 0;
    MLA_TRY(mla_attention_workspace_size(dtype, MLA_PREC_TENSOR, batch, sq, sk, heads, kv_rank, rope, v_dim, causal,
                                         &need));
    if (need > kNoAllocScratchBytes)
        return mla::set_error(MLA_ERR_WORKSPACE,
                              "MLA no-alloc attention: this shape needs %zu bytes of scratch, above the fixed "
                              "maximum of %zu bytes (use mla_attention with your own workspace)",
                              need, kNoAllocScratchBytes);
    void* ws = nullptr;
    MLA_TRY(scratch_address(&ws));
    return mla_attention(dtype, MLA_PREC_TENSOR, q_absorbed, q_rope, c_kv, pe_cache, W_uv, batch, sq, sk, heads,
                         kv_rank, rope, v_dim, scale, causal, out, ws, kNoAllocScratchBytes, stream);
}

MLA_API size_t mla_attention_noalloc_max_scratch(void) { return kNoAllocScratchBytes; }

}  // extern "C"
