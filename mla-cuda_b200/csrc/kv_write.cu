// KV-cache write: the step upstream of the decode read. For every new token
// (b, s) of a decode or prefill step:
//
//   kv        = x[b, s] @ W_kv_a                       [kv_rank + rope]
//   c_kv[b, slot[s]]     = RMSNorm(kv[:kv_rank]) * kv_norm_w
//   pe_cache[b, slot[s]] = RoPE(kv[kv_rank:], positions[s])
//
// The reference has no kernel for this step (its caches are inputs, and the
// write is only mentioned: exhaustive_benchmark_suite.py:189). The arithmetic
// composes the reference's own functions: rmsnorm (:252-258, accumulate dtype,
// the normalised value narrowed to the storage dtype before the gain) and
// apply_rope (:210-232, interleaved pairs, theta 10000, angles in the
// accumulate dtype, cos / sin narrowed to the storage dtype).
//
// The projection is a split-K tcgen05 GEMM (3xTF32 for fp32 storage in exact
// precision, kind::tf32 in tensor precision, kind::f16 for 16-bit storage)
// into fp32 partials; one block per token then sums the partials, normalises,
// rotates and writes the two cache rows. A slot outside [0, capacity) is not
// written: the kernel records code 950 in the device status block instead.
#include "qprep.cuh"
#include "tc_gemm.cuh"

#include <cmath>
#include <type_traits>

namespace mla {

constexpr int kErrKvSlot = 950;

namespace {

constexpr int kMaxKvRank = 1024;

template <typename T>
struct KvRope { float inv_freq[kMaxRopePairs]; };

// One block of 256 threads per token m = b * sq + s.
template <typename T>
__global__ void __launch_bounds__(256) kv_norm_rope_write_kernel(
    const float* __restrict__ P, int splits, int64_t M, int64_t sq, int64_t kv_rank, int64_t rope,
    const T* __restrict__ gain, const int64_t* __restrict__ positions, const int64_t* __restrict__ slots,
    int64_t capacity, float eps, const KvRope<T> tab, T* __restrict__ c_kv, T* __restrict__ pe_cache,
    int* __restrict__ err)
{
    const int64_t m = blockIdx.x;
    const int64_t s = m % sq, b = m / sq;
    const int64_t ncols = kv_rank + rope;
    const int64_t slot = slots[s];
    const bool ok = slot >= 0 && slot < capacity;
    if (!ok) {
        if (threadIdx.x == 0) atomicCAS(err, 0, kErrKvSlot);
        return;
    }
    auto col = [&](int64_t n) {
        float v = 0.f;
        for (int z = 0; z < splits; ++z) v += P[(int64_t(z) * M + m) * ncols + n];
        return v;
    };
    // RMSNorm over the latent part
    float kept[kMaxKvRank / 256];
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < kMaxKvRank / 256; ++e) {
        const int64_t n = threadIdx.x + int64_t(e) * 256;
        kept[e] = n < kv_rank ? col(n) : 0.f;
        ss = fmaf(kept[e], kept[e], ss);
    }
    __shared__ float red[8];
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < 8; ++w) tot += red[w];
    const float inv_rms = 1.f / sqrtf(tot / float(kv_rank) + eps);
    T* crow = c_kv + (b * capacity + slot) * kv_rank;
#pragma unroll
    for (int e = 0; e < kMaxKvRank / 256; ++e) {
        const int64_t n = threadIdx.x + int64_t(e) * 256;
        if (n < kv_rank) crow[n] = cvt<T>(cvt<float>(cvt<T>(kept[e] * inv_rms)) * cvt<float>(gain[n]));
    }
    // RoPE on the rope part, one pair per thread
    const float pos = float(positions[s]);
    T* prow = pe_cache + (b * capacity + slot) * rope;
    for (int64_t j = threadIdx.x; j < rope / 2; j += 256) {
        const float ev = col(kv_rank + 2 * j), od = col(kv_rank + 2 * j + 1);
        const float ang = pos * tab.inv_freq[j];
        const float c = cvt<float>(cvt<T>(cosf(ang))), sn = cvt<float>(cvt<T>(sinf(ang)));
        prow[2 * j] = cvt<T>(ev * c - od * sn);
        prow[2 * j + 1] = cvt<T>(ev * sn + od * c);
    }
}

struct KvPlan {
    int split;
    int64_t chunk;
    size_t total;
};

KvPlan make_kv_plan(int64_t M, int64_t hidden, int64_t ncols, int64_t bk) {
    KvPlan p{};
    const int64_t tiles = ceil_div(M, 128) * ceil_div(ncols, 128);
    const int64_t kblocks = ceil_div(hidden, bk);
    int64_t s = sm_count() / (tiles > 0 ? tiles : 1);
    if (s > kblocks / 4) s = kblocks / 4;
    if (s > 16) s = 16;
    if (s < 1) s = 1;
    const int64_t cb = ceil_div(kblocks, s);
    p.chunk = cb * bk;
    p.split = int(ceil_div(kblocks, cb));
    p.total = align_up(size_t(p.split) * M * ncols * sizeof(float), 256);
    return p;
}

}  // namespace

bool kv_write_supported(mla_dtype_t dt, int64_t hidden, int64_t kv_rank, int64_t rope) {
    const int64_t v = dt == MLA_DTYPE_F32 ? 4 : 8;
    return dt != MLA_DTYPE_F64 && kv_rank <= kMaxKvRank && rope % 2 == 0 && rope / 2 <= kMaxRopePairs &&
           (kv_rank + rope) % 32 == 0 && hidden % v == 0;
}

template <typename T>
size_t kv_write_workspace(int64_t M, int64_t hidden, int64_t kv_rank, int64_t rope) {
    return make_kv_plan(M, hidden, kv_rank + rope, tc_gemm_bk<T>()).total;
}

template <typename T>
mla_status_t kv_write(const void* x, const void* W_kv_a, const void* kv_norm_w, const int64_t* positions,
                      const int64_t* slots, int64_t batch, int64_t sq, int64_t hidden, int64_t kv_rank, int64_t rope,
                      int64_t capacity, double eps, bool exact, void* c_kv, void* pe_cache, void* workspace,
                      cudaStream_t st) {
    const int64_t M = batch * sq;
    const int64_t ncols = kv_rank + rope;
    const KvPlan p = make_kv_plan(M, hidden, ncols, tc_gemm_bk<T>());
    DeviceStatus* dst = nullptr;
    MLA_TRY(device_status_block(&dst));
    float* P = static_cast<float*>(workspace);
    TcGemm g{};   // kv = x [M, hidden] @ W_kv_a [hidden, kv_rank + rope]
    g.A = x; g.a_dims[0] = hidden; g.a_dims[1] = 1; g.a_dims[2] = M; g.a_ld[0] = hidden; g.a_ld[1] = hidden;
    g.B = W_kv_a; g.b_mn = true; g.b_dims[0] = ncols; g.b_dims[1] = hidden; g.b_dims[2] = 1;
    g.b_ld[0] = ncols; g.b_ld[1] = ncols * hidden;
    g.M = M; g.N = ncols; g.K = hidden; g.Z = p.split; g.spb = p.split; g.k_chunk = p.chunk;
    g.C = P; g.c_is_t = false; g.c_ldm = ncols; g.c_ldz = M * ncols; g.bn = 128; g.err = &dst->code;
    g.split3 = exact && std::is_same<T, float>::value;
    MLA_TRY(tc_gemm<T>(g, st));
    KvRope<T> tab{};
    // 1 / fp32(10000^(2j/rope)) in fp32, as the reference's apply_rope computes its
    // inverse frequencies (an fp32 power, then an fp32 division)
    for (int64_t j = 0; j < rope / 2; ++j)
        tab.inv_freq[j] = 1.0f / float(std::pow(10000.0, double(2 * j) / double(rope)));
    kv_norm_rope_write_kernel<T><<<unsigned(M), 256, 0, st>>>(
        P, p.split, M, sq, kv_rank, rope, static_cast<const T*>(kv_norm_w), positions, slots, capacity, float(eps),
        tab, static_cast<T*>(c_kv), static_cast<T*>(pe_cache), &dst->code);
    return check_launch("KV-cache write");
}

#define MLA_KV(T) \
    template size_t kv_write_workspace<T>(int64_t, int64_t, int64_t, int64_t); \
    template mla_status_t kv_write<T>(const void*, const void*, const void*, const int64_t*, const int64_t*, \
                                      int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, double, bool, void*, \
                                      void*, void*, cudaStream_t);
MLA_KV(float)
MLA_KV(__half)
MLA_KV(__nv_bfloat16)
#undef MLA_KV

}  // namespace mla

using namespace mla;

extern "C" {

mla_status_t mla_kv_cache_write_workspace_size(mla_dtype_t dtype, mla_precision_t precision, int64_t batch,
                                               int64_t sq, int64_t hidden, int64_t kv_rank, int64_t rope,
                                               size_t* bytes) {
    if (!bytes) return set_error(MLA_ERR_INVALID_ARGUMENT, "MLA: bytes must not be NULL");
    if (precision != MLA_PREC_EXACT && precision != MLA_PREC_TENSOR)
        return set_error(MLA_ERR_UNSUPPORTED, "MLA: unknown precision %d", int(precision));
    if (batch < 0 || sq < 0 || hidden <= 0 || kv_rank <= 0 || rope < 0)
        return set_error(MLA_ERR_INVALID_ARGUMENT, "MLA kv_cache_write: invalid sizes");
    if (!kv_write_supported(dtype, hidden, kv_rank, rope))
        return set_error(MLA_ERR_UNSUPPORTED,
                         "MLA kv_cache_write: needs fp32 / fp16 / bf16, kv_rank <= 1024, even rope, "
                         "kv_rank + rope a multiple of 32, hidden a multiple of 16 bytes");
    const int64_t M = batch * sq;
    if (M == 0) { *bytes = 0; return MLA_OK; }
    *bytes = dtype == MLA_DTYPE_F32 ? kv_write_workspace<float>(M, hidden, kv_rank, rope)
           : dtype == MLA_DTYPE_F16 ? kv_write_workspace<__half>(M, hidden, kv_rank, rope)
                                    : kv_write_workspace<__nv_bfloat16>(M, hidden, kv_rank, rope);
    return MLA_OK;
}

mla_status_t mla_kv_cache_write(mla_dtype_t dtype, mla_precision_t precision, const void* x, const void* W_kv_a,
                                const void* kv_norm_w, const int64_t* positions, const int64_t* slots,
                                int64_t batch, int64_t sq, int64_t hidden, int64_t kv_rank, int64_t rope,
                                int64_t capacity, double eps, void* c_kv, void* pe_cache, void* workspace,
                                size_t workspace_bytes, void* stream) {
    size_t need = 0;
    MLA_TRY(mla_kv_cache_write_workspace_size(dtype, precision, batch, sq, hidden, kv_rank, rope, &need));
    if (batch * sq == 0) return MLA_OK;
    if (capacity <= 0) return set_error(MLA_ERR_INVALID_ARGUMENT, "MLA kv_cache_write: capacity must be positive");
    if (!x || !W_kv_a || !kv_norm_w || !positions || !slots || !c_kv || (rope > 0 && !pe_cache))
        return set_error(MLA_ERR_INVALID_ARGUMENT, "MLA kv_cache_write: null pointer");
    if (!workspace || workspace_bytes < need)
        return set_error(MLA_ERR_WORKSPACE, "MLA kv_cache_write: workspace of %zu bytes needed, %zu given", need,
                         workspace ? workspace_bytes : size_t(0));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const bool exact = precision == MLA_PREC_EXACT;
    switch (dtype) {
        case MLA_DTYPE_F32:
            return kv_write<float>(x, W_kv_a, kv_norm_w, positions, slots, batch, sq, hidden, kv_rank, rope, capacity,
                                   eps, exact, c_kv, pe_cache, workspace, st);
        case MLA_DTYPE_F16:
            return kv_write<__half>(x, W_kv_a, kv_norm_w, positions, slots, batch, sq, hidden, kv_rank, rope,
                                    capacity, eps, exact, c_kv, pe_cache, workspace, st);
        default:
            return kv_write<__nv_bfloat16>(x, W_kv_a, kv_norm_w, positions, slots, batch, sq, hidden, kv_rank, rope,
                                           capacity, eps, exact, c_kv, pe_cache, workspace, st);
    }
}

}  // extern "C"
