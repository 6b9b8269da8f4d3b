// Merge of attention computed over disjoint key shards (Sk sharding across
// GPUs): each shard p gives its normalised output O_p and the log-sum-exp
// lse_p of its scaled scores. Softmax over the union of the keys is
//   out = sum_p exp(lse_p - L) O_p,   L = log sum_p exp(lse_p),
// which also holds after the W_uv projection because it is linear. Done in
// fp32; one warp per row.
#include "lse_combine.cuh"

#include <cmath>

namespace mla {
namespace {

template <typename T>
__global__ void __launch_bounds__(256) lse_combine_kernel(int64_t parts, int64_t rows, int64_t v_dim,
                                                          const T* __restrict__ outs, const float* __restrict__ lses,
                                                          T* __restrict__ out, float* __restrict__ lse_out) {
    const int64_t r = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    float M = -INFINITY;
    for (int64_t p = 0; p < parts; ++p) M = fmaxf(M, lses[p * rows + r]);
    float S = 0.f;
    for (int64_t p = 0; p < parts; ++p) S += (M == -INFINITY) ? 0.f : expf(lses[p * rows + r] - M);
    const float L = (S > 0.f) ? M + logf(S) : -INFINITY;
    for (int64_t v = lane; v < v_dim; v += 32) {
        float acc = 0.f;
        for (int64_t p = 0; p < parts; ++p) {
            const float lp = lses[p * rows + r];
            if (lp == -INFINITY) continue;
            acc += expf(lp - L) * cvt<float>(outs[(p * rows + r) * v_dim + v]);
        }
        out[r * v_dim + v] = cvt<T>(acc);
    }
    if (lse_out && lane == 0) lse_out[r] = L;
}

__global__ void fill_kernel(float* p, int64_t n, float v) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
        p[i] = v;
}

}  // namespace

template <typename T>
mla_status_t lse_combine(int64_t parts, int64_t rows, int64_t v_dim, const void* outs, const float* lses, void* out,
                         float* lse_out, cudaStream_t st) {
    if constexpr (std::is_same<T, double>::value) {
        // fp64 partials are combined in fp64 precision by the caller's own code; not built here
        return set_error(MLA_ERR_UNSUPPORTED, "MLA mla_lse_combine: fp64 is not supported");
    } else {
        const int64_t blocks = ceil_div(rows * 32, 256);
        lse_combine_kernel<T><<<unsigned(blocks), 256, 0, st>>>(parts, rows, v_dim, static_cast<const T*>(outs), lses,
                                                                static_cast<T*>(out), lse_out);
        return check_launch("log-sum-exp combine");
    }
}

mla_status_t fill_neg_inf(float* p, int64_t n, cudaStream_t st) {
    int64_t blocks = ceil_div(n, 256);
    if (blocks > 4096) blocks = 4096;
    if (blocks < 1) blocks = 1;
    fill_kernel<<<unsigned(blocks), 256, 0, st>>>(p, n, -INFINITY);
    return check_launch("lse fill");
}

template mla_status_t lse_combine<float>(int64_t, int64_t, int64_t, const void*, const float*, void*, float*, cudaStream_t);
template mla_status_t lse_combine<double>(int64_t, int64_t, int64_t, const void*, const float*, void*, float*, cudaStream_t);
template mla_status_t lse_combine<__half>(int64_t, int64_t, int64_t, const void*, const float*, void*, float*, cudaStream_t);
template mla_status_t lse_combine<__nv_bfloat16>(int64_t, int64_t, int64_t, const void*, const float*, void*, float*,
                                                 cudaStream_t);

}  // namespace mla
