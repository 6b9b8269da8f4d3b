// Log-sum-exp merge of partial attention outputs (key shards).
#pragma once

#include "common.cuh"

namespace mla {

// out[r, :] = sum_p exp(lse[p, r] - L[r]) * outs[p, r, :],  L[r] = log sum_p exp(lse[p, r]).
template <typename T>
mla_status_t lse_combine(int64_t parts, int64_t rows, int64_t v_dim, const void* outs, const float* lses, void* out,
                         float* lse_out, cudaStream_t st);

// Fills n floats with -inf (the log-sum-exp of an empty key set).
mla_status_t fill_neg_inf(float* p, int64_t n, cudaStream_t st);

}  // namespace mla
