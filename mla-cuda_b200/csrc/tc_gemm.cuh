// Tensor-core (tcgen05) GEMM for the dense stages of the MLA forward:
// 2a1 / 2a2 (split-K projections) and 2c / 3d (one GEMM per head).
#pragma once

#include "common.cuh"

namespace mla {

// C[z][m][n] = sum_k A[z][m][k] * B[z][k][n], accumulated in fp32 on the tensor
// cores (kind::tf32 for fp32 operands, kind::f16 for bf16 / fp16).
//   A : 3-D tensor {K, Ay, M} (innermost first), element (k, y, m) at
//       k + y*a_ld[0] + m*a_ld[1]; a batched GEMM reads y = z.
//   B : MN-major {N, K, Bz}: element (n, k, z) at n + k*b_ld[0] + z*b_ld[1]
//       (a row-major [K][N] weight), or K-major {K, N, Bz}: (k, n, z) at
//       k + n*b_ld[0] + z*b_ld[1] (a row-major [N][K] weight).
//   split: z indexes slices of K (chunk k_chunk, a multiple of the K block);
//       otherwise z indexes the batch (y of A, z of B).
//   C : element (m, n) of slice / batch z at c + m*c_ldm + z*c_ldz + n, stored
//       as fp32 or as the storage dtype (c_is_t).
struct TcGemm {
    const void* A; int64_t a_dims[3]; int64_t a_ld[2];
    const void* B; bool b_mn; int64_t b_dims[3]; int64_t b_ld[2];
    int64_t M, N, K;
    int Z; bool split; int64_t k_chunk;
    void* C; bool c_is_t; int64_t c_ldm, c_ldz;
    int bn;          // 128 or 256 output columns per CTA
    int* err;        // device error word (bounded waits)
};

template <typename T> mla_status_t tc_gemm(const TcGemm& g, cudaStream_t st);

// K block of the GEMM (one 128-byte swizzle row of the operand dtype).
template <typename T> constexpr int tc_gemm_bk() { return 128 / int(sizeof(T)); }

}  // namespace mla
