// Tensor-core (tcgen05) GEMM for the dense stages of the MLA forward:
// 2a1 / 2a2 (split-K projections) and 2c / 3d (one GEMM per head).
#pragma once

#include "common.cuh"

namespace mla {

// Optional epilogue of the persistent kernel for the q up-projection (2a2):
// instead of storing C, each row m's columns are split per head h into the nope
// part, stored to q_nope[m, h, :] in the operand dtype (the left operand of 2c),
// and the rope part, rotated by positions[m % sq] * inv_freq[j] (interleaved
// pairs, cos / sin in fp32 as the reference's apply_rope computes them for fp32
// storage) and stored to q_rope[m, h, :] in fp32. Needs N = heads*(nope+rope),
// nope and rope multiples of 32, and no split-K.
struct GemmRopeEpilogue {
    void* q_nope;
    float* q_rope;
    const int64_t* positions;
    int64_t sq, heads, nope, rope;
    float inv_freq[64];
};

// C[z][m][n] = sum_k A[z][m][k] * B[z][k][n], accumulated in fp32 on the tensor
// cores (kind::tf32 for fp32 operands, kind::f16 for bf16 / fp16).
//   A : 3-D tensor, element (k, y, m) at k + y*a_ld[0] + m*a_ld[1] with dims
//       {K, Ay, M}; y is the batch.
//   B : MN-major {N, K, Bz}: element (n, k, z) at n + k*b_ld[0] + z*b_ld[1]
//       (a row-major [K][N] weight), or K-major {K, N, Bz}: (k, n, z) at
//       k + n*b_ld[0] + z*b_ld[1] (a row-major [N][K] weight).
//   Z launches = batches x spb: launch z works on batch z / spb and on K slice
//       z % spb (k_chunk elements, a multiple of the K block; spb = 1: all of K).
//   C : element (m, n) of launch z at c + m*c_ldm + z*c_ldz + n, stored as fp32
//       or as the storage dtype (c_is_t).
//   split3 (fp32 only): 3xTF32 — each operand is split into a tf32 head and an
//       fp32 remainder and A*B is accumulated as hi*hi + hi*lo + lo*hi, which
//       keeps products to about 2^-21 relative (fp32-class accuracy) at a third
//       of the tf32 rate.
struct TcGemm {
    const void* A; int64_t a_dims[3]; int64_t a_ld[2];
    const void* B; bool b_mn; int64_t b_dims[3]; int64_t b_ld[2];
    int64_t M, N, K;
    int Z; int spb; int64_t k_chunk;
    void* C; bool c_is_t; int64_t c_ldm, c_ldz;
    int bn;          // 128 or 256 output columns per CTA (192: persistent form only)
    bool split3;
    // optional second operand pair, accumulated after A*B: C += A2*B2 over K2
    // (same layouts and boxes as A / B; spb must be 1)
    const void* A2; int64_t a2_dims[3]; int64_t a2_ld[2];
    const void* B2; int64_t b2_dims[3]; int64_t b2_ld[2];
    int64_t K2;
    // optional: rowmax[(z*M + m)*ntiles + tile] = max of row m over the tile's
    // columns n < n_valid (fp32 output; ntiles = ceil(N / bn))
    float* rowmax; int64_t n_valid;
    int* err;        // device error word (bounded waits)
    const GemmRopeEpilogue* rope_epi;   // optional (persistent form only); C is unused then
};

template <typename T> mla_status_t tc_gemm(const TcGemm& g, cudaStream_t st);

// K block of the GEMM (one 128-byte swizzle row of the operand dtype).
template <typename T> constexpr int tc_gemm_bk() { return 128 / int(sizeof(T)); }

}  // namespace mla
