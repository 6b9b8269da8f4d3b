// CUDA-core (FFMA / DFMA) tiled GEMM main loop used by the exact-arithmetic
// path (MLA_PREC_EXACT). A "problem" object supplies element loaders, so the
// same main loop serves every contraction of the MLA forward: the two Q
// projections, the W_uk absorption, the 576-deep score product, P @ c_kv and
// the W_uv up-projection. Operands are converted to the accumulate dtype as
// they are staged, so fp16/bf16 storage accumulates in fp32 and fp64 in fp64.
//
// Block shape: 256 threads, each owning a TM x TN register tile. Shared
// memory holds two buffers of A^T[BK][BM] and B[BK][BN] (rows padded by 4
// elements); the next K tile is fetched into registers while the current one
// is multiplied, so there is one __syncthreads per K tile. With TM = TN = 8 a
// thread's rows and columns are split into two runs of four at {4t, BM/2+4t},
// which keeps every vector shared-memory read of a warp conflict-free.
#pragma once

#include "common.cuh"

namespace mla {

template <typename AccT, int BM_, int BN_, int BK_, int TM_, int TN_>
struct SimtCfg {
    using Acc = AccT;
    static constexpr int BM = BM_, BN = BN_, BK = BK_, TM = TM_, TN = TN_;
    static constexpr int kThreads = 256;
    static constexpr int kTX = BN / TN;
    static constexpr int kTY = BM / TM;
    static_assert(kTX * kTY == kThreads, "tile must map onto 256 threads");
    static_assert((BM * BK) % kThreads == 0 && (BN * BK) % kThreads == 0, "staging");
    static constexpr int kAPer = BM * BK / kThreads;
    static constexpr int kBPer = BN * BK / kThreads;
    static constexpr int kAStride = BM + 4;
    static constexpr int kBStride = BN + 4;
    static constexpr size_t kSmemBytes = size_t(2) * BK * (kAStride + kBStride) * sizeof(Acc);

    // Row (m) of the tile held in accumulator row i of thread ty.
    __device__ static __forceinline__ int m_of(int ty, int i) {
        if constexpr (TM == 8) return (i < 4) ? ty * 4 + i : BM / 2 + ty * 4 + (i - 4);
        else return ty * TM + i;
    }
    __device__ static __forceinline__ int n_of(int tx, int j) {
        if constexpr (TN == 8) return (j < 4) ? tx * 4 + j : BN / 2 + tx * 4 + (j - 4);
        else return tx * TN + j;
    }
};

// Problem interface (duck-typed):
//   static constexpr bool kAKFast;   // A source is contiguous along k
//   static constexpr bool kBNFast;   // B source is contiguous along n
//   Acc a(int64_t m_local, int64_t k) const;   // 0 outside the problem
//   Acc b(int64_t k, int64_t n_local) const;   // 0 outside the problem
//   void on_a(int slot, int64_t m_local, Acc v); // optional observer (row sums)
template <class Cfg, class P>
__device__ __forceinline__ void simt_gemm_mainloop(
    const P& p, int64_t k_begin, int64_t k_end,
    typename Cfg::Acc (&acc)[Cfg::TM][Cfg::TN], typename Cfg::Acc* smem)
{
    using Acc = typename Cfg::Acc;
    constexpr int BM = Cfg::BM, BN = Cfg::BN, BK = Cfg::BK, TM = Cfg::TM, TN = Cfg::TN;
    const int tid = threadIdx.x;
    const int tx = tid % Cfg::kTX;
    const int ty = tid / Cfg::kTX;

    Acc* As = smem;                               // [2][BK][kAStride]
    Acc* Bs = smem + 2 * BK * Cfg::kAStride;      // [2][BK][kBStride]

#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = Acc(0);

    Acc ra[Cfg::kAPer], rb[Cfg::kBPer];

    auto a_coord = [&](int i, int& ml, int& kl) {
        const int e = tid + i * Cfg::kThreads;
        if constexpr (P::kAKFast) { kl = e % BK; ml = e / BK; }
        else { ml = e % BM; kl = e / BM; }
    };
    auto b_coord = [&](int i, int& kl, int& nl) {
        const int e = tid + i * Cfg::kThreads;
        if constexpr (P::kBNFast) { nl = e % BN; kl = e / BN; }
        else { kl = e % BK; nl = e / BK; }
    };
    auto fetch = [&](int64_t k0) {
#pragma unroll
        for (int i = 0; i < Cfg::kAPer; ++i) {
            int ml, kl; a_coord(i, ml, kl);
            const int64_t k = k0 + kl;
            ra[i] = (k < k_end) ? p.a(ml, k) : Acc(0);
        }
#pragma unroll
        for (int i = 0; i < Cfg::kBPer; ++i) {
            int kl, nl; b_coord(i, kl, nl);
            const int64_t k = k0 + kl;
            rb[i] = (k < k_end) ? p.b(k, nl) : Acc(0);
        }
    };
    auto stash = [&](int buf) {
        Acc* as = As + buf * BK * Cfg::kAStride;
        Acc* bs = Bs + buf * BK * Cfg::kBStride;
#pragma unroll
        for (int i = 0; i < Cfg::kAPer; ++i) {
            int ml, kl; a_coord(i, ml, kl);
            as[kl * Cfg::kAStride + ml] = ra[i];
        }
#pragma unroll
        for (int i = 0; i < Cfg::kBPer; ++i) {
            int kl, nl; b_coord(i, kl, nl);
            bs[kl * Cfg::kBStride + nl] = rb[i];
        }
    };

    const int64_t ntiles = (k_end > k_begin) ? (k_end - k_begin + BK - 1) / BK : 0;
    if (ntiles == 0) return;
    fetch(k_begin);
    stash(0);
    __syncthreads();
    for (int64_t t = 0; t < ntiles; ++t) {
        const int buf = int(t & 1);
        if (t + 1 < ntiles) fetch(k_begin + (t + 1) * BK);
        const Acc* as = As + buf * BK * Cfg::kAStride;
        const Acc* bs = Bs + buf * BK * Cfg::kBStride;
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            Acc av[TM], bv[TN];
#pragma unroll
            for (int i = 0; i < TM; ++i) av[i] = as[kk * Cfg::kAStride + Cfg::m_of(ty, i)];
#pragma unroll
            for (int j = 0; j < TN; ++j) bv[j] = bs[kk * Cfg::kBStride + Cfg::n_of(tx, j)];
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) acc[i][j] = fma(av[i], bv[j], acc[i][j]);
        }
        if (t + 1 < ntiles) stash(buf ^ 1);
        __syncthreads();
    }
}

// The common configurations: a 128x128 tile for row counts that fill it and a
// 16x128 tile for decode-sized row counts (B*Sq <= 16), where a tall tile
// would spend most of its FMAs on rows that do not exist.
template <typename Acc> using CfgBig = SimtCfg<Acc, 128, 128, 8, 8, 8>;
template <typename Acc> using CfgSmall = SimtCfg<Acc, 16, 128, 16, 1, 8>;

}  // namespace mla
