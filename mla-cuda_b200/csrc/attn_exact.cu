// Absorbed MLA attention in exact arithmetic (MLA_PREC_EXACT) on CUDA cores.
// Reference semantics: launch_mla_attention (mla_kernels.cu:1479-1682) and the
// PyTorch path mla_attention_official (exhaustive_benchmark_suite.py:289-304).
//
// A "row" is one (b, q, h) query; the Sq*H rows of batch b share that batch's
// c_kv / pe_cache. Four launches:
//
//   scores   S[row, k] = (q_absorbed[row] . c_kv[b,k] + q_rope[row] . pe[b,k]) / scale
//            one 576-deep contraction; also the max of each 128-key tile per row
//   rowmax   M[row] = max over tiles
//   pv       O_z[row, :] = sum_{k in split z} exp(S[row,k] - M[row]) * c_kv[b,k,:]
//            l_z[row]    = sum_{k in split z} exp(S[row,k] - M[row])
//   out      out[row, :] = (sum_z O_z[row, :] / sum_z l_z[row]) @ W_uv[h]^T
//
// This path is bound by CUDA-core FMA throughput, not by memory, so the scores
// are staged once in the accumulate dtype. Because the global row max is known
// before P @ c_kv runs, each probability is a single exp(S - M) with no
// rescaling of partial sums. Key splits of the P @ c_kv product are combined
// by plain sums in the last launch, which keeps the result deterministic.
#include "qprep.cuh"
#include "simt_gemm.cuh"

#include <type_traits>

namespace mla {
namespace {

template <typename T, typename Acc>
struct ScoreProblem {
    static constexpr bool kAKFast = true;
    static constexpr bool kBNFast = false;
    const T* qa; const T* qr; const T* ckv; const T* pe;
    int64_t rows_b, sk, R, D, bi, m0, n0;
    __device__ Acc a(int64_t ml, int64_t k) const {
        const int64_t row = m0 + ml;
        if (row >= rows_b) return Acc(0);
        const int64_t g = bi * rows_b + row;
        return (k < R) ? cvt<Acc>(qa[g * R + k]) : cvt<Acc>(qr[g * D + (k - R)]);
    }
    __device__ Acc b(int64_t k, int64_t nl) const {
        const int64_t n = n0 + nl;
        if (n >= sk) return Acc(0);
        const int64_t key = bi * sk + n;
        return (k < R) ? cvt<Acc>(ckv[key * R + k]) : cvt<Acc>(pe[key * D + (k - R)]);
    }
};

// grid = (key tiles, row tiles, batch)
template <class Cfg, typename T>
__global__ void __launch_bounds__(256) scores_kernel(
    const T* __restrict__ qa, const T* __restrict__ qr, const T* __restrict__ ckv,
    const T* __restrict__ pe, typename Cfg::Acc* __restrict__ S, typename Cfg::Acc* __restrict__ tile_max,
    int64_t rows_b, int64_t sq, int64_t heads, int64_t sk, int64_t R, int64_t D, int64_t ld,
    int64_t n_key_tiles, typename Cfg::Acc scale, int causal)
{
    using Acc = typename Cfg::Acc;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    ScoreProblem<T, Acc> p{qa, qr, ckv, pe, rows_b, sk, R, D, int64_t(blockIdx.z),
                           int64_t(blockIdx.y) * Cfg::BM, int64_t(blockIdx.x) * Cfg::BN};
    Acc acc[Cfg::TM][Cfg::TN];
    simt_gemm_mainloop<Cfg>(p, 0, R + D, acc, reinterpret_cast<Acc*>(smem_raw));

    const int tx = threadIdx.x % Cfg::kTX, ty = threadIdx.x / Cfg::kTX;
    static_assert(Cfg::kTX == 16, "tile-max reduction assumes 16 lanes per row group");
#pragma unroll
    for (int i = 0; i < Cfg::TM; ++i) {
        const int64_t row = p.m0 + Cfg::m_of(ty, i);
        const bool row_ok = row < rows_b;
        const int64_t g = p.bi * rows_b + row;
        // Causal: query q of sq sits at absolute key index sk - sq + q.
        const int64_t last_key = causal ? (sk - sq + row / heads) : (sk - 1);
        Acc mx = neg_inf<Acc>();
#pragma unroll
        for (int j = 0; j < Cfg::TN; ++j) {
            const int64_t n = p.n0 + Cfg::n_of(tx, j);
            if (!row_ok || n >= sk) continue;
            const Acc s = (n <= last_key) ? acc[i][j] / scale : neg_inf<Acc>();
            S[g * ld + n] = s;
            mx = s > mx ? s : mx;
        }
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) {
            const Acc o = __shfl_xor_sync(0xffffffffu, mx, off);
            mx = o > mx ? o : mx;
        }
        if (tx == 0 && row_ok) tile_max[g * n_key_tiles + blockIdx.x] = mx;
    }
}

template <typename Acc>
__global__ void __launch_bounds__(256) rowmax_kernel(
    const Acc* __restrict__ tile_max, Acc* __restrict__ row_max, int64_t rows, int64_t ntiles)
{
    for (int64_t r = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; r < rows;
         r += int64_t(gridDim.x) * blockDim.x) {
        Acc mx = neg_inf<Acc>();
        for (int64_t t = 0; t < ntiles; ++t) {
            const Acc v = tile_max[r * ntiles + t];
            mx = v > mx ? v : mx;
        }
        row_max[r] = mx;
    }
}

template <typename T, typename Acc>
struct PVProblem {
    static constexpr bool kAKFast = true;
    static constexpr bool kBNFast = true;
    const Acc* S; const Acc* mrow_s; const T* ckv;
    int64_t rows_b, sk, R, ld, bi, m0, n0;
    __device__ Acc a(int64_t ml, int64_t k) const {
        const int64_t row = m0 + ml;
        if (row >= rows_b) return Acc(0);
        return fexp(S[(bi * rows_b + row) * ld + k] - mrow_s[ml]);
    }
    __device__ Acc b(int64_t k, int64_t nl) const {
        const int64_t n = n0 + nl;
        return (n < R) ? cvt<Acc>(ckv[(bi * sk + k) * R + n]) : Acc(0);
    }
};

// grid = (latent tiles, row tiles, batch * splits)
template <class Cfg, typename T>
__global__ void __launch_bounds__(256) pv_kernel(
    const typename Cfg::Acc* __restrict__ S, const typename Cfg::Acc* __restrict__ row_max,
    const T* __restrict__ ckv, typename Cfg::Acc* __restrict__ O_part, typename Cfg::Acc* __restrict__ l_part,
    int64_t rows_b, int64_t rows_total, int64_t sk, int64_t R, int64_t ld, int splits, int64_t chunk)
{
    using Acc = typename Cfg::Acc;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ Acc mrow_s[Cfg::BM];
    const int64_t b = blockIdx.z / splits;
    const int z = int(blockIdx.z % splits);
    const int64_t m0 = int64_t(blockIdx.y) * Cfg::BM;
    for (int i = threadIdx.x; i < Cfg::BM; i += blockDim.x)
        mrow_s[i] = (m0 + i < rows_b) ? row_max[b * rows_b + m0 + i] : Acc(0);
    __syncthreads();

    PVProblem<T, Acc> p{S, mrow_s, ckv, rows_b, sk, R, ld, b, m0, int64_t(blockIdx.x) * Cfg::BN};
    const int64_t kb = int64_t(z) * chunk;
    const int64_t ke = (kb + chunk < sk) ? kb + chunk : sk;
    Acc acc[Cfg::TM][Cfg::TN];
    simt_gemm_mainloop<Cfg>(p, kb, ke, acc, reinterpret_cast<Acc*>(smem_raw));

    const int tx = threadIdx.x % Cfg::kTX, ty = threadIdx.x / Cfg::kTX;
#pragma unroll
    for (int i = 0; i < Cfg::TM; ++i) {
        const int64_t row = m0 + Cfg::m_of(ty, i);
        if (row >= rows_b) continue;
        Acc* o = O_part + (int64_t(z) * rows_total + b * rows_b + row) * R;
#pragma unroll
        for (int j = 0; j < Cfg::TN; ++j) {
            const int64_t n = p.n0 + Cfg::n_of(tx, j);
            if (n < R) o[n] = acc[i][j];
        }
    }
    // Softmax denominators of this split: one warp per row, first latent tile only.
    if (blockIdx.x == 0) {
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        for (int i = warp; i < Cfg::BM; i += Cfg::kThreads / 32) {
            const int64_t row = m0 + i;
            if (row >= rows_b) break;
            const Acc* srow = S + (b * rows_b + row) * ld;
            Acc l = Acc(0);
            for (int64_t k = kb + lane; k < ke; k += 32) l += fexp(srow[k] - mrow_s[i]);
            for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
            if (lane == 0) l_part[int64_t(z) * rows_total + b * rows_b + row] = l;
        }
    }
}

template <typename T, typename Acc>
struct OutProblem {
    static constexpr bool kAKFast = true;
    static constexpr bool kBNFast = false;
    const Acc* O_part; const Acc* inv_l_s; const T* W;
    int64_t M, heads, R, V, rows_total, h, m0, n0;
    int splits;
    __device__ Acc a(int64_t ml, int64_t k) const {
        const int64_t m = m0 + ml;
        if (m >= M) return Acc(0);
        const int64_t g = m * heads + h;
        Acc v = Acc(0);
        for (int z = 0; z < splits; ++z) v += O_part[(int64_t(z) * rows_total + g) * R + k];
        return v * inv_l_s[ml];
    }
    __device__ Acc b(int64_t k, int64_t nl) const {
        const int64_t n = n0 + nl;
        return (n < V) ? cvt<Acc>(W[(h * V + n) * R + k]) : Acc(0);
    }
};

// grid = (v tiles, (b,q) tiles, heads)
template <class Cfg, typename T>
__global__ void __launch_bounds__(256) out_kernel(
    const typename Cfg::Acc* __restrict__ O_part, const typename Cfg::Acc* __restrict__ l_part,
    const T* __restrict__ W_uv, T* __restrict__ out,
    int64_t M, int64_t heads, int64_t R, int64_t V, int64_t rows_total, int splits,
    const typename Cfg::Acc* __restrict__ row_max, float* __restrict__ lse)
{
    using Acc = typename Cfg::Acc;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ Acc inv_l_s[Cfg::BM];
    const int64_t h = blockIdx.z;
    const int64_t m0 = int64_t(blockIdx.y) * Cfg::BM;
    for (int i = threadIdx.x; i < Cfg::BM; i += blockDim.x) {
        Acc l = Acc(0);
        if (l_part == nullptr) {
            l = Acc(1);   // context already normalised
        } else if (m0 + i < M) {
            for (int z = 0; z < splits; ++z) l += l_part[int64_t(z) * rows_total + (m0 + i) * heads + h];
        }
        inv_l_s[i] = (l > Acc(0)) ? Acc(1) / l : Acc(0);
        // partial attention: log-sum-exp of the row's scaled scores
        if (lse && l_part && blockIdx.x == 0 && m0 + i < M) {
            const int64_t g = (m0 + i) * heads + h;
            lse[g] = float(row_max[g] + log(l));
        }
    }
    __syncthreads();
    OutProblem<T, Acc> p{O_part, inv_l_s, W_uv, M, heads, R, V, rows_total, h, m0,
                         int64_t(blockIdx.x) * Cfg::BN, splits};
    Acc acc[Cfg::TM][Cfg::TN];
    simt_gemm_mainloop<Cfg>(p, 0, R, acc, reinterpret_cast<Acc*>(smem_raw));
    const int tx = threadIdx.x % Cfg::kTX, ty = threadIdx.x / Cfg::kTX;
#pragma unroll
    for (int i = 0; i < Cfg::TM; ++i) {
        const int64_t m = m0 + Cfg::m_of(ty, i);
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < Cfg::TN; ++j) {
            const int64_t n = p.n0 + Cfg::n_of(tx, j);
            if (n < V) out[(m * heads + h) * V + n] = cvt<T>(acc[i][j]);
        }
    }
}

struct APlan {
    int64_t rows_b, rows_total, ld, n_key_tiles, chunk;
    int splits;
    bool small_rows;   // Sq*H <= 16: 16-row tiles for scores / pv
    bool small_out;    // B*Sq <= 16: 16-row tiles for the W_uv product
    size_t off_S, off_tmax, off_rmax, off_O, off_l, total;
};

template <typename T>
APlan make_plan(const AArgs& a) {
    using Acc = acc_t<T>;
    APlan p{};
    p.rows_b = a.sq * a.heads;
    p.rows_total = a.batch * p.rows_b;
    p.ld = (a.sk + 3) / 4 * 4;
    p.small_rows = p.rows_b <= 16;
    p.small_out = a.batch * a.sq <= 16;
    const int64_t bn = CfgBig<Acc>::BN;   // 128 keys per score tile in both configs
    p.n_key_tiles = ceil_div(a.sk, bn);
    const int64_t bm = p.small_rows ? 16 : 128;
    const int64_t ctas = ceil_div(a.kv_rank, 128) * ceil_div(p.rows_b, bm) * a.batch;
    const int64_t want = 4LL * 2 * sm_count();
    int64_t s = want / (ctas > 0 ? ctas : 1);
    const int64_t max_split = ceil_div(a.sk, 128);      // at least 128 keys per split
    if (s > max_split) s = max_split;
    if (s > 65535 / (a.batch > 0 ? a.batch : 1)) s = 65535 / (a.batch > 0 ? a.batch : 1);
    if (s < 1) s = 1;
    const int64_t bk = 16;
    int64_t chunk = ceil_div(ceil_div(a.sk, s), bk) * bk;
    if (chunk < bk) chunk = bk;
    p.chunk = chunk;
    p.splits = int(ceil_div(a.sk, chunk));
    if (p.splits < 1) p.splits = 1;
    size_t off = 0;
    p.off_S = off;    off = align_up(off + size_t(p.rows_total) * p.ld * sizeof(Acc), 256);
    p.off_tmax = off; off = align_up(off + size_t(p.rows_total) * p.n_key_tiles * sizeof(Acc), 256);
    p.off_rmax = off; off = align_up(off + size_t(p.rows_total) * sizeof(Acc), 256);
    p.off_O = off;    off = align_up(off + size_t(p.splits) * p.rows_total * a.kv_rank * sizeof(Acc), 256);
    p.off_l = off;    off = align_up(off + size_t(p.splits) * p.rows_total * sizeof(Acc), 256);
    p.total = off;
    return p;
}

template <class Cfg, typename Kern>
void set_smem(Kern kern) {
    if (Cfg::kSmemBytes > 48 * 1024)
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(Cfg::kSmemBytes));
}

template <class Cfg, typename T>
mla_status_t run_scores_pv(const AArgs& a, const APlan& p, typename Cfg::Acc* S, typename Cfg::Acc* tmax,
                           typename Cfg::Acc* rmax, typename Cfg::Acc* O, typename Cfg::Acc* l,
                           cudaStream_t st) {
    using Acc = typename Cfg::Acc;
    {
        auto kern = scores_kernel<Cfg, T>;
        set_smem<Cfg>(kern);
        dim3 grid(unsigned(ceil_div(a.sk, Cfg::BN)), unsigned(ceil_div(p.rows_b, Cfg::BM)), unsigned(a.batch));
        kern<<<grid, 256, Cfg::kSmemBytes, st>>>(
            static_cast<const T*>(a.q_absorbed), static_cast<const T*>(a.q_rope),
            static_cast<const T*>(a.c_kv), static_cast<const T*>(a.pe_cache), S, tmax,
            p.rows_b, a.sq, a.heads, a.sk, a.kv_rank, a.rope, p.ld, p.n_key_tiles, Acc(a.scale), a.causal);
        MLA_TRY(check_launch("attention scores"));
    }
    {
        int64_t blocks = ceil_div(p.rows_total, 256);
        if (blocks > 65535) blocks = 65535;
        rowmax_kernel<Acc><<<unsigned(blocks), 256, 0, st>>>(tmax, rmax, p.rows_total, p.n_key_tiles);
        MLA_TRY(check_launch("attention row max"));
    }
    {
        auto kern = pv_kernel<Cfg, T>;
        set_smem<Cfg>(kern);
        dim3 grid(unsigned(ceil_div(a.kv_rank, Cfg::BN)), unsigned(ceil_div(p.rows_b, Cfg::BM)),
                  unsigned(a.batch * p.splits));
        kern<<<grid, 256, Cfg::kSmemBytes, st>>>(S, rmax, static_cast<const T*>(a.c_kv), O, l, p.rows_b,
                                                 p.rows_total, a.sk, a.kv_rank, p.ld, p.splits, p.chunk);
        MLA_TRY(check_launch("attention P @ c_kv"));
    }
    return MLA_OK;
}

template <class Cfg, typename T>
mla_status_t run_out(const AArgs& a, const APlan& p, const typename Cfg::Acc* O, const typename Cfg::Acc* l,
                     cudaStream_t st, const typename Cfg::Acc* row_max = nullptr) {
    auto kern = out_kernel<Cfg, T>;
    set_smem<Cfg>(kern);
    const int64_t M = a.batch * a.sq;
    dim3 grid(unsigned(ceil_div(a.v_dim, Cfg::BN)), unsigned(ceil_div(M, Cfg::BM)), unsigned(a.heads));
    kern<<<grid, 256, Cfg::kSmemBytes, st>>>(O, l, static_cast<const T*>(a.W_uv), static_cast<T*>(a.out), M,
                                             a.heads, a.kv_rank, a.v_dim, p.rows_total, p.splits, row_max, a.lse);
    return check_launch("attention W_uv output");
}

}  // namespace

// Step 3d alone, from a context that is already normalised ([B*Sq*H, kv_rank]
// fp32); used after the tensor-core attention's segment combine.
template <typename T>
mla_status_t attn_out_normalized(const AArgs& a, const float* O, cudaStream_t st) {
    APlan p{};
    p.rows_total = a.batch * a.sq * a.heads;
    p.splits = 1;
    if constexpr (std::is_same<acc_t<T>, float>::value) {
        if (a.batch * a.sq <= 16) return run_out<CfgSmall<float>, T>(a, p, O, nullptr, st);
        return run_out<CfgBig<float>, T>(a, p, O, nullptr, st);
    } else {
        return set_error(MLA_ERR_UNSUPPORTED, "MLA: fp32 context with fp64 storage");
    }
}
template mla_status_t attn_out_normalized<float>(const AArgs&, const float*, cudaStream_t);
template mla_status_t attn_out_normalized<__half>(const AArgs&, const float*, cudaStream_t);
template mla_status_t attn_out_normalized<__nv_bfloat16>(const AArgs&, const float*, cudaStream_t);

template <typename T>
size_t attn_exact_workspace(const AArgs& a) { return make_plan<T>(a).total; }

template <typename T>
mla_status_t attn_exact(const AArgs& a, cudaStream_t st) {
    using Acc = acc_t<T>;
    const APlan p = make_plan<T>(a);
    char* ws = static_cast<char*>(a.workspace);
    Acc* S = reinterpret_cast<Acc*>(ws + p.off_S);
    Acc* tmax = reinterpret_cast<Acc*>(ws + p.off_tmax);
    Acc* rmax = reinterpret_cast<Acc*>(ws + p.off_rmax);
    Acc* O = reinterpret_cast<Acc*>(ws + p.off_O);
    Acc* l = reinterpret_cast<Acc*>(ws + p.off_l);
    if (p.small_rows) {
        MLA_TRY((run_scores_pv<CfgSmall<Acc>, T>(a, p, S, tmax, rmax, O, l, st)));
    } else {
        MLA_TRY((run_scores_pv<CfgBig<Acc>, T>(a, p, S, tmax, rmax, O, l, st)));
    }
    if (p.small_out) return run_out<CfgSmall<Acc>, T>(a, p, O, l, st, rmax);
    return run_out<CfgBig<Acc>, T>(a, p, O, l, st, rmax);
}

template size_t attn_exact_workspace<float>(const AArgs&);
template size_t attn_exact_workspace<double>(const AArgs&);
template size_t attn_exact_workspace<__half>(const AArgs&);
template size_t attn_exact_workspace<__nv_bfloat16>(const AArgs&);
template mla_status_t attn_exact<float>(const AArgs&, cudaStream_t);
template mla_status_t attn_exact<double>(const AArgs&, cudaStream_t);
template mla_status_t attn_exact<__half>(const AArgs&, cudaStream_t);
template mla_status_t attn_exact<__nv_bfloat16>(const AArgs&, cudaStream_t);

}  // namespace mla
