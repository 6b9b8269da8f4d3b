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
//
// fp32 storage runs the same four steps with the three contractions on the
// tensor cores in 3xTF32 (fp32-class products, fp32 accumulation drained into a
// round-to-nearest sum every 64 K elements):
//   S    = q_absorbed @ c_kv^T, then S += q_rope @ pe^T      (per batch)
//   rows P = exp(S/scale - M) in place, l = sum P, M = max    (one warp per row)
//   ctx  = P @ c_kv split over keys, reduced and divided by l (per batch)
//   out  = ctx[:, h] @ W_uv[h]^T                               (per head)
#include "qprep.cuh"
#include "simt_gemm.cuh"
#include "tc_gemm.cuh"

#include <algorithm>
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

// ------------------------------------------------------------ fp32 on the tensor cores (3xTF32)
namespace {

// One warp per row: scaled, causally masked scores -> unnormalised probabilities
// in place, with the row max and the sum of the probabilities.
__global__ void __launch_bounds__(256) softmax_rows_kernel(
    float* __restrict__ S, float* __restrict__ row_max, float* __restrict__ row_sum,
    int64_t rows_total, int64_t ld, int64_t sk, int64_t sq, int64_t heads, float scale, int causal)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int64_t g = blockIdx.x * 8LL + warp; g < rows_total; g += int64_t(gridDim.x) * 8) {
        float* srow = S + g * ld;
        const int64_t q = (g / heads) % sq;
        const int64_t last_key = causal ? (sk - sq + q) : (sk - 1);
        const int64_t n = last_key + 1 < sk ? last_key + 1 : sk;     // keys that are visible
        float mx = neg_inf<float>();
        for (int64_t k = lane; k < n; k += 32) {
            const float v = srow[k] / scale;
            mx = v > mx ? v : mx;
        }
        for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        const bool none = !(mx > neg_inf<float>());                    // every key masked
        float l = 0.f;
        for (int64_t k = lane; k < sk; k += 32) {
            const float pk = (k < n && !none) ? fexp(srow[k] / scale - mx) : 0.f;
            srow[k] = pk;
            l += pk;
        }
        for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
        if (lane == 0) {
            row_max[g] = mx;
            row_sum[g] = l;
        }
    }
}

// Non-causal rows: the row max comes from the per-tile maxima the score GEMM
// wrote, so the scores are read once. One warp per row, 16-byte accesses.
__global__ void __launch_bounds__(256) softmax_rows_tilemax_kernel(
    float* __restrict__ S, const float* __restrict__ tile_max, int ntiles, float* __restrict__ row_max,
    float* __restrict__ row_sum, int64_t rows_total, int64_t ld, int64_t sk, float scale)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int64_t g = blockIdx.x * 8LL + warp; g < rows_total; g += int64_t(gridDim.x) * 8) {
        float mx = neg_inf<float>();
        for (int t = lane; t < ntiles; t += 32) mx = fmaxf(mx, tile_max[g * ntiles + t]);
        for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        mx = mx / scale;                      // max(S) / scale == max(S / scale) for scale > 0
        float4* srow = reinterpret_cast<float4*>(S + g * ld);
        float l = 0.f;
        for (int64_t c = lane; 4 * c < sk; c += 32) {
            float4 v = srow[c];
            const int64_t k = 4 * c;
            v.x = fexp(v.x / scale - mx);
            v.y = k + 1 < sk ? fexp(v.y / scale - mx) : 0.f;
            v.z = k + 2 < sk ? fexp(v.z / scale - mx) : 0.f;
            v.w = k + 3 < sk ? fexp(v.w / scale - mx) : 0.f;
            srow[c] = v;
            l += (v.x + v.y) + (v.z + v.w);
        }
        for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
        if (lane == 0) {
            row_max[g] = mx;
            row_sum[g] = l;
        }
    }
}

// ctx[g, :] = sum over key slices of the partial products / l[g]; lse[g] = M + log l.
// parts: [batch][slices][rows_b][R]; ctx: [rows_total][R] with g = b * rows_b + row.
__global__ void __launch_bounds__(256) ctx_reduce_kernel(
    const float* __restrict__ parts, const float* __restrict__ row_max, const float* __restrict__ row_sum,
    float* __restrict__ ctx, float* __restrict__ lse, int64_t rows_b, int64_t rows_total, int64_t R, int slices)
{
    const int64_t total4 = rows_total * R / 4;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total4; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t e = i * 4;
        const int64_t g = e / R, r = e % R;
        const int64_t b = g / rows_b, row = g % rows_b;
        const float l = row_sum[g];
        const float inv = l > 0.f ? 1.f / l : 0.f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int z = 0; z < slices; ++z) {
            const float4 v = *reinterpret_cast<const float4*>(parts + ((b * slices + z) * rows_b + row) * R + r);
            acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
        }
        acc.x *= inv; acc.y *= inv; acc.z *= inv; acc.w *= inv;
        *reinterpret_cast<float4*>(ctx + e) = acc;
        if (lse && r == 0) lse[g] = row_max[g] + logf(l);
    }
}

struct T3Plan {
    int64_t rows_b, rows_total, ld, chunk, ntiles;
    int slices;
    size_t off_S, off_tmax, off_max, off_sum, off_parts, off_ctx, total;
};

T3Plan make_t3plan(const AArgs& a) {
    T3Plan p{};
    p.rows_b = a.sq * a.heads;
    p.rows_total = a.batch * p.rows_b;
    p.ld = (a.sk + 31) / 32 * 32;
    // key slices of P @ c_kv (one CTA per SM): the slice count in 1..8 whose CTAs fill
    // their last wave best, at least 8 K blocks per slice
    const int64_t tiles = ceil_div(p.rows_b, 128) * ceil_div(a.kv_rank, 128) * a.batch;
    const int64_t kblocks = ceil_div(a.sk, 32);
    const int64_t sms = sm_count();
    int64_t s = 1;
    double best = 0.0;
    for (int64_t c = 1; c <= 8 && c <= kblocks / 8; ++c) {
        if (c * a.batch > 65535) break;
        const int64_t ctas = tiles * c;
        const double fill = double(ctas) / double(ceil_div(ctas, sms) * sms);
        if (fill > best + 0.02) { best = fill; s = c; }
    }
    const int64_t cb = ceil_div(kblocks, s);
    p.chunk = cb * 32;
    p.slices = int(ceil_div(kblocks, cb));
    size_t off = 0;
    p.off_S = off;     off = align_up(off + size_t(p.rows_total) * p.ld * sizeof(float), 256);
    p.ntiles = ceil_div(p.ld, 128);
    p.off_tmax = off;  off = align_up(off + size_t(p.rows_total) * p.ntiles * sizeof(float), 256);
    p.off_max = off;   off = align_up(off + size_t(p.rows_total) * sizeof(float), 256);
    p.off_sum = off;   off = align_up(off + size_t(p.rows_total) * sizeof(float), 256);
    p.off_parts = off; off = align_up(off + size_t(p.slices) * p.rows_total * a.kv_rank * sizeof(float), 256);
    p.off_ctx = off;   off = align_up(off + size_t(p.rows_total) * a.kv_rank * sizeof(float), 256);
    p.total = off;
    return p;
}

// TMA needs 16-byte strides and the GEMM 32-column tiles of the latent.
bool t3_supported(const AArgs& a) {
    return a.kv_rank % 32 == 0 && a.rope % 4 == 0 && a.rope > 0 && a.sk > 0 && a.batch > 0 && a.sq > 0 &&
           a.heads > 0 && a.batch * a.sq * a.heads * a.sk < (int64_t(1) << 31);
}

mla_status_t attn_exact_t3(const AArgs& a, cudaStream_t st) {
    const T3Plan p = make_t3plan(a);
    char* ws = static_cast<char*>(a.workspace);
    DeviceStatus* dst = nullptr;
    MLA_TRY(device_status_block(&dst));
    int* err = &dst->code;
    float* S = reinterpret_cast<float*>(ws + p.off_S);
    float* rmax = reinterpret_cast<float*>(ws + p.off_max);
    float* rsum = reinterpret_cast<float*>(ws + p.off_sum);
    float* parts = reinterpret_cast<float*>(ws + p.off_parts);
    float* ctx = reinterpret_cast<float*>(ws + p.off_ctx);

    // S[b] = q_absorbed[b] [rows_b, R] @ c_kv[b]^T + q_rope[b] @ pe[b]^T in one GEMM (the
    // rope pair is a second K phase); keys past sk read as zeros (TMA fill) and land
    // in the padding columns [sk, ld)
    TcGemm g1{};
    g1.A = a.q_absorbed; g1.a_dims[0] = a.kv_rank; g1.a_dims[1] = a.batch; g1.a_dims[2] = p.rows_b;
    g1.a_ld[0] = p.rows_b * a.kv_rank; g1.a_ld[1] = a.kv_rank;
    g1.B = a.c_kv; g1.b_mn = false; g1.b_dims[0] = a.kv_rank; g1.b_dims[1] = a.sk; g1.b_dims[2] = a.batch;
    g1.b_ld[0] = a.kv_rank; g1.b_ld[1] = a.sk * a.kv_rank;
    g1.A2 = a.q_rope; g1.a2_dims[0] = a.rope; g1.a2_dims[1] = a.batch; g1.a2_dims[2] = p.rows_b;
    g1.a2_ld[0] = p.rows_b * a.rope; g1.a2_ld[1] = a.rope;
    g1.B2 = a.pe_cache; g1.b2_dims[0] = a.rope; g1.b2_dims[1] = a.sk; g1.b2_dims[2] = a.batch;
    g1.b2_ld[0] = a.rope; g1.b2_ld[1] = a.sk * a.rope; g1.K2 = a.rope;
    g1.M = p.rows_b; g1.N = p.ld; g1.K = a.kv_rank; g1.Z = int(a.batch); g1.spb = 1; g1.k_chunk = a.kv_rank;
    g1.C = S; g1.c_ldm = p.ld; g1.c_ldz = p.rows_b * p.ld; g1.bn = 128; g1.split3 = true; g1.err = err;
    float* tmax = reinterpret_cast<float*>(ws + p.off_tmax);
    if (!a.causal) {   // per-tile row maxima for the one-pass softmax
        g1.rowmax = tmax;
        g1.n_valid = a.sk;
    }
    MLA_TRY(tc_gemm<float>(g1, st));

    {
        int64_t blocks = ceil_div(p.rows_total, 8);
        if (blocks > 16LL * sm_count()) blocks = 16LL * sm_count();
        if (!a.causal)
            softmax_rows_tilemax_kernel<<<unsigned(blocks), 256, 0, st>>>(S, tmax, int(p.ntiles), rmax, rsum,
                                                                          p.rows_total, p.ld, a.sk, float(a.scale));
        else
            softmax_rows_kernel<<<unsigned(blocks), 256, 0, st>>>(S, rmax, rsum, p.rows_total, p.ld, a.sk, a.sq,
                                                                  a.heads, float(a.scale), a.causal);
        MLA_TRY(check_launch("attention softmax rows"));
    }

    TcGemm g3{};      // parts[b][z] = P[b][:, keys of slice z] @ c_kv[b][keys of slice z, :]
    g3.A = S; g3.a_dims[0] = a.sk; g3.a_dims[1] = a.batch; g3.a_dims[2] = p.rows_b;
    g3.a_ld[0] = p.rows_b * p.ld; g3.a_ld[1] = p.ld;
    g3.B = a.c_kv; g3.b_mn = true; g3.b_dims[0] = a.kv_rank; g3.b_dims[1] = a.sk; g3.b_dims[2] = a.batch;
    g3.b_ld[0] = a.kv_rank; g3.b_ld[1] = a.sk * a.kv_rank;
    g3.M = p.rows_b; g3.N = a.kv_rank; g3.K = a.sk; g3.Z = int(a.batch) * p.slices; g3.spb = p.slices;
    g3.k_chunk = p.chunk;
    g3.C = parts; g3.c_ldm = a.kv_rank; g3.c_ldz = p.rows_b * a.kv_rank; g3.bn = 128; g3.split3 = true; g3.err = err;
    MLA_TRY(tc_gemm<float>(g3, st));

    {
        int64_t blocks = ceil_div(p.rows_total * a.kv_rank / 4, 256);
        if (blocks > 32LL * sm_count()) blocks = 32LL * sm_count();
        ctx_reduce_kernel<<<unsigned(blocks), 256, 0, st>>>(parts, rmax, rsum, ctx, a.lse, p.rows_b, p.rows_total,
                                                            a.kv_rank, p.slices);
        MLA_TRY(check_launch("attention context reduce"));
    }
    if (a.v_dim % 32 != 0) return attn_out_normalized<float>(a, ctx, st);
    TcGemm g4{};      // out[:, h] = ctx[:, h] @ W_uv[h]^T
    const int64_t groups = a.batch * a.sq;
    g4.A = ctx; g4.a_dims[0] = a.kv_rank; g4.a_dims[1] = a.heads; g4.a_dims[2] = groups;
    g4.a_ld[0] = a.kv_rank; g4.a_ld[1] = a.heads * a.kv_rank;
    g4.B = a.W_uv; g4.b_mn = false; g4.b_dims[0] = a.kv_rank; g4.b_dims[1] = a.v_dim; g4.b_dims[2] = a.heads;
    g4.b_ld[0] = a.kv_rank; g4.b_ld[1] = a.v_dim * a.kv_rank;
    g4.M = groups; g4.N = a.v_dim; g4.K = a.kv_rank; g4.Z = int(a.heads); g4.spb = 1; g4.k_chunk = a.kv_rank;
    g4.C = a.out; g4.c_is_t = true; g4.c_ldm = a.heads * a.v_dim; g4.c_ldz = a.v_dim; g4.bn = 128;
    g4.split3 = true; g4.err = err;
    return tc_gemm<float>(g4, st);
}

}  // namespace

// Problems past the tensor-core path's 2^31 score limit (long prefill) run it per
// sequence and per block of queries. Under causal masking a query block
// [q0, q1) needs only the keys its last query sees, Sk - (Sq - q1), so each block
// is an ordinary smaller problem on the same cache rows.
struct T3Chunks {
    int64_t rows;   // queries per call
    bool on;
};
T3Chunks t3_chunks(const AArgs& a) {
    T3Chunks c{0, false};
    if (t3_supported(a)) return c;
    AArgs one = a;
    one.batch = 1;
    one.sq = 1;
    if (!t3_supported(one)) return c;
    const int64_t fit = ((int64_t(1) << 31) - 1) / (a.heads * a.sk);   // queries per call under the limit
    const int64_t n = ceil_div(a.sq, fit);
    c.rows = ceil_div(a.sq, n);
    c.on = true;
    return c;
}
AArgs t3_chunk_args(const AArgs& a, int64_t b, int64_t q0, int64_t rows) {
    AArgs c = a;
    const int64_t q1 = q0 + rows;
    c.batch = 1;
    c.sq = rows;
    c.sk = a.causal ? a.sk - (a.sq - q1) : a.sk;
    const int64_t row0 = b * a.sq + q0;   // first (sequence, query) row of the block
    const size_t es = sizeof(float);
    c.q_absorbed = static_cast<const char*>(a.q_absorbed) + size_t(row0 * a.heads * a.kv_rank) * es;
    c.q_rope = static_cast<const char*>(a.q_rope) + size_t(row0 * a.heads * a.rope) * es;
    c.c_kv = static_cast<const char*>(a.c_kv) + size_t(b * a.sk * a.kv_rank) * es;
    c.pe_cache = static_cast<const char*>(a.pe_cache) + size_t(b * a.sk * a.rope) * es;
    c.out = static_cast<char*>(a.out) + size_t(row0 * a.heads * a.v_dim) * es;
    c.lse = a.lse ? a.lse + row0 * a.heads : nullptr;
    return c;
}

template <typename T>
size_t attn_exact_workspace(const AArgs& a) {
    if (std::is_same<T, float>::value && t3_supported(a)) return make_t3plan(a).total;
    if (std::is_same<T, float>::value) {
        const T3Chunks ch = t3_chunks(a);
        if (ch.on) {
            AArgs c = a;
            c.batch = 1;
            c.sq = ch.rows;
            return make_t3plan(c).total;   // the largest block (all keys)
        }
    }
    return make_plan<T>(a).total;
}

template <typename T>
mla_status_t attn_exact(const AArgs& a, cudaStream_t st) {
    using Acc = acc_t<T>;
    if (std::is_same<T, float>::value && t3_supported(a)) return attn_exact_t3(a, st);
    if (std::is_same<T, float>::value) {
        const T3Chunks ch = t3_chunks(a);
        if (ch.on) {
            for (int64_t b = 0; b < a.batch; ++b)
                for (int64_t q0 = 0; q0 < a.sq; q0 += ch.rows)
                    MLA_TRY(attn_exact_t3(t3_chunk_args(a, b, q0, std::min(ch.rows, a.sq - q0)), st));
            return MLA_OK;
        }
    }
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
